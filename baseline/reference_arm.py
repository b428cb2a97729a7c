"""``bench.py --impl reference``: the unmodified reference (``baseline/_ref``) on the same box.

What runs is the reference's own public API and stock code path (pretrain.py):
``create_dataloader`` (V1Dataset + numba multipack sampler over an on-disk synthetic dataset
in its format), ``create_model_and_carry`` (HRM + LMHead on CUDA, FSDP2 ``fully_shard`` per
TransformerBlock + root, AdamATan2) and the ``torch.compile``d ``train_batch`` (forward,
backward, optimizer step), called exactly as its training loop calls it
(pretrain.py:355-364). Nothing of the HRM-Text B200 framework is on this path.

Environment shims (none changes the reference's computation):
* ``hydra``, ``omegaconf`` and ``coolname`` are not installed; pretrain.py only needs them at
  import time (decorator, type names), so minimal stand-ins are registered;
* the image's default ``CXX`` wrapper (/opt/gcc/bin/g++) cannot link OpenMP, which Inductor's
  CPU kernels need (the reference's optimizer scalars live on the CPU); ``CXX`` is pointed at
  the system g++ for this process;
* FlashAttention-3 is sm_90a-only; ``baseline/fa3_standin/flash_attn_interface.py`` provides
  the three entry points the reference calls, on FlashAttention-2 kernels.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
import time
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def _unavailable(reason: str) -> None:
    print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def _install_import_shims() -> None:
    try:
        import hydra  # noqa: F401
    except ImportError:
        hydra = types.ModuleType("hydra")
        hydra.main = lambda **kw: (lambda fn: fn)
        sys.modules["hydra"] = hydra
    try:
        import omegaconf  # noqa: F401
    except ImportError:
        oc = types.ModuleType("omegaconf")
        oc.DictConfig = dict

        class OmegaConf:  # only referenced, never called on this path
            @staticmethod
            def to_container(cfg, resolve=True):
                return dict(cfg)
        oc.OmegaConf = OmegaConf
        sys.modules["omegaconf"] = oc
    try:
        import coolname  # noqa: F401
    except ImportError:
        cn = types.ModuleType("coolname")
        cn.generate_slug = lambda n=2: "bench-run"
        sys.modules["coolname"] = cn
    sys.path.insert(0, os.path.join(HERE, "fa3_standin"))
    sys.path.insert(0, REF)


def run_reference(args, metric, sizes, vocab, max_seq_len, clock_sampler_cls) -> None:
    if not os.path.isfile(os.path.join(REF, "pretrain.py")):
        _unavailable("baseline/_ref is missing (the reference has no packaging metadata; copy its source tree there)")
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    os.environ.setdefault("RANK", str(rank))
    os.environ.setdefault("WORLD_SIZE", str(world))
    os.environ.setdefault("WANDB_MODE", "disabled")
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"  # Inductor's CPU codegen needs an OpenMP-capable g++
    torch.cuda.set_device(local)
    from datetime import timedelta
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=1800))

    _install_import_shims()
    try:
        import pretrain as ref  # the reference's pretrain.py
        from models.common import wrap_tensor
    except Exception as exc:  # pragma: no cover
        _unavailable(f"importing the reference failed: {type(exc).__name__}: {exc}")
        return

    size = sizes[args.size]
    tokens_per_gpu = size["global_batch_8"] // 8
    global_batch = tokens_per_gpu * world
    lr = size["lr"]

    # On-disk synthetic dataset in the reference's format (same distribution as our arm).
    sys.path.insert(0, os.path.dirname(HERE))
    from hrm_text_b200.data.synthetic import write_dataset
    n_batches = args.warmup + args.steps
    num_docs = int(2.2 * n_batches * global_batch / 800) + 64
    data_dir = os.path.join(tempfile.gettempdir(), f"hrm_ref_bench_{args.size}_{world}_{os.getpid() if world == 1 else 0}")
    if rank == 0:
        write_dataset(data_dir, num_docs=num_docs, vocab=vocab, max_seq_len=max_seq_len, epochs=1, seed=1234)
    dist.barrier()

    overrides = {"arch": ref_arch(args.size), "data": {"path": data_dir}, "global_batch_size": global_batch,
                 "epochs": 1, "lr": lr, "lr_min_ratio": 1.0, "lr_warmup_steps": 0, "weight_decay": 0.1,
                 "beta1": 0.9, "beta2": 0.95, "ema": 0.9999}
    config = ref.PretrainConfig(**overrides)
    torch.random.manual_seed(config.seed + rank)
    train_state, train_loader, meta = ref.init_train(config, rank=rank, world_size=world)
    train_state.model.train()

    batches = []
    for batch, info in train_loader:
        batches.append((batch, info))
        if len(batches) >= n_batches:
            break
    if len(batches) < n_batches:
        _unavailable("synthetic dataset produced too few batches")
        return
    h2d = sum(v.numel() * v.element_size() for v in batches[0][0].values())

    def step(i):
        batch, info = batches[i % len(batches)]
        train_state.step += 1
        ref.update_lr(config, train_state)
        extra = {"bp_steps": 5}
        return ref.train_batch(train_state, batch | {k: wrap_tensor(torch.tensor(v, device="cpu"))
                                                     for k, v in info.items()}, **extra)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    clocks = clock_sampler_cls(local)
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    start.record()
    for i in range(args.steps):
        metrics = step(args.warmup + i)
    end.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    dist.barrier()
    t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    device_ms = float(t.item())

    e2e = None
    if not args.no_e2e:
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(args.steps):
            metrics = step(i)
            float(metrics["loss"][0].item())
        torch.cuda.synchronize()
        w = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device="cuda")
        dist.all_reduce(w, op=dist.ReduceOp.MAX)
        wall = float(w.item())
        e2e = {"value": global_batch * args.steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": 4, "ms_per_step": 1000.0 * wall / args.steps}

    if rank == 0:
        from flash_attn_interface import BACKEND
        line = {
            "metric": metric, "value": global_batch * args.steps / (device_ms / 1000.0), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": device_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic packed PrefixLM on disk in the reference format, reference V1Dataset + multipack",
            "config": {"model": f"HRM-Text {args.size}", "global_batch": global_batch, "seq_len": max_seq_len,
                       "tokens_per_gpu": tokens_per_gpu, "bp_steps": 5, "parallelism": f"fsdp2-dp{world}",
                       "attention_standin": f"flash_attn_interface stand-in on {BACKEND}",
                       "l2": "inputs larger than L2"},
            "clocks": clock_info, "e2e": e2e, "impl": "reference",
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


def ref_arch(size: str) -> dict:
    """The reference's arch config for net=hrm and the given size (read from its YAML files)."""
    import yaml
    arch = {}
    for path in (os.path.join(REF, "config", "arch", "net", "hrm.yaml"),
                 os.path.join(REF, "config", "arch", "size", f"{size}.yaml")):
        with open(path) as f:
            arch.update(yaml.safe_load(f))
    return arch
