"""Checkpoints in the reference's on-disk layout (reference pretrain.py:227-293, 376-383).

Layout under ``checkpoint_path``:

* ``fsdp2_epoch_{e}/`` — a ``torch.distributed.checkpoint`` (DCP) directory holding
  ``{"model": <parameter FQNs + persistent buffers>, "optim": {"state": {fqn: {step, exp_avg,
  exp_avg_sq, param_ema}}, "param_groups": [...]}}`` — the structure that
  ``get_optimizer_state_dict`` produces for the reference's FSDP2 model, so the reference's
  ``inference_load_checkpoint`` and ``conversion/convert_to_hf.py`` read it unchanged;
* ``carry_epoch_{e}.{rank}.pt`` — the recurrent carry (``None`` for every shipped model);
* ``all_config.yaml`` / ``train_metadata.yaml`` — written once at the start of training.

The engine keeps each parameter's fp32 master weights and optimizer state as dim-0 shards;
they are saved as DTensor ``Shard(0)`` views (no gather) and loaded back in place, so a
checkpoint saved on N ranks can be resumed on M ranks (DCP re-shards on load).

``save_training_state``/``load_training_state`` additionally store the mid-epoch position
(step, epoch, batch index, RNG state) next to the DCP directory — an extension over the
reference, whose resume restarts at step 0 of epoch 1 (pretrain.py:353-359).
"""
from __future__ import annotations

import glob
import os
from pathlib import Path
from typing import Optional

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp

from .engine import ShardedParameters


def _mesh(params: ShardedParameters):
    from torch.distributed.device_mesh import init_device_mesh
    return init_device_mesh("cuda" if params.on_cuda else "cpu", (params.world,))


def _dist_tensor(params: ShardedParameters, buf: torch.Tensor, slot, mesh):
    """This rank's rows of one parameter (a view into a shard buffer), as a DTensor when sharded."""
    r0, r1 = slot.local_rows(params.rank)
    local = params.shard_view(buf, slot)[: r1 - r0].view((r1 - r0,) + tuple(slot.shape[1:]))
    if mesh is None:
        return local
    from torch.distributed.tensor import DTensor, Shard
    full_stride = torch.empty(slot.shape, device="meta").stride()
    return DTensor.from_local(local, mesh, [Shard(0)], run_check=False, shape=torch.Size(slot.shape),
                              stride=full_stride)


def _distributed(params: ShardedParameters) -> bool:
    return dist.is_initialized() and params.world > 1


def build_state_dict(params: ShardedParameters, model: torch.nn.Module, lr: float = 0.0) -> dict:
    mesh = _mesh(params) if _distributed(params) else None
    model_sd, optim_state = {}, {}
    step = torch.tensor(float(params.step_count), dtype=torch.float32)
    for s in params.slots:
        model_sd[s.fqn] = _dist_tensor(params, params.master, s, mesh)
        st = {"step": step.clone()}
        if params.exp_avg is not None:
            st["exp_avg"] = _dist_tensor(params, params.exp_avg, s, mesh)
        st["exp_avg_sq"] = _dist_tensor(params, params.exp_avg_sq, s, mesh)
        if params.param_ema is not None:
            st["param_ema"] = _dist_tensor(params, params.param_ema, s, mesh)
        optim_state[s.fqn] = st
    for name, buf in model.named_buffers():
        owner = model.get_submodule(name.rsplit(".", 1)[0]) if "." in name else model
        if name.rsplit(".", 1)[-1] in getattr(owner, "_non_persistent_buffers_set", set()):
            continue
        model_sd[name] = buf
    # lr is a 0-d CPU tensor, as in the reference's optimizer param group (pretrain.py:158-162)
    group = {"lr": torch.tensor(float(lr), dtype=torch.float32), "betas": (params.beta1, params.beta2),
             "weight_decay": params.weight_decay, "ema": params.ema, "params": [s.fqn for s in params.slots]}
    return {"model": model_sd, "optim": {"state": optim_state, "param_groups": [group]}}


def checkpoint_dir(path: str, epoch: int) -> str:
    return os.path.join(path, f"fsdp2_epoch_{epoch}")


def latest_epoch(path: str) -> Optional[int]:
    found = glob.glob(os.path.join(path, "fsdp2_epoch_*"))
    return max(int(Path(f).name.split("_")[-1]) for f in found) if found else None


def save_checkpoint(params: ShardedParameters, model, path: str, epoch: int, carry=None, lr: float = 0.0,
                    rank: int = 0) -> str:
    ckpt = checkpoint_dir(path, epoch)
    dcp.save(build_state_dict(params, model, lr), checkpoint_id=ckpt, no_dist=not _distributed(params))
    torch.save(carry, os.path.join(path, f"carry_epoch_{epoch}.{rank}.pt"))
    return ckpt


def load_checkpoint(params: ShardedParameters, model, path: str, epoch: Optional[int] = None,
                    betas: Optional[tuple] = None, weight_decay: Optional[float] = None, ema=None,
                    weights_only_from_ema: bool = False) -> int:
    """Load a checkpoint into the engine in place; returns the epoch loaded.

    Optimizer hyper-parameters come from the current run (the reference restores its
    config's betas / weight_decay / ema after loading, pretrain.py:254-260).
    ``weights_only_from_ema`` copies the EMA into the weights and resets the optimizer state
    (pretrain.py:262-265).
    """
    if epoch is None:
        epoch = latest_epoch(path)
        if epoch is None:
            raise FileNotFoundError(f"No checkpoint found in {path}")
    sd = build_state_dict(params, model)
    dcp.load(sd, checkpoint_id=checkpoint_dir(path, epoch), no_dist=not _distributed(params))
    steps = [st["step"] for st in sd["optim"]["state"].values()]
    params.step_count = int(steps[0].item()) if steps else 0
    if betas is not None:
        params.beta1, params.beta2 = betas
    if weight_decay is not None:
        params.weight_decay = weight_decay
    if ema is not None or params.param_ema is not None:
        params.ema = ema
    if weights_only_from_ema:
        if params.param_ema is not None:
            params.master.copy_(params.param_ema)
        reset_optimizer_state(params)
    params.refresh_compute()
    return epoch


def reset_optimizer_state(params: ShardedParameters) -> None:
    if params.exp_avg is not None:
        params.exp_avg.zero_()
    params.exp_avg_sq.zero_()
    if params.param_ema is not None:
        params.param_ema.copy_(params.master)
    params.step_count = 0


def save_training_state(path: str, epoch: int, state: dict, rank: int = 0) -> None:
    """Mid-epoch resume info (step counters, loader position, RNG) for rank ``rank``."""
    blob = dict(state)
    blob["torch_rng"] = torch.get_rng_state()
    if torch.cuda.is_available():
        blob["cuda_rng"] = torch.cuda.get_rng_state()
    torch.save(blob, os.path.join(path, f"train_state_epoch_{epoch}.{rank}.pt"))


def load_training_state(path: str, epoch: int, rank: int = 0) -> Optional[dict]:
    f = os.path.join(path, f"train_state_epoch_{epoch}.{rank}.pt")
    if not os.path.exists(f):
        return None
    blob = torch.load(f, weights_only=False)
    torch.set_rng_state(blob.pop("torch_rng"))
    cuda_rng = blob.pop("cuda_rng", None)
    if cuda_rng is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state(cuda_rng)
    return blob


def write_run_files(path: str, config_dump: dict, metadata_dump: dict, model_source: Optional[str] = None) -> None:
    """``all_config.yaml`` + ``train_metadata.yaml`` (+ a copy of the model source file)."""
    import shutil

    import yaml
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "all_config.yaml"), "w") as f:
        yaml.dump(config_dump, f)
    with open(os.path.join(path, "train_metadata.yaml"), "w") as f:
        yaml.dump(metadata_dump, f)
    if model_source is not None and os.path.exists(model_source):
        shutil.copy(model_source, os.path.join(path, os.path.basename(model_source)))


def read_run_files(path: str) -> tuple[dict, dict]:
    import yaml
    with open(os.path.join(path, "all_config.yaml")) as f:
        config = yaml.safe_load(f)
    with open(os.path.join(path, "train_metadata.yaml")) as f:
        metadata = yaml.safe_load(f)
    return config, metadata
