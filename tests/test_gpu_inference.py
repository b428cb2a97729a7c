"""Inference on the framework's kernels: KV-cache prefill and decode through the fused
kernels (RMSNorm, tcgen05 GEMMs with RoPE / SwiGLU / residual epilogues, decode attention with
the gate fused) against the fp32 torch oracle, the CUDA-graph decode step against the eager
one, and no library GEMM on the decode path."""
import numpy as np
import pytest
import torch

from gpu_utils import assert_close

pytestmark = pytest.mark.gpu


def _models(device):
    from hrm_text_b200.runtime.factory import arch_preset, build_model
    cfg = arch_preset("hrm", "L") | dict(vocab_size=256, max_seq_len=128, n_layers=2, hidden_size=256, num_heads=2)
    torch.manual_seed(0)
    gpu = build_model(cfg, device).to(torch.bfloat16).eval()
    cpu = build_model(cfg, "cpu").eval()
    cpu.load_state_dict({k: v.float().cpu() for k, v in gpu.state_dict().items()})
    return gpu, cpu


def test_cached_prefill_and_decode_match_oracle(cuda_device):
    from hrm_text_b200.inference.engine import _slot_view, decode_step, prefill
    from hrm_text_b200.models.common import oracle_mode
    gpu, cpu = _models(cuda_device)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, 256, 17), rng.integers(0, 256, 9)]
    steps = rng.integers(0, 256, (4, 2))
    caches = {"gpu": gpu.create_cache(max_batch_size=2, max_seq_len=64, dtype=torch.bfloat16, device=cuda_device),
              "cpu": cpu.create_cache(max_batch_size=2, max_seq_len=64, dtype=torch.float32, device="cpu")}
    with torch.inference_mode():
        for i, pr in enumerate(prompts):
            lg = prefill(gpu, None, torch.as_tensor(pr, device=cuda_device), _slot_view(caches["gpu"], i))
            with oracle_mode():
                lc = prefill(cpu, None, torch.as_tensor(pr), _slot_view(caches["cpu"], i))
            assert_close(lg.float().cpu(), lc, 5e-2, f"prefill logits {i}")
        lengths = torch.tensor([len(p) for p in prompts], dtype=torch.int32)
        for t in range(len(steps)):
            tok = torch.as_tensor(steps[t])
            lg = decode_step(gpu, None, tok.to(cuda_device), caches["gpu"], lengths.to(cuda_device))
            with oracle_mode():
                lc = decode_step(cpu, None, tok, caches["cpu"], lengths)
            assert_close(lg.float().cpu(), lc, 5e-2, f"decode logits step {t}")
            lengths += 1


def test_graphed_generation_equals_eager(cuda_device):
    from hrm_text_b200.inference.engine import generate_tokens
    gpu, _ = _models(cuda_device)
    rng = np.random.default_rng(2)
    prompts = [(i, rng.integers(0, 256, n)) for i, n in enumerate([5, 17, 9, 30])]
    runs = []
    for graph in (False, True):
        runs.append(dict(generate_tokens(gpu, None, iter(prompts), max_tokens=64, max_generation=8, batch_size=2,
                                         stop_token=-1, temp=0.0, device=cuda_device, use_cuda_graph=graph)))
    assert sorted(runs[0]) == [0, 1, 2, 3]
    for pid in runs[0]:
        assert runs[0][pid].tolist() == runs[1][pid].tolist(), pid
        assert runs[0][pid].size == 8


def test_decode_step_runs_no_library_gemm(cuda_device):
    from torch.profiler import ProfilerActivity, profile

    from hrm_text_b200.inference.engine import decode_step
    gpu, _ = _models(cuda_device)
    cache = gpu.create_cache(max_batch_size=4, max_seq_len=64, dtype=torch.bfloat16, device=cuda_device)
    tok = torch.zeros(4, dtype=torch.long, device=cuda_device)
    lengths = torch.full((4,), 3, dtype=torch.int32, device=cuda_device)
    with torch.inference_mode():
        decode_step(gpu, None, tok, cache, lengths)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            decode_step(gpu, None, tok, cache, lengths)
            torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    ours = [n for n in names if "hrm::" in n]
    library = [n for n in names if "hrm::" not in n and any(s in n.lower() for s in ("gemm", "nvjet", "xmma", "cutlass", "gemv"))]
    assert ours and not library, library[:5]
