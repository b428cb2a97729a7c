"""Model-FLOP accounting and the throughput meter used in the training log."""
import numpy as np
import torch

from hrm_text_b200.models.layers import prefixlm_allowed
from hrm_text_b200.runtime.factory import arch_preset, build_model
from hrm_text_b200.runtime.perf import ThroughputMeter, _attention_pairs, step_flops


def test_attention_pairs_match_the_mask():
    cu = np.array([0, 5, 9, 20, 0, 0], dtype=np.int32)
    pl = np.array([2, 4, 0, 0, 0], dtype=np.int32)
    want = sum(int(prefixlm_allowed(int(cu[i + 1] - cu[i]), int(pl[i])).sum()) for i in range(3))
    assert _attention_pairs(cu, pl, False) == want


def test_hrm_l_linear_flops_per_token():
    cfg = arch_preset("hrm", "L") | dict(vocab_size=32768, max_seq_len=4096)
    with torch.device("meta"):
        m = build_model(cfg, "meta")
    T = 1024
    batch = {"inputs": torch.zeros(T, dtype=torch.int32)}  # no packing: linear layers and head only
    per_token = step_flops(m, batch, {"bp_steps": 5}) / T
    stack = sum(p.numel() for p in m.model.L_level.parameters())
    assert per_token == (8 * 2 + 5 * 4) * stack + 6 * 32768 * 1280
    assert abs(per_token / 1e9 - 9.7) < 0.1  # 9.7 GF of linear-layer work per token for L at bp_steps = 5


def test_meter_reports_on_cpu():
    meter = ThroughputMeter(torch.device("cpu"), peak_tflops=1.0)
    meter.begin()
    for _ in range(3):
        meter.step(tokens_global=100, flops_local=1e9)
    out = meter.report()
    assert set(out) == {"perf/tokens_per_s", "perf/step_ms", "perf/tflops_per_gpu", "perf/mfu"}
    assert out["perf/tokens_per_s"] > 0 and out["perf/mfu"] > 0
