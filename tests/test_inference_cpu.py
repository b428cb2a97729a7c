"""KV-cache generation (prefill + decode) must equal greedy decoding by full recomputation."""
import numpy as np
import torch

from hrm_text_b200.inference.engine import generate_tokens
from hrm_text_b200.runtime.factory import arch_preset, build_model


def _model():
    cfg = arch_preset("hrm", "L") | dict(vocab_size=256, max_seq_len=128, n_layers=2, hidden_size=256, num_heads=2)
    torch.manual_seed(0)
    return build_model(cfg).eval()


def _greedy_recompute(model, prompt: np.ndarray, steps: int) -> list[int]:
    toks = list(prompt)
    P = len(prompt)
    out = []
    for _ in range(steps):
        T = len(toks)
        cu = torch.zeros(T + 1, dtype=torch.int32)
        cu[1] = T
        pl = torch.tensor([P] + [0] * (T - 1), dtype=torch.int32)
        batch = {"inputs": torch.tensor(toks, dtype=torch.int32), "position_ids": torch.arange(T, dtype=torch.int32),
                 "prefix_lens": pl, "cu_seqlens": cu}
        with torch.no_grad():
            logits = model(carry=None, batch=batch)[-1]
        nxt = int(logits[-1].argmax())
        out.append(nxt)
        toks.append(nxt)
    return out


def test_cached_generation_matches_recompute():
    model = _model()
    rng = np.random.default_rng(0)
    prompts = [(i, rng.integers(0, 256, n)) for i, n in enumerate([5, 17, 9])]
    got = dict(generate_tokens(model, None, iter(prompts), max_tokens=64, max_generation=6, batch_size=2,
                               stop_token=-1, temp=0.0, device=torch.device("cpu")))
    assert sorted(got) == [0, 1, 2]
    for pid, prompt in prompts:
        assert got[pid].tolist() == _greedy_recompute(model, prompt, len(got[pid])), pid


def test_too_long_prompt_yields_empty():
    model = _model()
    out = list(generate_tokens(model, None, iter([(7, np.arange(70) % 256)]), max_tokens=64, max_generation=4,
                               batch_size=1, stop_token=-1, device=torch.device("cpu")))
    assert out == [(7, out[0][1])] and out[0][1].size == 0
