"""Fused token sampling kernel: greedy equals torch.argmax; Gumbel-max sampling follows
softmax(logits / temp) (frequency test) and is reproducible for the same seed and offset."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_greedy_matches_argmax(dtype):
    from hrm_text_b200._native import cuda
    torch.manual_seed(0)
    logits = torch.randn(7, 32768, device="cuda").to(dtype)
    logits[3, 100] = logits[3, 200] = 50.0  # tie: the first index wins, as torch.argmax
    out = cuda().sample_tokens(logits, 0.0, 1, 1)
    assert torch.equal(out, logits.float().argmax(-1))


def test_gumbel_frequencies_and_reproducibility():
    from hrm_text_b200._native import cuda
    probs = torch.tensor([0.5, 0.25, 0.15, 0.1], device="cuda")
    temp = 0.7
    logits = (probs.log() * temp).repeat(20000, 1)  # softmax(logits / temp) == probs
    a = cuda().sample_tokens(logits, temp, 1234, 7)
    b = cuda().sample_tokens(logits, temp, 1234, 7)
    c = cuda().sample_tokens(logits, temp, 1234, 8)
    assert torch.equal(a, b) and not torch.equal(a, c)
    freq = torch.bincount(a, minlength=4).float() / a.numel()
    torch.testing.assert_close(freq, probs, atol=0.015, rtol=0)
