"""KV-cache attention kernels vs the fp32 torch reference of the same op."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cache(B, S, H, dev):
    from hrm_text_b200.models.layers import Cache
    return Cache(torch.randn(B, S, H, 128, device=dev).bfloat16(), torch.randn(B, S, H, 128, device=dev).bfloat16())


@pytest.mark.parametrize("B,H,S", [(3, 4, 700), (1, 10, 64), (16, 2, 4096)])
def test_decode_matches_reference(B, H, S):
    from hrm_text_b200.models.layers import Cache, cached_attention_reference
    from hrm_text_b200.ops.decode import kv_decode
    torch.manual_seed(0)
    dev = torch.device("cuda")
    c1 = _cache(B, S, H, dev)
    c2 = Cache(c1.keys.clone(), c1.values.clone())
    lengths = torch.randint(0, S - 1, (B,), device=dev)
    lengths[0] = 0                     # first token of a sequence
    q, k, v = (torch.randn(B, 1, H, 128, device=dev).bfloat16() for _ in range(3))
    out = kv_decode(q, k, v, c1, lengths)
    ref = cached_attention_reference(q, k, v, c2, lengths, is_causal=True)
    torch.testing.assert_close(c1.keys, c2.keys)
    torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("causal", [False, True])
def test_prefill_matches_reference(causal):
    from hrm_text_b200.models.layers import Cache, cached_attention_reference
    from hrm_text_b200.ops.decode import kv_prefill
    torch.manual_seed(1)
    dev = torch.device("cuda")
    H, L, S = 4, 300, 512
    c1 = _cache(1, S, H, dev)
    c2 = Cache(c1.keys.clone(), c1.values.clone())
    q, k, v = (torch.randn(1, L, H, 128, device=dev).bfloat16() for _ in range(3))
    out = kv_prefill(q, k, v, c1, causal)
    ref = cached_attention_reference(q, k, v, c2, 0, is_causal=causal)
    torch.testing.assert_close(c1.values, c2.values)
    torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=2e-2)
