"""tcgen05 GEMM and its fused epilogues vs fp32 torch references."""
import pytest
import torch
import torch.nn.functional as F

from gpu_utils import assert_close

pytestmark = pytest.mark.gpu

# M >= 1024 runs the CTA-pair kernel (256-row tiles; 1300 leaves a partial pair tile); the
# last shape's weight gradient (K = 8192 tokens, 2048 x 2048) takes the K-chunk split-K path
SHAPES = [(256, 256, 128), (300, 512, 192), (1000, 1280, 1280), (128, 768, 64), (1300, 768, 512),
          (2048, 1280, 1280), (8192, 2048, 2048)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_fwd(cuda_device, M, N, K):
    from hrm_text_b200.ops import gemm as G
    torch.manual_seed(0)
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    w = torch.randn(N, K, device=cuda_device).bfloat16()
    ref = x.float() @ w.float().T
    assert_close(G.linear(x, w), ref, 1e-2, "fwd")
    r = torch.randn(M, N, device=cuda_device).bfloat16()
    assert_close(G.linear(x, w, residual=r), ref + r.float(), 1e-2, "fwd+residual")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_dgrad_wgrad(cuda_device, M, N, K):
    from hrm_text_b200.ops import gemm as G
    torch.manual_seed(1)
    dy = torch.randn(M, N, device=cuda_device).bfloat16()
    w = torch.randn(N, K, device=cuda_device).bfloat16()
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    assert_close(G.linear_dgrad(dy, w), dy.float() @ w.float(), 1e-2, "dgrad")
    grad = torch.full((N, K), 0.5, device=cuda_device)
    G.linear_wgrad_(dy, x, grad)
    assert_close(grad, 0.5 + dy.float().T @ x.float(), 1e-3, "wgrad accumulate")


@pytest.mark.parametrize("M", [384, 1300])
def test_linear_rope(cuda_device, M):
    from hrm_text_b200.models.layers import apply_rotary_pos_emb, rope_tables
    from hrm_text_b200.ops import gemm as G
    torch.manual_seed(2)
    H, K = 2, 256
    N = 4 * H * 128
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    w = torch.randn(N, K, device=cuda_device).bfloat16()
    pos = torch.randint(0, 1000, (M,), device=cuda_device, dtype=torch.int32)
    cos, sin = rope_tables(128, 1024, 10000.0, device=cuda_device)
    out = G.linear_rope(x, w, pos, cos[:, :64].contiguous(), sin[:, :64].contiguous(), H * 128, 3 * H * 128)
    ref = (x.float() @ w.float().T).view(M, 4 * H, 128)
    cs = (cos[pos.long()], sin[pos.long()])
    ref[:, H:3 * H] = apply_rotary_pos_emb(ref[:, H:3 * H], cs)
    assert_close(out, ref.view(M, N), 1e-2, "rope epilogue")


@pytest.mark.parametrize("M", [300, 1500])
def test_linear_swiglu_fwd_bwd(cuda_device, M):
    from hrm_text_b200.ops import gemm as G
    torch.manual_seed(3)
    K, I = 256, 384
    x = torch.randn(M, K, device=cuda_device).bfloat16()
    w = (torch.randn(2 * I, K, device=cuda_device) / 16).bfloat16()
    gu, h = G.linear_swiglu(x, w)
    gu_ref = x.float() @ w.float().T
    assert_close(gu, gu_ref, 1e-2, "gate|up")
    g, u = gu_ref.bfloat16().float().chunk(2, -1)
    assert_close(h, F.silu(g) * u, 2e-2, "silu*up")
    wd = torch.randn(512, I, device=cuda_device).bfloat16()
    dy = torch.randn(M, 512, device=cuda_device).bfloat16()
    dgu = G.linear_dgrad_swiglu(dy, wd, gu)
    gr = g.clone().requires_grad_(True)
    ur = u.clone().requires_grad_(True)
    (F.silu(gr) * ur).backward((dy.float() @ wd.float()).bfloat16().float())
    assert_close(dgu, torch.cat([gr.grad, ur.grad], -1), 2e-2, "swiglu bwd")


@pytest.mark.parametrize("T,H,V,chunk", [(500, 256, 2048, 8192), (1200, 256, 2048, 512), (2048, 1280, 32768, 8192)])
def test_lm_head_cross_entropy(cuda_device, T, H, V, chunk):
    """Chunked LM head + CE (no [T, V] logits stored) against fp32 F.cross_entropy, with
    ragged ignored labels (every 7th row and a block of 37 rows)."""
    from hrm_text_b200.ops.loss import lm_head_cross_entropy
    torch.manual_seed(4)
    x = torch.randn(T, H, device=cuda_device).bfloat16().requires_grad_(True)
    w = (torch.randn(V, H, device=cuda_device) / (H ** 0.5)).bfloat16().requires_grad_(True)
    labels = torch.randint(0, V, (T,), device=cuda_device, dtype=torch.int32)
    labels[::7] = -100
    labels[100:137] = -100
    loss, correct = lm_head_cross_entropy(x, w, labels, chunk=chunk)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    logits = (xr @ wr.T).bfloat16().float()
    ref = F.cross_entropy(logits, labels.long(), ignore_index=-100, reduction="sum")
    assert abs(loss.item() - ref.item()) <= 2e-3 * abs(ref.item())
    valid = labels >= 0
    ref_correct = (logits.argmax(-1) == labels.long()) & valid
    assert (correct == ref_correct).float().mean().item() > 0.995
    (loss * 0.01).backward()
    (ref * 0.01).backward()
    assert_close(x.grad, xr.grad, 3e-2, "d hidden")
    assert_close(w.grad, wr.grad, 3e-2, "d weight")


@pytest.mark.parametrize("M", [1, 7, 32, 128])
def test_decode_linear_epilogues(cuda_device, M):
    """Decode-step linear layers (split-K tcgen05 GEMM + epilogue kernel) against fp32 torch."""
    from hrm_text_b200.models.layers import rope_tables
    from hrm_text_b200.ops import gemm as G
    torch.manual_seed(7)
    H, hidden, inter = 2, 256, 1536
    x = torch.randn(M, hidden, device=cuda_device).bfloat16()
    w = (torch.randn(4 * hidden, hidden, device=cuda_device) / 16).bfloat16()
    ref = (x.float() @ w.float().T).bfloat16().float()
    r = torch.randn(M, 4 * hidden, device=cuda_device).bfloat16()
    assert_close(G.infer_linear(x, w), ref, 1e-2, "store")
    assert_close(G.infer_linear(x, w, residual=r), ref + r.float(), 1e-2, "residual")
    cos, sin = rope_tables(128, 64, 10000.0, device=cuda_device)
    pos = torch.randint(0, 64, (M,), device=cuda_device, dtype=torch.int32)
    out = G.infer_linear_rope(x, w, pos, cos[:, :64].contiguous(), sin[:, :64].contiguous(), hidden, 3 * hidden)
    heads = ref.view(M, 4 * H, 128)
    c, s = cos[pos.long()][:, None], sin[pos.long()][:, None]
    rot = torch.cat([-heads[..., 64:], heads[..., :64]], -1)
    want = heads.clone()
    want[:, H:3 * H] = heads[:, H:3 * H] * c + rot[:, H:3 * H] * s
    assert_close(out, want.view(M, -1), 1e-2, "rope")
    wg = (torch.randn(2 * inter, hidden, device=cuda_device) / 16).bfloat16()
    gu = (x.float() @ wg.float().T).bfloat16().float()
    g, u = gu[:, :inter], gu[:, inter:]
    assert_close(G.infer_swiglu(x, wg), torch.nn.functional.silu(g) * u, 2e-2, "swiglu")
    wd = (torch.randn(hidden, inter, device=cuda_device) / 40).bfloat16()  # long K: many split-K units
    h = torch.randn(M, inter, device=cuda_device).bfloat16()
    assert_close(G.infer_linear(h, wd), h.float() @ wd.float().T, 1e-2, "long K")
