import pytest
import torch

from hrm_text_b200.models.baselines.hrm_nocarry_bp_warmup import bp_steps_schedule, split_bp_steps
from hrm_text_b200.models.layers import prefixlm_allowed, prefixlm_attention_reference
from hrm_text_b200.runtime.factory import arch_preset, build_model


def test_reference_fqns_and_counts():
    cfg = arch_preset("hrm", "L") | dict(vocab_size=32768, max_seq_len=4096)
    with torch.device("meta"):
        m = build_model(cfg, "meta")
    names = [n for n, _ in m.named_parameters()]
    assert "embed_tokens.embedding_weight" in names and "lm_head.weight" in names
    assert "model.H_level.core.layers.11.attn.gqkv_proj.weight" in names
    assert "model.L_level.core.layers.0.mlp.down_proj.weight" in names
    assert "model.zL_init" in dict(m.named_buffers())
    total = sum(p.numel() for p in m.parameters())
    assert abs(total / 1e9 - 0.61) < 0.01
    shapes = dict(m.named_parameters())
    assert shapes["model.H_level.core.layers.0.attn.gqkv_proj.weight"].shape == (5120, 1280)
    assert shapes["model.H_level.core.layers.0.mlp.gate_up_proj.weight"].shape == (7168, 1280)


def test_xl_size():
    cfg = arch_preset("hrm", "XL") | dict(vocab_size=32768, max_seq_len=4096)
    m = build_model(cfg, "meta")
    assert abs(sum(p.numel() for p in m.parameters()) / 1e9 - 1.08) < 0.01


def test_bp_split_and_schedule():
    assert split_bp_steps(5, 2) == (2, 3)
    assert split_bp_steps(2, 2) == (1, 1)
    assert bp_steps_schedule(0, 1000, 0.2, 2, 5) == 2
    assert bp_steps_schedule(100, 1000, 0.2, 2, 5) == 3
    assert bp_steps_schedule(200, 1000, 0.2, 2, 5) == 5
    assert bp_steps_schedule(5, 1000, 0.0, 2, 5) == 5


def test_call_plan_matches_recurrence():
    cfg = arch_preset("hrm", "L") | dict(vocab_size=512, max_seq_len=64, n_layers=2, hidden_size=256, num_heads=2)
    m = build_model(cfg).model
    plan = m.call_plan(5)
    assert [c.state for c in plan] == ["L", "L", "L", "H", "L", "L", "L", "H"]
    assert [c.inject for c in plan] == ["H", "H", "H", "L", "H", "H", "H", "L"]
    assert [c.grad for c in plan] == [False, False, False, True, True, True, True, True]
    assert [c.slot for c in plan][:4] == [("L", 0), ("L", 1), ("L", 2), ("H", 0)]
    assert [c.grad for c in m.call_plan(2)] == [False] * 6 + [True, True]


def test_prefixlm_mask():
    m = prefixlm_allowed(5, 2)
    want = torch.tensor([[1, 1, 0, 0, 0], [1, 1, 0, 0, 0], [1, 1, 1, 0, 0], [1, 1, 1, 1, 0], [1, 1, 1, 1, 1]]).bool()
    assert torch.equal(m, want)
    assert torch.equal(prefixlm_allowed(3, 3), torch.ones(3, 3).bool())


def test_attention_oracle_no_cross_doc_and_zero_padding():
    torch.manual_seed(0)
    T, H, D = 20, 2, 8
    q, k, v = (torch.randn(T, H, D) for _ in range(3))
    cu = torch.tensor([0, 6, 15, 0, 0], dtype=torch.int32)
    pl = torch.tensor([2, 0, 0, 0], dtype=torch.int32)
    out = prefixlm_attention_reference(q, k, v, False, pl, cu)
    assert out[15:].abs().max() == 0
    v2 = v.clone()
    v2[6:15] += 10.0  # second document's values must not affect the first
    out2 = prefixlm_attention_reference(q, k, v2, False, pl, cu)
    torch.testing.assert_close(out[:6], out2[:6])


@pytest.mark.parametrize("net", ["hrm", "rins", "transformer", "trm", "trm_match_recurrence", "ut"])
def test_every_family_trains_on_cpu(net):
    from hrm_text_b200.data.synthetic import packed_batches
    from hrm_text_b200.runtime.engine import TrainEngine
    cfg = arch_preset(net, "L") | dict(vocab_size=512, max_seq_len=256, n_layers=2, hidden_size=256, num_heads=2)
    torch.manual_seed(0)
    m = build_model(cfg)
    eng = TrainEngine(m, beta1=0.9, beta2=0.95, weight_decay=0.1, ema=None)
    batch, _ = next(iter(packed_batches(256, 512, 256, num_batches=1, median=64.0)))
    extra = {"bp_steps": 3} if net == "hrm" else {}
    loss, metrics = eng.train_step(batch, lr=1e-3, **extra)
    assert torch.isfinite(loss)
    assert metrics["loss"][1] > 0


def test_family_call_plans_and_cache_layouts():
    base = dict(vocab_size=512, max_seq_len=64, n_layers=2, hidden_size=256, num_heads=2)
    trm = build_model(arch_preset("trm_match_recurrence", "L") | base).model
    plan = trm.call_plan()
    assert {c.stack for c in plan} == {"L_level"}
    assert [c.state for c in plan] == ["L", "L", "L", "H"] * 2
    assert [c.grad for c in plan] == [False, False, False, True, True, True, True, True]

    rins = build_model(arch_preset("rins", "L") | base).model
    plan = rins.call_plan()
    assert [c.stack for c in plan] == ["L_level"] * 7 + ["H_level"]
    assert [c.grad for c in plan] == [False] * 3 + [True] * 5
    assert plan[-1].inject is None and rins.output_state == "L"

    ut = build_model(arch_preset("ut", "L") | base).model
    assert [(c.slot, c.grad) for c in ut.call_plan()] == [((0,), False), ((1,), False), ((2,), True), ((3,), True)]

    kw = dict(max_batch_size=1, max_seq_len=8, device="cpu", dtype=torch.float32)
    hrm = build_model(arch_preset("hrm", "L") | base).model
    cache = hrm.create_cache(**kw)
    assert sorted(cache) == ["H", "L"] and len(cache["H"]) == 2 and len(cache["L"]) == 6
    cache = rins.create_cache(**kw)
    assert len(cache["L"]) == 7 and isinstance(cache["L"][0], list) and not isinstance(cache["H"][0], list)
    assert isinstance(ut.create_cache(**kw), list) and len(ut.create_cache(**kw)) == 4
