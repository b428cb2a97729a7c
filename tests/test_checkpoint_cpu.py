"""DCP checkpoints: save/resume round trip (1 and 2 ranks) and the reference loader's view."""
import os
import sys
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hrm_text_b200.data.synthetic import packed_batches
from hrm_text_b200.runtime.checkpoint import load_checkpoint, save_checkpoint
from hrm_text_b200.runtime.engine import TrainEngine
from hrm_text_b200.runtime.factory import arch_preset, build_model

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def tiny_cfg():
    return arch_preset("hrm", "L") | dict(vocab_size=512, max_seq_len=256, n_layers=2, hidden_size=256, num_heads=2)


def _train(engine, steps=2, rank=0, world=1):
    for b, _ in packed_batches(256, 512, 256, rank=rank, world=world, num_batches=steps, median=64.0):
        engine.train_step(b, lr=1e-3, bp_steps=3)


def _full(engine, buf=None):
    return {s.fqn: engine.params.full_param_fp32(s, buf) for s in engine.params.slots}


def test_roundtrip_single_rank(tmp_path):
    torch.manual_seed(0)
    eng = TrainEngine(build_model(tiny_cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99)
    _train(eng)
    save_checkpoint(eng.params, eng.model, str(tmp_path), epoch=1, lr=1e-3)
    assert os.path.isdir(tmp_path / "fsdp2_epoch_1") and os.path.exists(tmp_path / "carry_epoch_1.0.pt")
    torch.manual_seed(1)
    eng2 = TrainEngine(build_model(tiny_cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99)
    assert load_checkpoint(eng2.params, eng2.model, str(tmp_path)) == 1
    for k, v in _full(eng).items():
        torch.testing.assert_close(_full(eng2)[k], v)
    torch.testing.assert_close(eng2.params.exp_avg_sq, eng.params.exp_avg_sq)
    torch.testing.assert_close(eng2.params.param_ema, eng.params.param_ema)
    assert eng2.params.step_count == eng.params.step_count == 2
    torch.testing.assert_close(eng2.model.model.zL_init, eng.model.model.zL_init)
    p = dict(eng2.model.named_parameters())["lm_head.weight"]
    torch.testing.assert_close(p, _full(eng)["lm_head.weight"])  # compute weights refreshed


def test_weights_only_from_ema(tmp_path):
    torch.manual_seed(0)
    eng = TrainEngine(build_model(tiny_cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.5)
    _train(eng)
    ema_full = _full(eng, eng.params.param_ema)
    save_checkpoint(eng.params, eng.model, str(tmp_path), epoch=3)
    eng2 = TrainEngine(build_model(tiny_cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.5)
    load_checkpoint(eng2.params, eng2.model, str(tmp_path), weights_only_from_ema=True)
    for k, v in ema_full.items():
        torch.testing.assert_close(_full(eng2)[k], v)
    assert eng2.params.step_count == 0 and float(eng2.params.exp_avg_sq.abs().max()) == 0.0


def _save_two_ranks(rank, world, path, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)  # identical init on both ranks
        eng = TrainEngine(build_model(tiny_cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99)
        _train(eng, rank=rank, world=world)
        full = _full(eng)
        save_checkpoint(eng.params, eng.model, path, epoch=2, rank=rank)
        if rank == 0:
            torch.save(full, os.path.join(path, "expected.pt"))
    finally:
        dist.destroy_process_group()


def test_two_rank_save_single_rank_load(tmp_path):
    mp.spawn(_save_two_ranks, args=(2, str(tmp_path), 29671), nprocs=2, join=True)
    expected = torch.load(tmp_path / "expected.pt")
    eng = TrainEngine(build_model(tiny_cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99)
    load_checkpoint(eng.params, eng.model, str(tmp_path), epoch=2)
    for k, v in expected.items():
        torch.testing.assert_close(_full(eng)[k], v)


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference source tree not present")
def test_reference_loader_reads_our_checkpoint(tmp_path):
    """The reference's own model + AdamATan2 + get_optimizer_state_dict load our checkpoint."""
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.state_dict import get_optimizer_state_dict
    torch.manual_seed(0)
    eng = TrainEngine(build_model(tiny_cfg()), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99)
    _train(eng)
    save_checkpoint(eng.params, eng.model, str(tmp_path), epoch=1, lr=1e-3)

    stub = types.ModuleType("flash_attn_interface")
    stub._flash_attn_backward = stub.maybe_contiguous = stub.flash_attn_with_kvcache = None
    saved = {k: sys.modules.get(k) for k in ("flash_attn_interface",)}
    sys.modules["flash_attn_interface"] = stub
    sys.path.insert(0, REF)
    try:
        for k in list(sys.modules):
            if k == "models" or k.startswith("models."):
                del sys.modules[k]
        from models.adam_atan2 import AdamATan2 as RefAdam
        from models.baselines.hrm_nocarry_bp_warmup import HierarchicalReasoningModel as RefHRM
        from models.lm_head import LMHead as RefHead
        cfg = tiny_cfg()
        ref = RefHead(RefHRM(cfg), cfg)
        opt = RefAdam(ref.parameters(), lr=torch.tensor(0.0), betas=(0.9, 0.95), weight_decay=0.1, ema=0.99)
        osd = get_optimizer_state_dict(ref, opt)
        dcp.load({"model": ref.state_dict(), "optim": osd}, checkpoint_id=str(tmp_path / "fsdp2_epoch_1"),
                 no_dist=True)
        ours = _full(eng)
        for name, p in ref.named_parameters():
            torch.testing.assert_close(p.detach(), ours[name])
        ema = _full(eng, eng.params.param_ema)
        assert set(osd["state"]) == set(ours)
        torch.testing.assert_close(osd["state"]["lm_head.weight"]["param_ema"], ema["lm_head.weight"])
        assert float(osd["state"]["lm_head.weight"]["step"]) == 2.0
    finally:
        sys.path.remove(REF)
        for k in list(sys.modules):
            if k == "models" or k.startswith("models."):
                del sys.modules[k]
        for k, v in saved.items():
            if v is not None:
                sys.modules[k] = v
            else:
                sys.modules.pop(k, None)
