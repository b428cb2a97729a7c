"""Failure detection on the host (no GPU is faulted, trapped or hung by any of these):

* a step that overruns its deadline is reported by the step watchdog;
* a rank that stops heart-beating is listed as stale by its peers;
* a rank that leaves the job makes the survivors' next collective fail (short process-group
  timeout) instead of hanging;
* a truncated checkpoint shard makes the load fail loudly.
"""
import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hrm_text_b200.runtime.watchdog import Heartbeat, StepWatchdog


def test_step_watchdog_fires_once_on_overrun():
    fired = []
    wd = StepWatchdog(0.2, on_timeout=lambda step, elapsed: fired.append((step, elapsed)), poll_s=0.02)
    try:
        with wd.step(1):
            time.sleep(0.05)       # within the deadline
        time.sleep(0.3)            # disarmed: nothing fires between steps
        assert fired == []
        with wd.step(2):
            time.sleep(0.6)        # overruns
        assert len(fired) == 1 and fired[0][0] == 2 and fired[0][1] > 0.2
    finally:
        wd.close()


def test_heartbeat_lists_silent_rank():
    store = dist.HashStore()
    hb0 = Heartbeat(store, rank=0, world=3, interval_s=0.05)
    hb1 = Heartbeat(store, rank=1, world=3, interval_s=0.05)
    try:
        time.sleep(0.2)
        assert hb0.stale_ranks(max_age_s=1.0) == [2]   # rank 2 never started
        hb1.stop()                                      # rank 1 goes silent
        time.sleep(0.6)
        assert hb0.stale_ranks(max_age_s=0.4) == [1, 2]
        assert hb0.last_beat(1) is not None
    finally:
        hb0.stop()
        hb1.stop()


def _peer_exit_worker(rank, world, port, out):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    x = torch.ones(4)
    dist.all_reduce(x)  # both ranks healthy
    if rank == 1:
        os._exit(0)    # leaves between steps, with no collective in flight
    t0 = time.monotonic()
    try:
        dist.all_reduce(x)
        result = "no error"
    except Exception as exc:  # the survivor must see an error, not hang
        result = f"error after {time.monotonic() - t0:.1f}s: {type(exc).__name__}"
    with open(out, "w") as f:
        f.write(result)
    os._exit(0)


def test_peer_exit_fails_next_collective(tmp_path):
    out = str(tmp_path / "rank0.txt")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_peer_exit_worker, args=(r, 2, 29631, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung after its peer left")
    text = open(out).read()
    assert text.startswith("error after"), text
    assert float(text.split()[2].rstrip("s:")) < 60


def test_truncated_checkpoint_fails_loudly(tmp_path):
    from hrm_text_b200.runtime.checkpoint import load_checkpoint, save_checkpoint
    from hrm_text_b200.runtime.engine import TrainEngine
    from hrm_text_b200.runtime.factory import arch_preset, build_model
    cfg = arch_preset("hrm", "L") | dict(vocab_size=512, max_seq_len=256, n_layers=2, hidden_size=256, num_heads=2)
    torch.manual_seed(0)
    eng = TrainEngine(build_model(cfg), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99)
    save_checkpoint(eng.params, eng.model, str(tmp_path), epoch=1)
    shard_dir = tmp_path / "fsdp2_epoch_1"
    shards = sorted(p for p in shard_dir.iterdir() if p.suffix == ".distcp")
    assert shards
    data = shards[0].read_bytes()
    shards[0].write_bytes(data[: len(data) // 3])
    eng2 = TrainEngine(build_model(cfg), beta1=0.9, beta2=0.95, weight_decay=0.1, ema=0.99)
    from torch.distributed.checkpoint.api import CheckpointException  # a BaseException subclass
    with pytest.raises((Exception, CheckpointException)):
        load_checkpoint(eng2.params, eng2.model, str(tmp_path))
