"""Host-side scheduling of the fused-collective copy jobs (hrm_text_b200.parallel.fused), on CPU.

The multi-GPU engine hands every GEMM launch at most one weight gather and one gradient push.
These tests drive that bookkeeping with the device launches replaced by a recorder:
* the first step records the first-use order and gathers each weight standalone at its use;
* from the second step on, the first weight is gathered at the start of the step and every
  other weight by the GEMM launched before its first use, in first-use order;
* a weight whose gather no GEMM carried before its use is gathered standalone there;
* pushes queued after a weight's last gradient ride on the next GEMM, and the ones left at
  the end of the backward run standalone.
"""
from collections import deque

import torch

from hrm_text_b200.parallel.fused import F1Info, F2Info, FusedCollectives, before_use


def _fake(names_f1, names_f2):
    fc = object.__new__(FusedCollectives)
    fc.counters = torch.zeros(4, dtype=torch.int32)
    fc.local_counts = torch.zeros(max(1, len(names_f2)), dtype=torch.int32)
    fc.f1 = {n: F1Info(n, None, None, 0, owner=fc) for n in names_f1}
    fc.f2 = {n: F2Info(n, None, 0, 0, 0, i, owner=fc) for i, n in enumerate(names_f2)}
    fc.order = None
    fc._recording = []
    fc._gather_queue = deque()
    fc._push_queue = deque()
    fc._gathered = set()
    fc._desc_cache = {}
    fc.log = []

    def run(g, p):
        if g is not None:
            fc._gathered.add(g.fqn)
        fc.log.append(("standalone", g and g.fqn, p and p.fqn))

    fc._run_standalone = run
    fc._descriptor = lambda g, p: (g and g.fqn, p and p.fqn)
    return fc


class _W:
    def __init__(self, info):
        self._f1 = info


def _gemm(fc):
    """One GEMM launch: it takes whatever jobs are queued."""
    jobs = fc.take_jobs()
    fc.log.append(("gemm", jobs))


def test_first_step_records_order_and_gathers_at_use():
    fc = _fake(["a", "b", "c"], [])
    fc.reset_step()
    for n in ("a", "b", "c"):
        before_use(_W(fc.f1[n]))
        _gemm(fc)
    fc.flush()
    assert [e for e in fc.log if e[0] == "standalone"] == [("standalone", n, None) for n in ("a", "b", "c")]
    assert [i.fqn for i in fc.order] == ["a", "b", "c"]
    # a second use in the same step gathers nothing
    fc.log.clear()
    before_use(_W(fc.f1["a"]))
    assert fc.log == []


def test_later_steps_gather_ahead_inside_gemms():
    fc = _fake(["a", "b", "c"], [])
    fc.reset_step()
    for n in ("a", "b", "c"):
        before_use(_W(fc.f1[n]))
        _gemm(fc)
    fc.flush()
    fc.log.clear()
    fc.reset_step()  # step 2: the first weight at the start of the step
    assert fc.log == [("standalone", "a", None)]
    fc.log.clear()
    for n in ("a", "b", "c"):
        before_use(_W(fc.f1[n]))
        _gemm(fc)
    # the GEMM of a carries b's gather, the GEMM of b carries c's; nothing runs standalone
    assert fc.log == [("gemm", ("b", None)), ("gemm", ("c", None)), ("gemm", None)]


def test_missing_carrier_falls_back_to_a_standalone_gather():
    fc = _fake(["a", "b", "c"], [])
    fc.reset_step()
    for n in ("a", "b", "c"):
        before_use(_W(fc.f1[n]))
        _gemm(fc)
    fc.flush()
    fc.reset_step()
    fc.log.clear()
    before_use(_W(fc.f1["a"]))
    before_use(_W(fc.f1["b"]))  # no GEMM launched in between: b is gathered here
    _gemm(fc)                   # ... and this GEMM carries c's gather instead
    before_use(_W(fc.f1["c"]))
    assert fc.log == [("standalone", "b", None), ("gemm", ("c", None))]


def test_pushes_ride_on_the_next_gemm_and_the_rest_are_flushed():
    fc = _fake([], ["p", "q", "r"])
    fc.reset_step()
    fc.queue_push(fc.f2["p"])
    _gemm(fc)
    fc.queue_push(fc.f2["q"])
    fc.queue_push(fc.f2["r"])
    _gemm(fc)
    fc.flush()
    assert fc.log == [("gemm", (None, "p")), ("gemm", (None, "q")), ("standalone", None, "r")]
    # a new step starts with an empty push queue and cleared counts
    fc.queue_push(fc.f2["p"])
    fc.counters.fill_(3)
    fc.reset_step()
    assert not fc._push_queue and int(fc.counters.sum()) == 0
