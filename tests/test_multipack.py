import numpy as np
import pytest

from hrm_text_b200._native import host
from hrm_text_b200.data.multipack import (MultipackDistributedBatchSampler, allocate_py, lpt_check_py,
                                          lpt_with_result_py)


@pytest.mark.parametrize("seed", range(5))
def test_lpt_primitives_match_python(seed):
    rng = np.random.default_rng(seed)
    a = rng.integers(1, 500, size=int(rng.integers(1, 80))).astype(np.int64)
    a[: len(a) // 3] = a[0]  # force ties
    for n in (1, 2, 3, 8):
        for c in (300, 1000, 5000):
            assert host().lpt_check(a, c, n) == lpt_check_py(a, c, n)
        for r in range(n):
            np.testing.assert_array_equal(host().lpt_with_result(a, n, r), lpt_with_result_py(a, n, r))


@pytest.mark.parametrize("n,c", [(1, 2048), (2, 2048), (8, 21504), (3, 777)])
def test_allocate_matches_python(n, c):
    rng = np.random.default_rng(n * 131 + c)
    lengths = np.clip(rng.lognormal(np.log(300), 1.0, 400), 16, c).astype(np.int64)
    start = 0
    while start < lengths.size:
        for r in range(n):
            got = host().allocate(lengths, start, r, c, n)
            want = allocate_py(lengths, start, r, c, n)
            assert got[0] == want[0] and got[1] == want[1] and got[3] == want[3]
            np.testing.assert_array_equal(got[2], want[2])
        start += got[1]


def test_sampler_partitions_every_step():
    rng = np.random.default_rng(0)
    lengths = np.clip(rng.lognormal(np.log(512), 1.0, 2000), 16, 4096).astype(np.int64)
    n, c = 4, 8192
    plans = [list(MultipackDistributedBatchSampler(c, lengths, n, r, drop_last_batch=True).iter()) for r in range(n)]
    assert len({len(p) for p in plans}) == 1 and len(plans[0]) > 10
    for step in range(len(plans[0])):
        idx = np.concatenate([plans[r][step] for r in range(n)])
        assert len(set(idx.tolist())) == idx.size  # disjoint
        for r in range(n):
            assert lengths[plans[r][step]].sum() <= c  # fits
    s = MultipackDistributedBatchSampler(c, lengths, n, 0, drop_last_batch=True)
    list(s.iter())
    assert 0.9 < s.efficiency() <= 1.0
