"""Batches with repeated keys (unique_key=false) larger than one merge block
(GPU): a power-law key stream whose hot keys repeat across every block of
the duplicate merge, checked against the oracle, which takes the occurrences
one by one in input order as the reference's non-unique kernels do
(insert_or_assign_kernel.h:1044-1123, find_or_insert_kernel.h:336-425).
Scores merge per strategy: Lfu sums, EpochLfu sums the low 32 bits and
saturates, Customized keeps the last occurrence's score
(score_functor.h:157-160, :297-309, :431-455). The table never fills a
bucket here, so the result does not depend on thread order."""
import numpy as np
import pytest

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import GpuOps, make_table

pytestmark = pytest.mark.gpu

STRATS = {H.EvictStrategy.kLfu: O.LFU, H.EvictStrategy.kEpochLfu: O.EPOCH_LFU,
          H.EvictStrategy.kCustomized: O.CUSTOMIZED}
RESERVED = np.uint64(0xFFFFFFFFFFFFFFFC)


def power_law_batch(rng, universe, n, s=1.2):
    """ids in [0, universe) with P(id) ~ (id + 1)^-s: the top ids repeat
    thousands of times in a batch of n."""
    w = 1.0 / np.arange(1, universe + 1) ** s
    ids = rng.choice(universe, size=n, p=w / w.sum())
    return ids


def scores_for(strategy, rng, n):
    if strategy == H.EvictStrategy.kEpochLfu:
        # low words near 2^31: the hot keys' sums saturate at 2^32 - 1
        return rng.integers(1 << 30, 1 << 31, n).astype(np.uint64)
    if strategy == H.EvictStrategy.kLfu:
        return rng.integers(1, 1000, n).astype(np.uint64)
    return rng.permutation(np.arange(1, n + 1, dtype=np.uint64))


def live(state):
    keys, scores = state[0], state[1]
    m = keys < RESERVED
    return dict(zip(keys[m].tolist(), scores[m].tolist()))


@pytest.mark.parametrize("strategy", list(STRATS))
@pytest.mark.parametrize("op", ["find_or_insert", "insert_or_assign"])
def test_repeated_keys_across_merge_blocks(strategy, op):
    rng = np.random.default_rng(31 + strategy)
    dim, cap, universe, n = 4, 128 * 2048, 6000, 40000
    t = make_table(cap, dim=dim, strategy=strategy, epoch=7)
    o = O.OracleTable(cap, cap, dim=dim, strategy=STRATS[strategy])
    o.set_global_epoch(7)
    g = GpuOps(t, dim)
    key_of = np.unique(rng.integers(1, 1 << 62, 2 * universe, dtype=np.uint64))
    key_of = rng.permutation(key_of)[:universe]
    # half of the universe is resident before the batch
    pre = key_of[1::2]
    pv = rng.standard_normal((len(pre), dim)).astype(np.float32)
    ps = scores_for(strategy, rng, len(pre))
    g.insert_or_assign(pre, pv, ps)
    o.insert_or_assign(pre, pv, ps)
    keys = key_of[power_law_batch(rng, universe, n)]
    vals = rng.standard_normal((n, dim)).astype(np.float32)
    sc = scores_for(strategy, rng, n)
    if op == "find_or_insert":
        got = g.find_or_insert(keys, vals, sc, unique=False)
        ref, _ = o.find_or_insert(keys, vals, sc)
        np.testing.assert_array_equal(got, ref)
    else:
        g.insert_or_assign(keys, vals, sc, unique=False)
        o.insert_or_assign(keys, vals, sc)
    assert live(t.get_state()) == live(o.get_state())
    distinct = np.unique(keys)
    gv, gf, _ = g.find(distinct)
    rv, rf = o.find(distinct)[:2]
    assert gf.all() and rf.all()
    np.testing.assert_array_equal(gv, rv)
    # the hot keys did repeat across merge blocks of 1024 inputs
    assert np.bincount(np.searchsorted(np.sort(distinct), keys)).max() > 2000


@pytest.mark.parametrize("dim", [5, 33, 136])
def test_repeated_keys_rows_of_any_width(dim):
    """The merge's row copies at row widths that take each copy path: 20-byte
    rows (4-byte vectors, several rows per warp), 132-byte rows (33 vectors,
    a warp per row) and 544-byte rows (34 16-byte vectors, a warp per row);
    results against the oracle, as above."""
    rng = np.random.default_rng(500 + dim)
    cap, universe, n = 128 * 256, 3000, 12000
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kLfu)
    o = O.OracleTable(cap, cap, dim=dim, strategy=O.LFU)
    g = GpuOps(t, dim)
    key_of = rng.permutation(np.unique(rng.integers(1, 1 << 62, 2 * universe,
                                                    dtype=np.uint64)))[:universe]
    pre = key_of[1::2]
    pv = rng.standard_normal((len(pre), dim)).astype(np.float32)
    ps = rng.integers(1, 50, len(pre)).astype(np.uint64)
    g.insert_or_assign(pre, pv, ps)
    o.insert_or_assign(pre, pv, ps)
    keys = key_of[power_law_batch(rng, universe, n)]
    vals = rng.standard_normal((n, dim)).astype(np.float32)
    sc = rng.integers(1, 50, n).astype(np.uint64)
    got = g.find_or_insert(keys, vals, sc, unique=False)
    ref, _ = o.find_or_insert(keys, vals, sc)
    np.testing.assert_array_equal(got, ref)
    assert live(t.get_state()) == live(o.get_state())
    distinct = np.unique(keys)
    gv, gf, _ = g.find(distinct)
    rv, rf = o.find(distinct)[:2]
    assert gf.all() and rf.all()
    np.testing.assert_array_equal(gv, rv)
