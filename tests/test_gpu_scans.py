"""erase_if / export_batch_if / size_if with the built-in predicate (GPU).

Reference: hkv_hashtable.h:2409-2476 (erase_if; remove_kernel.h:114-203: a
matching live slot becomes a RECLAIM tombstone with score 0 and its bucket's
size drops), :2623-2731 (export_batch_if: the matching live slots of
[offset, offset + n), counter set), :2829-2846 (size_if). The expected
results are the same predicates applied to the table's raw state on the
host.
"""
import numpy as np
import pytest
import torch

import hkv_b200 as H
from hkv_gpu import GpuOps, host, make_table
from hkv_testutil import live_set

pytestmark = pytest.mark.gpu
RES = np.uint64(0xFFFFFFFFFFFFFFFC)


def _table(rng, dim=4, cap=128 * 64):
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kCustomized)
    keys = np.unique(rng.integers(1, 1 << 62, 7000, dtype=np.uint64))[:6000]
    GpuOps(t, dim).insert_or_assign(keys, rng.standard_normal((len(keys), dim)).astype(np.float32),
                                    rng.integers(1, 10000, len(keys)).astype(np.uint64))
    return t


def _match(keys, scores, mask, value, cmp, thr):
    live = keys < RES
    m = live & ((keys & np.uint64(mask)) == np.uint64(value))
    ops = {None: lambda s: np.ones_like(s, bool), "<": lambda s: s < thr, "<=": lambda s: s <= thr,
           ">": lambda s: s > thr, ">=": lambda s: s >= thr, "==": lambda s: s == thr}
    return m & ops[cmp](scores)


CASES = [(0, 0, ">=", 5000), (0x3, 0x1, None, 0), (0x1, 0x1, ">", 7000), (0xF0, 0x30, "<", 3000)]


@pytest.mark.parametrize("mask,value,cmp,thr", CASES)
def test_size_and_export_if(mask, value, cmp, thr):
    rng = np.random.default_rng(31)
    t = _table(rng)
    keys, scores, _, _, vals = t.get_state()
    want = _match(keys, scores, mask, value, cmp, np.uint64(thr))
    pred = H.predicate(mask, value, cmp, thr)
    d = torch.zeros(1, dtype=torch.int64, device="cuda")
    t.size_if(pred, d)
    assert int(d.item()) == int(want.sum())
    cap = t.capacity()
    # export in two windows; the union is the matching set
    got = {}
    for off, n in ((0, cap // 3), (cap // 3, cap)):
        ek = torch.zeros(cap, dtype=torch.int64, device="cuda")
        ev = torch.zeros((cap, 4), device="cuda")
        es = torch.zeros(cap, dtype=torch.int64, device="cuda")
        t.export_batch_if(pred, n, off, d, ek, ev, es)
        c = int(d.item())
        sub = slice(off, min(off + n, cap))
        assert c == int(want[sub].sum())
        got.update(live_set(host(ek, np.uint64)[:c], host(es, np.uint64)[:c], host(ev)[:c]))
    assert got == live_set(keys[want], scores[want], vals[want])


def test_erase_if_tombstones():
    rng = np.random.default_rng(32)
    t = _table(rng)
    keys, scores, dig, sizes, vals = t.get_state()
    want = _match(keys, scores, 0x1, 0x1, "<", np.uint64(4000))
    n = t.erase_if(H.predicate(0x1, 0x1, "<", 4000))
    assert n == int(want.sum())
    k2, s2, d2, z2, v2 = t.get_state()
    assert (k2[want] == np.uint64(0xFFFFFFFFFFFFFFFE)).all() and (s2[want] == 0).all()
    assert (d2[want] == d2[want][0]).all()  # the reclaim digest
    keep = ~want
    assert (k2[keep] == keys[keep]).all() and (s2[keep] == scores[keep]).all()
    per_bucket = want.reshape(-1, 128).sum(axis=1)
    assert (z2 == sizes - per_bucket).all()
    assert t.size() == int((keys < RES).sum()) - n
    # erased keys are gone, the others still found
    f = GpuOps(t, 4).contains(keys[keys < RES])
    assert (f == keep[keys < RES]).all()
