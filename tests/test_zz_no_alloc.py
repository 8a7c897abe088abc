"""hkv_find_or_insert_noalloc: find_or_insert without device allocation (GPU).

Some callers cannot allocate device memory while they serve lookups, for
example a service that gives all its GPU memory to a fixed arena at start-up.
For them the library offers a find_or_insert for batches that may repeat
keys whose scratch is one fixed device array instead of per-call
allocations. This test calls it through the C ABI and checks that two calls
in a row give exactly what the allocating entry point (hkv_find_or_insert
with unique_key=false) gives on a twin table, and what the CPU oracle's
find_or_insert (oracle/hkv_oracle.c, one key after another as the reference
processes a batch) gives: the same returned values and the same table
contents (every live key with its score and value, and every bucket's size;
integer and byte work, so the comparison is exact). Slot
positions inside a bucket are not compared: when several keys of a batch
land in one bucket, which of them takes which free slot depends on thread
timing in either entry point. It lives in its own file, collected last, and
passes alone or after the other tests.
"""
import numpy as np
import pytest
import torch

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import dev, host, make_table
from hkv_testutil import live_set

pytestmark = pytest.mark.gpu


def _batch(rng, distinct, repeats, dim):
    keys = rng.choice(distinct, repeats, replace=True).astype(np.uint64)
    vals = rng.standard_normal((repeats, dim)).astype(np.float32)
    scores = rng.integers(1, 50, repeats).astype(np.uint64)
    return keys, vals, scores


def test_noalloc_matches_allocating_entry_point_on_two_calls():
    rng = np.random.default_rng(4242)
    cap, dim = 128 * 512, 32
    ref = make_table(cap, dim=dim, strategy=H.EvictStrategy.kLfu)
    nal = make_table(cap, dim=dim, strategy=H.EvictStrategy.kLfu)
    ora = O.OracleTable(cap, cap, dim=dim, strategy=O.LFU)
    pool = np.unique(rng.integers(1, 1 << 62, 9000, dtype=np.uint64))
    for call in range(2):
        # call 0 inserts; call 1 mixes hits on call 0's keys with new keys
        distinct = pool[:6000] if call == 0 else pool[3000:9000]
        keys, vals, scores = _batch(rng, distinct, 15000, dim)
        out_ref = dev(vals)
        out_nal = dev(vals)
        ref.find_or_insert(len(keys), dev(keys), out_ref, dev(scores), unique_key=False)
        nal.find_or_insert_noalloc(len(keys), dev(keys), out_nal, dev(scores))
        torch.cuda.synchronize()
        assert torch.equal(out_ref, out_nal), f"returned values differ on call {call}"
        out_ora, _ = ora.find_or_insert(keys, vals, scores)
        assert (host(out_nal) == out_ora).all(), f"values differ from the oracle on call {call}"
        rk, rs, _, rz, rv = ref.get_state()
        nk, ns, _, nz, nv = nal.get_state()
        assert (rz == nz).all(), f"bucket sizes differ on call {call}"
        assert live_set(rk, rs, rv) == live_set(nk, ns, nv), \
            f"table contents differ on call {call}"
        ok, os_, _, oz, ov = ora.get_state()
        assert (oz == nz).all(), f"bucket sizes differ from the oracle on call {call}"
        assert live_set(ok, os_, ov) == live_set(nk, ns, nv), \
            f"table contents differ from the oracle on call {call}"
        nal.check_device_error()
    assert ref.size() == nal.size() > 0


def test_noalloc_rejects_batches_beyond_its_scratch():
    t = make_table(128 * 64, dim=32, strategy=H.EvictStrategy.kLfu)
    n = 16385
    keys = torch.arange(1, n + 1, dtype=torch.int64, device="cuda")
    vals = torch.zeros((n, 32), device="cuda")
    sc = torch.ones(n, dtype=torch.int64, device="cuda")
    with pytest.raises(H.HkvException):
        t.find_or_insert_noalloc(n, keys, vals, sc)
    assert t.size() == 0
    # rows are found or inserted in place, so any row width works
    wide = make_table(128 * 64, dim=256, strategy=H.EvictStrategy.kLfu)
    k4 = torch.tensor([5, 6, 5, 7], dtype=torch.int64, device="cuda")
    vals = torch.arange(4 * 256, dtype=torch.float32, device="cuda").reshape(4, 256)
    first = vals.clone()
    wide.find_or_insert_noalloc(4, k4, vals, sc[:4])
    torch.cuda.synchronize()
    assert wide.size() == 3
    # the repeated key reads back its first occurrence's row
    assert torch.equal(vals[2], first[0]) and torch.equal(vals[[0, 1, 3]], first[[0, 1, 3]])


def test_noalloc_refuses_a_batch_that_would_grow_the_table_and_takes_no_memory():
    """A table that can still grow: a batch that would trigger auto-grow fails
    (growing allocates) and leaves the capacity alone; calls that fit take no
    device memory (free device memory is the same before and after, once the
    first call has looked up the array's address)."""
    cap, dim = 128 * 64, 32
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kLfu, max_capacity=4 * cap)
    rng = np.random.default_rng(77)
    base = np.unique(rng.integers(1, 1 << 62, 4200, dtype=np.uint64))[:4000]
    k0, v0, s0 = dev(base), dev(rng.standard_normal((4000, dim)).astype(np.float32)), \
        dev(np.ones(4000, np.uint64))
    t.find_or_insert_noalloc(2000, k0[:2000], v0[:2000], s0[:2000])
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    t.find_or_insert_noalloc(1800, k0[2000:3800], v0[2000:3800], s0[2000:3800])
    t.find_or_insert_noalloc(200, k0[:200], v0[:200], s0[:200])  # hits (the load
    # factor check counts them as if new: 3800 + 200 of 8192 slots)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert t.size() == 3800 and t.capacity() == cap
    # 3800 / 8192 + 1000 / 8192 > max_load_factor 0.5: the reference would grow
    more = dev(np.unique(rng.integers(1 << 62, 1 << 63, 1100, dtype=np.uint64))[:1000])
    with pytest.raises(RuntimeError):
        t.find_or_insert_noalloc(1000, more, v0[:1000], s0[:1000])
    assert t.capacity() == cap and t.size() == 3800
    t.check_device_error()
