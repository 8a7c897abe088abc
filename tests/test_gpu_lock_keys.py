"""lock_keys / unlock_keys and find_or_insert* with locked_key_ptrs (GPU).

Reference: HashTable::lock_keys / unlock_keys (hkv_hashtable.h:1744-1806,
lock_keys_kernel.h, unlock_keys_kernel.h) and the expectations of
tests/test_lock_unlock_keys.cpp: present keys lock with a non-null key-word
address and succeed, absent keys get null and fail, unlock succeeds once.
Also the properties documented at hkv_lock_keys: a locked key is not found
by lookups or inserts, its slot is never an eviction victim, and the table
cannot grow while keys are locked.
"""
import numpy as np
import pytest
import torch

import hkv_b200 as H
from hkv_gpu import GpuOps, dev, host, make_table
from hkv_testutil import keys_for_bucket, random_keys

pytestmark = pytest.mark.gpu

USER_LOCK = np.uint64(0xFFFFFFFFFFFFFFFC)


def word_at(ptr):
    from cuda.bindings import runtime as rt
    out = np.zeros(1, np.uint64)
    (err,) = rt.cudaMemcpy(out.ctypes.data, int(ptr), 8, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess
    return out[0]


def write_row(ptr, row):
    from cuda.bindings import runtime as rt
    row = np.ascontiguousarray(row, np.float32)
    (err,) = rt.cudaMemcpy(int(ptr), row.ctypes.data, row.nbytes,
                           rt.cudaMemcpyKind.cudaMemcpyHostToDevice)
    assert err == rt.cudaError_t.cudaSuccess


def lock(t, keys, scores=None):
    n = len(keys)
    ptrs = torch.zeros(max(n, 1), dtype=torch.int64, device="cuda")
    ok = torch.zeros(max(n, 1), dtype=torch.bool, device="cuda")
    t.lock_keys(n, dev(keys), ptrs, ok, scores=None if scores is None else dev(scores))
    torch.cuda.synchronize()
    return ptrs, host(ptrs)[:n], host(ok)[:n].astype(bool)


def unlock(t, ptrs, keys):
    n = len(keys)
    ok = torch.zeros(max(n, 1), dtype=torch.bool, device="cuda")
    t.unlock_keys(n, ptrs, dev(keys), ok)
    torch.cuda.synchronize()
    return host(ok)[:n].astype(bool)


def test_lock_unlock_existing_absent_and_partial():
    rng = np.random.default_rng(71)
    dim = 4
    t = make_table(128 * 64, dim=dim, strategy=H.EvictStrategy.kLru)
    g = GpuOps(t, dim)
    keys = random_keys(rng, 500)
    vals = rng.standard_normal((500, dim)).astype(np.float32)
    g.insert_or_assign(keys, vals)
    absent = np.setdiff1d(random_keys(rng, 150), keys)[:100]
    batch = np.concatenate([keys[:200], absent])
    dptrs, ptrs, ok = lock(t, batch)
    assert ok[:200].all() and not ok[200:].any()
    assert (ptrs[:200] != 0).all() and (ptrs[200:] == 0).all()
    assert len(set(ptrs[:200].tolist())) == 200
    assert all(word_at(p) == USER_LOCK for p in ptrs[:20])
    assert t.size() == 500  # a locked key still occupies its slot
    # lookups do not see a locked key (its key word holds the lock marker)
    _, f, _ = g.find(keys)
    assert not f[:200].any() and f[200:].all()
    assert not g.contains(keys[:200]).any()
    # erase leaves it alone
    g.t.erase(10, dev(keys[:10]))
    torch.cuda.synchronize()
    back = unlock(t, dptrs, batch)
    assert back[:200].all() and not back[200:].any()
    v, f, _ = g.find(keys)
    assert f.all() and (v == vals).all()
    # a second unlock finds no lock
    assert not unlock(t, dptrs, batch)[:200].any()
    t.check_device_error()


def test_lock_applies_the_hit_score_rule():
    rng = np.random.default_rng(72)
    for strategy, expect in ((H.EvictStrategy.kLfu, lambda old, s: old + s),
                             (H.EvictStrategy.kCustomized, lambda old, s: s)):
        t = make_table(128 * 64, dim=4, strategy=strategy)
        g = GpuOps(t, 4)
        keys = random_keys(rng, 300)
        old = rng.integers(1, 1000, 300).astype(np.uint64)
        g.insert_or_assign(keys, np.zeros((300, 4), np.float32), old)
        sc = rng.integers(1, 1000, 300).astype(np.uint64)
        dptrs, _, ok = lock(t, keys, sc)
        assert ok.all()
        assert unlock(t, dptrs, keys).all()
        _, f, s = g.find(keys)
        assert f.all() and (s == expect(old, sc)).all()


def test_locked_slot_is_never_the_victim():
    rng = np.random.default_rng(73)
    cap, dim = 128 * 64, 4
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kCustomized)
    g = GpuOps(t, dim)
    full = keys_for_bucket(rng, cap, 9, 128)
    scores = np.arange(1, 129, dtype=np.uint64)
    g.insert_or_assign(full, np.zeros((128, dim), np.float32), scores)
    # lock the two lowest-score keys (scores stay 1 and 2: Customized sets them)
    dptrs, _, ok = lock(t, full[:2], scores[:2])
    assert ok.all()
    new = keys_for_bucket(rng, cap, 9, 1, exclude=full)
    ek, _, es = g.insert_and_evict(new, np.ones((1, dim), np.float32),
                                   np.array([1000], np.uint64))
    # the lowest unlocked score (3) is evicted, not the locked 1 or 2
    assert ek.tolist() == [int(full[2])] and es.tolist() == [3]
    assert unlock(t, dptrs, full[:2]).all()
    assert g.contains(full[:2]).all() and not g.contains(full[2:3]).any()
    assert g.contains(new).all()
    t.check_device_error()


def test_find_or_insert_ptr_keeps_keys_locked():
    rng = np.random.default_rng(74)
    dim = 4
    t = make_table(128 * 64, dim=dim, strategy=H.EvictStrategy.kLru)
    g = GpuOps(t, dim)
    old = random_keys(rng, 100)
    g.insert_or_assign(old, np.full((100, dim), 7, np.float32))
    new = rng.permutation(np.setdiff1d(random_keys(rng, 150), old))[:100]
    keys = np.concatenate([old[:50], new])
    n = len(keys)
    vp = torch.zeros(n, dtype=torch.int64, device="cuda")
    f = torch.zeros(n, dtype=torch.bool, device="cuda")
    lp = torch.zeros(n, dtype=torch.int64, device="cuda")
    t.find_or_insert_ptr(n, dev(keys), vp, f, locked_key_ptrs=lp)
    torch.cuda.synchronize()
    hv, hf, hl = host(vp), host(f).astype(bool), host(lp)
    assert hf[:50].all() and not hf[50:].any()
    assert (hv != 0).all() and (hl != 0).all()
    assert all(word_at(p) == USER_LOCK for p in hl[:10])
    rows = rng.standard_normal((n, dim)).astype(np.float32)
    for i in range(0, n, 7):
        write_row(hv[i], rows[i])
    assert not g.contains(keys).any()  # still locked
    assert unlock(t, lp, keys).all()
    v, fnd, _ = g.find(keys)
    assert fnd.all()
    for i in range(0, n, 7):
        assert (v[i] == rows[i]).all()
    # repeated keys cannot be held locked twice
    with pytest.raises(H.HkvUnsupported):
        t.find_or_insert_ptr(2, dev(np.array([5, 5], np.uint64)), vp, f, unique_key=False,
                             locked_key_ptrs=lp)


def test_reserve_refused_while_locked_and_bad_unlocks():
    rng = np.random.default_rng(75)
    t = make_table(128 * 16, dim=4, max_capacity=128 * 64, strategy=H.EvictStrategy.kLru)
    g = GpuOps(t, 4)
    keys = random_keys(rng, 200)
    g.insert_or_assign(keys, np.zeros((200, 4), np.float32))
    dptrs, _, ok = lock(t, keys[:5])
    assert ok.all()
    with pytest.raises(RuntimeError):
        t.reserve(128 * 64)
    assert t.capacity() == 128 * 16
    # an address outside the table, a null pointer, a reserved key
    bogus = torch.tensor([8, 0, int(host(dptrs)[0])], dtype=torch.int64, device="cuda")
    assert not unlock(t, bogus, np.array([1, 2, 0xFFFFFFFFFFFFFFFF], np.uint64)).any()
    assert unlock(t, dptrs, keys[:5]).all()
    t.reserve(128 * 64)
    assert t.capacity() == 128 * 64 and g.contains(keys).all()


def test_insert_of_a_locked_key_places_a_second_copy():
    """As in the reference (insert_or_assign_kernel.h:128-140 compares the key
    word with the key itself), an insert does not see a locked key."""
    rng = np.random.default_rng(76)
    t = make_table(128 * 16, dim=4, strategy=H.EvictStrategy.kLru)
    g = GpuOps(t, 4)
    keys = random_keys(rng, 10)
    g.insert_or_assign(keys, np.zeros((10, 4), np.float32))
    dptrs, _, ok = lock(t, keys[:1])
    assert ok.all()
    g.insert_or_assign(keys[:1], np.ones((1, 4), np.float32))
    t.check_device_error()
    assert t.size() == 11
    v, f, _ = g.find(keys[:1])
    assert f.all() and (v == 1).all()
    assert unlock(t, dptrs, keys[:1]).all()
    assert g.contains(keys).all()
