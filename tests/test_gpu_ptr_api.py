"""find* and find_or_insert* (pointer-returning variants, GPU).

Reference: HashTable::find(n, keys, value_type** values, founds, scores)
(hkv_hashtable.h:2244-2264, find_ptr_with_digest_kernel.h) and
find_or_insert(n, keys, value_type** values, founds, scores, ...)
(hkv_hashtable.h:1658-1727, find_or_insert_ptr_kernel_v2.h): each key's
result is the address of its value row inside the table; a missed (find*) or
refused (find_or_insert*) key gets a null address; find_or_insert* places
keys, evicts and scores exactly as find_or_insert does, but copies no value.
The rows are read and written here through the addresses with cudaMemcpy.
"""
import numpy as np
import pytest
import torch

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import GpuOps, dev, host, make_table
from hkv_testutil import keys_for_bucket, one_key_per_bucket

pytestmark = pytest.mark.gpu


def _rt():
    from cuda.bindings import runtime as rt
    return rt


def read_row(ptr, dim):
    rt = _rt()
    out = np.empty(dim, np.float32)
    (err,) = rt.cudaMemcpy(out.ctypes.data, int(ptr), dim * 4,
                           rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess
    return out


def write_row(ptr, row):
    rt = _rt()
    row = np.ascontiguousarray(row, np.float32)
    (err,) = rt.cudaMemcpy(int(ptr), row.ctypes.data, row.nbytes,
                           rt.cudaMemcpyKind.cudaMemcpyHostToDevice)
    assert err == rt.cudaError_t.cudaSuccess


def ptrs(n):
    return torch.zeros(max(n, 1), dtype=torch.int64, device="cuda")


def test_find_ptr_addresses_rows():
    rng = np.random.default_rng(21)
    dim = 8
    t = make_table(128 * 64, dim=dim, strategy=H.EvictStrategy.kCustomized)
    ops = GpuOps(t, dim)
    keys = np.unique(rng.integers(1, 1 << 62, 3000, dtype=np.uint64))[:2000]
    vals = rng.standard_normal((len(keys), dim)).astype(np.float32)
    sc = np.arange(1, len(keys) + 1, dtype=np.uint64)
    ops.insert_or_assign(keys, vals, sc)
    q = np.concatenate([keys[:150], np.unique(rng.integers(1 << 62, 1 << 63, 60,
                                                          dtype=np.uint64))[:50]])
    q = np.concatenate([q, [np.uint64(0xFFFFFFFFFFFFFFFF)]])  # a reserved key
    p = ptrs(len(q))
    f = torch.zeros(len(q), dtype=torch.bool, device="cuda")
    s = torch.zeros(len(q), dtype=torch.int64, device="cuda")
    t.find_ptr(len(q), dev(q), p, f, s)
    torch.cuda.synchronize()
    hp, hf, hs = host(p), host(f).astype(bool), host(s, np.uint64)
    ref_v, ref_f, ref_s = ops.find(q)
    assert (hf == ref_f).all()
    assert ((hp != 0) == hf).all()
    assert (hs[hf] == ref_s[hf]).all()
    assert len(set(hp[hf].tolist())) == hf.sum()  # one row per key
    for i in np.nonzero(hf)[0][:40]:
        assert (read_row(hp[i], dim) == ref_v[i]).all()


def test_find_or_insert_ptr_unique_matches_find_or_insert():
    rng = np.random.default_rng(22)
    dim, cap = 4, 128 * 32
    # Customized, distinct scores: the result of a batch does not depend on
    # thread order, so table contents compare exactly
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kCustomized)
    o = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED)
    pre = np.unique(rng.integers(1, 1 << 62, 5000, dtype=np.uint64))[:4000]
    pv = rng.standard_normal((len(pre), dim)).astype(np.float32)
    scores = rng.permutation(np.arange(1, 100000, dtype=np.uint64))
    ps = scores[:len(pre)]
    GpuOps(t, dim).insert_or_assign(pre, pv, ps)
    o.insert_or_assign(pre, pv, ps)
    # new keys only (a mix of hits and evicting misses in one bucket has an
    # order-dependent result)
    keys = np.setdiff1d(np.unique(rng.integers(1, 1 << 62, 1500, dtype=np.uint64)), pre)[:1000]
    keys = rng.permutation(keys)
    ks = scores[len(pre):len(pre) + len(keys)]
    p = ptrs(len(keys))
    f = torch.zeros(len(keys), dtype=torch.bool, device="cuda")
    t.find_or_insert_ptr(len(keys), dev(keys), p, f, dev(ks))
    torch.cuda.synchronize()
    hp, hf = host(p), host(f).astype(bool)
    assert not hf.any()
    zeros = np.zeros((len(keys), dim), np.float32)
    _, res = o.find_or_insert(keys, zeros, ks)
    placed = hp != 0
    o_keys, o_sc, _, o_sz, _ = o.get_state()
    g_keys, g_sc, _, g_sz, _ = t.get_state()
    live = lambda k, s: {int(a): int(b) for a, b in zip(k, s) if a < np.uint64(0xFFFFFFFFFFFFFFFC)}
    assert live(g_keys, g_sc) == live(o_keys, o_sc)
    assert (g_sz == o_sz).all()
    # every key in the table now got an address; a key without one is not
    # in the table (a placed key can still be evicted later in the same batch
    # by a key with a higher score, which then owns that row)
    now = set(live(g_keys, g_sc))
    assert all(bool(pl) for k, pl in zip(keys, placed) if int(k) in now)
    assert not any(int(k) in now for k, pl in zip(keys, placed) if not pl)
    # rows written through the addresses of resident keys are what find returns
    new_rows = rng.standard_normal((len(keys), dim)).astype(np.float32)
    resident = [i for i in range(len(keys)) if int(keys[i]) in now][:60]
    for i in resident:
        write_row(hp[i], new_rows[i])
    fv, ff, _ = GpuOps(t, dim).find(keys)
    for i in resident:
        assert ff[i] and (fv[i] == new_rows[i]).all()
    # hits: addresses of the existing rows, found, score rule of find_or_insert
    hit = np.array([k for k in keys if int(k) in now], np.uint64)[:200]
    hs = scores[-200:]
    p2 = ptrs(len(hit))
    f2 = torch.zeros(len(hit), dtype=torch.bool, device="cuda")
    t.find_or_insert_ptr(len(hit), dev(hit), p2, f2, dev(hs))
    o.find_or_insert(hit, np.zeros((len(hit), dim), np.float32), hs)
    torch.cuda.synchronize()
    assert host(f2).astype(bool).all()
    g_keys, g_sc, _, _, _ = t.get_state()
    o_keys, o_sc, _, _, _ = o.get_state()
    assert live(g_keys, g_sc) == live(o_keys, o_sc)


def test_find_or_insert_ptr_repeated_keys_and_refusal():
    dim, cap = 4, 128 * 64
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kCustomized)
    rng = np.random.default_rng(5)
    ks = one_key_per_bucket(rng, cap, range(8))
    batch = np.concatenate([ks, ks, ks[:3]])
    sc = np.full(len(batch), 10, np.uint64)
    p = ptrs(len(batch))
    f = torch.zeros(len(batch), dtype=torch.bool, device="cuda")
    t.find_or_insert_ptr(len(batch), dev(batch), p, f, dev(sc), unique_key=False)
    torch.cuda.synchronize()
    hp, hf = host(p), host(f).astype(bool)
    # first occurrences are new, later ones find them; same row everywhere
    assert (~hf[:8]).all() and hf[8:].all()
    assert (hp[:8] != 0).all() and (hp[8:16] == hp[:8]).all() and (hp[16:] == hp[:3]).all()
    assert t.size() == 8
    # a full bucket refuses a lower score: null address, not found
    full = keys_for_bucket(rng, cap, 20, 128)
    GpuOps(t, dim).insert_or_assign(full, np.zeros((128, dim), np.float32),
                                    np.full(128, 100, np.uint64))
    low = keys_for_bucket(rng, cap, 20, 1, exclude=full)
    p3 = ptrs(1)
    f3 = torch.ones(1, dtype=torch.bool, device="cuda")
    t.find_or_insert_ptr(1, dev(low), p3, f3, dev(np.array([1], np.uint64)))
    torch.cuda.synchronize()
    assert int(host(p3)[0]) == 0 and not bool(host(f3)[0])


def test_locked_key_ptrs_need_unique_keys():
    """locked_key_ptrs keeps each placed key locked for the caller, which a
    key repeated in the batch cannot be twice: unique_key=false is refused
    (the locking itself is covered by test_gpu_lock_keys.py)."""
    t = make_table(128 * 8, dim=4, strategy=H.EvictStrategy.kLru)
    k = dev(np.array([5, 6], np.uint64))
    p = ptrs(2)
    f = torch.zeros(2, dtype=torch.bool, device="cuda")
    lk = ptrs(2)
    with pytest.raises(H.HkvUnsupported):
        H._check(H.lib().hkv_find_or_insert_ptr(t._h, 2, H._ptr(k), H._ptr(p), H._ptr(f),
                                                None, H._stream(None), False, False,
                                                H._ptr(lk)))
    assert t.size() == 0
