"""The CPU oracle against the reference's own known answers (CPU only).

Every expectation below is restated from a test of the reference
(yangzhen92/HierarchicalKV-ascend, tests/); the citation is on each test.
The reference cannot run here (it needs CANN and an Ascend NPU), so these
known answers are what pin the oracle.
"""
import random

import numpy as np
import pytest

import hkv_oracle as O

MASK64 = (1 << 64) - 1


def py_murmur3(k):
    """Independent restatement of the Murmur3 finalizer (utils.h:53-61)."""
    k ^= k >> 33
    k = (k * 0xFF51AFD7ED558CCD) & MASK64
    k ^= k >> 33
    k = (k * 0xC4CEB9FE1A85EC53) & MASK64
    k ^= k >> 33
    return k


def keys_in_bucket(capacity, bucket, count, rng, lo=1, hi=0xFFFFFFFFFFFFFFF0):
    """Key generator of tests/common/test_util.h:244-317: random keys whose
    Murmur3 hash lands in `bucket` of a power-of-two table."""
    out = set()
    while len(out) < count:
        k = rng.randrange(lo, hi)
        if ((py_murmur3(k) & (capacity - 1)) // 128) == bucket:
            out.add(k)
    return np.array(sorted(out), np.uint64)


# ---------------------------------------------------------------- primitives
def test_murmur3_matches_independent_restatement():
    rng = random.Random(7)
    for k in [0, 1, 2, 0xFFFFFFFFFFFFFFFF, 0xFFFFFFFFFFFFFFFE] + [
            rng.getrandbits(64) for _ in range(2000)]:
        assert O.murmur3(k) == py_murmur3(k)


def test_digest_and_reserved_digests():
    # types.h:97-127: digest = byte 4 of the hash; empty/reclaim digests are
    # the digests of EMPTY_KEY / RECLAIM_KEY
    assert O.L.hkvo_empty_digest() == (py_murmur3(O.EMPTY_KEY) >> 32) & 0xFF
    assert O.L.hkvo_reclaim_digest() == (py_murmur3(O.RECLAIM_KEY) >> 32) & 0xFF
    for k in (3, 1234567, 0xDEADBEEFCAFE):
        assert O.digest(k) == (py_murmur3(k) >> 32) & 0xFF


def test_reserved_keys_are_the_top_four_values():
    # types.h:67 RESERVED_KEY_MASK and IS_RESERVED_KEY, :153-156
    for k in range(0xFFFFFFFFFFFFFFFC, 0x10000000000000000):
        assert O.L.hkvo_is_reserved(k)
    for k in (0, 1, 0xFFFFFFFFFFFFFFFB, 0x7FFFFFFFFFFFFFFF):
        assert not O.L.hkvo_is_reserved(k)


@pytest.mark.parametrize("cap", [128, 1 << 20, 128 * 1000, 128 * 8191,
                                 128 * 3 * 7 * 11, (1 << 40) + 128])
def test_magic_division_is_exact(cap):
    # table.h:106-127 and utils.h:85-97 compute hashed % capacity
    import ctypes
    m, s = ctypes.c_uint64(), ctypes.c_uint64()
    O.L.hkvo_magic_div(cap, ctypes.byref(m), ctypes.byref(s))
    rng = random.Random(cap)
    for x in [0, 1, cap - 1, cap, cap + 1, MASK64, MASK64 - 1] + [
            rng.getrandbits(64) for _ in range(3000)]:
        assert O.L.hkvo_fast_mod(x, cap, m.value, s.value) == x % cap


# ------------------------------------------- score functor known answers
# tests/test_score_functor/test_score_functor.cpp:162-380
def test_kat_desired_lru():  # :162-168
    assert O.desired_when_missed(O.LRU, None, 0, 0, 9876543210) == 9876543210


def test_kat_desired_lfu():  # :170-175
    assert O.desired_when_missed(O.LFU, None, 0, 0, 0) == O.MAX_SCORE


def test_kat_desired_epoch_lru():  # :177-184
    epoch, cycle = 5, 0x100000000
    assert O.desired_when_missed(O.EPOCH_LRU, None, 0, epoch, cycle) == \
        (epoch << 32) | ((cycle >> 20) & 0xFFFFFFFF)


def test_kat_desired_epoch_lfu():  # :186-194
    assert O.desired_when_missed(O.EPOCH_LFU, [100], 0, 7, 0) == (7 << 32) | 100


def test_kat_desired_customized():  # :196-203
    assert O.desired_when_missed(O.CUSTOMIZED, [12345], 0, 0, 0) == 12345


def test_kat_update_lfu():  # :217-231: insert stores 999, a hit adds 999
    assert O.score_on_write(O.LFU, 0, [999], 0, 111, True) == 999
    assert O.score_on_write(O.LFU, 999, [999], 0, O.MAX_SCORE - 1, False) == 1998


def test_kat_update_lru_epoch_lru_customized():  # :205-215, :233-243, :260-270
    assert O.score_on_write(O.LRU, 7, None, 0, 123456, False) == 123456
    d = (5 << 32) | 123
    assert O.score_on_write(O.EPOCH_LRU, 7, None, 0, d, False) == d
    assert O.score_on_write(O.CUSTOMIZED, 7, None, 0, 88888, False) == 88888


def test_kat_update_epoch_lfu():  # :245-258
    d = (7 << 32) | 200
    first = O.score_on_write(O.EPOCH_LFU, 0, None, 0, d, True)
    assert first == d
    assert O.score_on_write(O.EPOCH_LFU, first, None, 0, d, False) == (7 << 32) | 400


def test_epoch_lfu_saturates():  # score_functor.h:297-309
    d = (3 << 32) | 10
    old = (2 << 32) | (0xFFFFFFFF - 5)
    assert O.score_on_write(O.EPOCH_LFU, old, None, 0, d, False) == (3 << 32) | 0xFFFFFFFF


def test_kat_update_with_digest():  # :272-352 (score part)
    assert O.score_on_write(O.LRU, 0, None, 0, 123, True) == 123
    assert O.score_on_write(O.LFU, 0, [333], 0, 0, True) == 333
    assert O.score_on_write(O.EPOCH_LRU, 0, None, 0, (3 << 32) | 456, False) == (3 << 32) | 456
    assert O.score_on_write(O.EPOCH_LFU, 0, None, 0, (9 << 32) | 777, True) == (9 << 32) | 777
    assert O.score_on_write(O.CUSTOMIZED, 0, None, 0, 99999, False) == 99999


def test_kat_update_without_missed():  # :354-480
    assert O.score_without_missed(O.LRU, 0, None, 0, 0, 555555) == 555555
    assert O.score_without_missed(O.LFU, 10, [20], 0, 0, 0) == 30
    assert O.score_without_missed(O.EPOCH_LRU, 0, None, 0, 11, 0x200000000) == \
        (11 << 32) | ((0x200000000 >> 20) & 0xFFFFFFFF)
    r = O.score_without_missed(O.EPOCH_LFU, (13 << 32) | 50, [20], 0, 13, 0)
    assert r & 0xFFFFFFFF == 70
    assert O.score_without_missed(O.CUSTOMIZED, 0, [77777], 0, 0, 0) == 77777
    assert O.score_without_missed(O.LFU, 20, [20], 0, 0, 0) == 40
    r = O.score_without_missed(O.EPOCH_LFU, (17 << 32) | 60, [20], 0, 17, 0)
    assert r & 0xFFFFFFFF == 80
    # null input scores leave Lfu/EpochLfu/Customized untouched
    assert O.score_without_missed(O.LFU, 5, None, 0, 0, 0) is None
    assert O.score_without_missed(O.CUSTOMIZED, 5, None, 0, 0, 0) is None


# ------------------------------------------------- table-level expectations
def _table(strategy, cap=128 * 4, dim=4, **kw):
    return O.OracleTable(cap, cap, dim=dim, strategy=strategy, **kw)


@pytest.mark.parametrize("strategy", [O.LRU, O.LFU, O.EPOCH_LRU, O.EPOCH_LFU,
                                      O.CUSTOMIZED])
def test_find_or_insert_strategy_scores(strategy):
    """tests/test_find_or_insert_evict_strategies.cpp:576-623: scores after
    two find_or_insert calls of the same keys: Lfu 2*s, EpochLfu
    (123<<32)|2*s, Customized s, Lru/EpochLru strictly increasing."""
    rng = np.random.default_rng(3)
    n = 300
    keys = rng.choice(1 << 40, n, replace=False).astype(np.uint64) + 1
    scores = rng.integers(1, 1000, n).astype(np.uint64)
    t = O.OracleTable(1024, 1024, dim=4, strategy=strategy)
    t.set_global_epoch(123)
    sc = None if strategy in (O.LRU, O.EPOCH_LRU) else scores
    t.set_clock(1 << 30)
    t.find_or_insert(keys, np.zeros((n, 4), np.float32), sc)
    _, f1, s1 = t.find(keys)
    t.set_clock(3 << 30)
    t.find_or_insert(keys, np.zeros((n, 4), np.float32), sc)
    _, f2, s2 = t.find(keys)
    assert f2.all()
    if strategy == O.LFU:
        assert (s2 == 2 * scores).all()
    elif strategy == O.EPOCH_LFU:
        assert ((s2 >> np.uint64(32)) == 123).all()
        assert ((s2 & np.uint64(0xFFFFFFFF)) == 2 * scores).all()
    elif strategy == O.CUSTOMIZED:
        assert (s2 == scores).all()
    elif strategy == O.LRU:
        assert (s2 > s1).all()
    else:
        assert ((s2 >> np.uint64(32)) == 123).all()
        assert ((s2 & np.uint64(0xFFFFFFFF)) > (s1 & np.uint64(0xFFFFFFFF))).all()


def test_insert_and_evict_reject_admission():
    """tests/test_insert_and_evict.cpp:679-767: a full bucket with scores
    500..627 refuses 64 new keys with scores 0..63; they are all reported with
    their own values; the bucket is unchanged."""
    rng = random.Random(11)
    cap, dim = 128 * 4, 4
    t = _table(O.CUSTOMIZED, cap, dim)
    high = keys_in_bucket(cap, 0, 128, rng)
    hv = (high.astype(np.float64) * 1e-5).astype(np.float32)[:, None].repeat(dim, 1)
    ek, _, _, _ = t.insert_and_evict(high, hv, np.arange(500, 628, dtype=np.uint64))
    assert len(ek) == 0
    low = keys_in_bucket(cap, 0, 64, rng, lo=100000000, hi=200000000)
    lv = np.arange(64 * dim, dtype=np.float32).reshape(64, dim)
    ek, ev, es, _ = t.insert_and_evict(low, lv, np.arange(64, dtype=np.uint64))
    assert len(ek) == 64
    assert set(ek.tolist()) == set(low.tolist())
    order = {int(k): i for i, k in enumerate(low)}
    for k, v, s in zip(ek, ev, es):
        assert (v == lv[order[int(k)]]).all()
        assert s == order[int(k)]  # desired score of a refused key
    assert t.contains(high).all()
    assert not t.contains(low).any()


def test_insert_and_evict_mixed_batch():
    """tests/test_insert_and_evict.cpp:769-961: update / insert / evict /
    reject in one batch: 16 old keys evicted + 16 new keys refused."""
    rng = random.Random(12)
    cap, dim = 128 * 4, 4
    t = _table(O.CUSTOMIZED, cap, dim)
    b0 = keys_in_bucket(cap, 0, 128, rng, hi=10000000)
    t.insert_and_evict(b0, np.ones((128, dim), np.float32), np.arange(1000, 1128, dtype=np.uint64))
    ka = keys_in_bucket(cap, 1, 32, rng, lo=200000000, hi=210000000)
    sa = np.arange(10, 42, dtype=np.uint64)
    t.insert_and_evict(ka, np.full((32, dim), 2, np.float32), sa)
    kb = keys_in_bucket(cap, 2, 32, rng, lo=300000000, hi=310000000)
    kc = keys_in_bucket(cap, 0, 16, rng, lo=100000000, hi=110000000)
    kd = keys_in_bucket(cap, 0, 16, rng, lo=400000000, hi=410000000)
    keys = np.concatenate([ka, kb, kc, kd])
    vals = np.concatenate([np.full((32, dim), 102, np.float32), np.full((32, dim), 3, np.float32),
                           np.full((16, dim), 4, np.float32), np.full((16, dim), 5, np.float32)])
    scores = np.concatenate([sa + 1000, np.arange(200, 232), np.arange(2000, 2016),
                             np.arange(16)]).astype(np.uint64)
    ek, _, _, _ = t.insert_and_evict(keys, vals, scores)
    assert len(ek) == 32
    evicted = set(ek.tolist())
    assert len(evicted & set(b0.tolist())) == 16
    assert len(evicted & set(kd.tolist())) == 16
    v, f, s = t.find(ka)
    assert f.all() and (v == 102).all() and (s == sa + 1000).all()
    assert t.contains(kb).all() and t.contains(kc).all() and not t.contains(kd).any()
    assert t.contains(b0).sum() == 128 - 16


def test_duplicate_new_key_full_bucket_accept_once():
    """tests/test_insert_and_evict.cpp (NonUniqueFalse_DuplicateNewKey_
    FullBucket_AcceptOnce): 4 copies of one new key, score 10000, into a full
    bucket with scores 0..127: one old key is evicted, size stays 128."""
    rng = random.Random(13)
    cap = 128 * 4
    t = _table(O.CUSTOMIZED, cap, 4)
    old = keys_in_bucket(cap, 0, 128, rng, hi=10000000)
    t.insert_and_evict(old, np.zeros((128, 4), np.float32), np.arange(128, dtype=np.uint64))
    k = keys_in_bucket(cap, 0, 1, rng, lo=10000001, hi=20000000)
    ek, _, _, _ = t.insert_and_evict(np.repeat(k, 4), np.arange(16, dtype=np.float32).reshape(4, 4),
                                     np.full(4, 10000, np.uint64))
    assert len(ek) == 1 and int(ek[0]) in set(old.tolist())
    assert t.size() == 128 and t.contains(k).all()


def test_duplicate_new_key_full_bucket_refused_per_input():
    """tests/test_insert_and_evict.cpp (..._RefusedPerInput): 3 copies of a key
    with score 1 into a full bucket with scores 1000..1127: 3 refusals."""
    rng = random.Random(14)
    cap = 128 * 4
    t = _table(O.CUSTOMIZED, cap, 4)
    old = keys_in_bucket(cap, 0, 128, rng, hi=10000000)
    t.insert_and_evict(old, np.zeros((128, 4), np.float32), np.arange(1000, 1128, dtype=np.uint64))
    k = keys_in_bucket(cap, 0, 1, rng, lo=10000001, hi=20000000)
    ek, _, _, _ = t.insert_and_evict(np.repeat(k, 3), np.zeros((3, 4), np.float32),
                                     np.ones(3, np.uint64))
    assert len(ek) == 3 and t.size() == 128


def test_duplicate_existing_key_matches_one_candidate():
    """tests/test_insert_and_evict.cpp (..._DuplicateExistingKey_NoEvict): the
    final (value, score) is one of the duplicates' (value, score) pairs."""
    t = _table(O.CUSTOMIZED, 128 * 8, 4)
    t.insert_and_evict(np.array([1001], np.uint64), np.ones((1, 4), np.float32),
                       np.array([10], np.uint64))
    vals = np.array([[10 + r] * 4 for r in range(4)], np.float32)
    ek, _, _, _ = t.insert_and_evict(np.full(4, 1001, np.uint64), vals,
                                     np.array([101, 102, 103, 104], np.uint64))
    assert len(ek) == 0 and t.size() == 1
    v, f, s = t.find(np.array([1001], np.uint64))
    cand = {(tuple(vals[r]), 101 + r) for r in range(4)}
    assert f[0] and (tuple(v[0]), int(s[0])) in cand


def test_reserved_keys_are_ignored():
    """tests/test_find.cpp:881, tests/test_contains.cpp:382: reserved keys are
    never found and never inserted."""
    t = _table(O.LRU, 128 * 8, 4)
    res = np.array([0xFFFFFFFFFFFFFFFC, 0xFFFFFFFFFFFFFFFD, 0xFFFFFFFFFFFFFFFE,
                    0xFFFFFFFFFFFFFFFF], np.uint64)
    t.insert_or_assign(res, np.ones((4, 4), np.float32))
    assert t.size() == 0
    assert not t.contains(res).any()


def test_erase_and_tombstone_reuse():
    """remove_kernel.h:79-110 + insert_or_assign_kernel.h:241-252: an erased
    slot becomes a RECLAIM tombstone (score 0); once a bucket has no EMPTY
    slot the tombstone is reused through the eviction path."""
    rng = random.Random(15)
    cap = 128 * 4
    t = _table(O.CUSTOMIZED, cap, 4)
    ks = keys_in_bucket(cap, 0, 128, rng)
    t.insert_or_assign(ks, np.zeros((128, 4), np.float32), np.arange(100, 228, dtype=np.uint64))
    t.erase(ks[:3])
    assert t.size() == 125
    keys, scores, digests, sizes, _ = t.get_state()
    assert (keys[:128] == O.RECLAIM_KEY).sum() == 3
    new = keys_in_bucket(cap, 0, 3, rng, lo=1 << 50, hi=1 << 51)
    res = t.insert_or_assign(new, np.zeros((3, 4), np.float32), np.array([1, 2, 3], np.uint64))
    assert (res == O.R_OCCUPIED_RECLAIMED).all()
    assert t.size() == 128 and t.contains(ks[3:]).all()


def test_reserve_exactness():
    """tests/test_reserve.cpp:37-170: capacity doubles exactly, never shrinks,
    size is kept, load factor is exact, every value is found after each
    doubling."""
    dim, key_num, init = 8, 1024, 128 * 16
    t = O.OracleTable(init, init * 16, dim=dim, strategy=O.LRU, max_load_factor=1.0)
    keys = np.arange(1, key_num + 1, dtype=np.uint64)
    vals = (keys.astype(np.float64) * 1e-5).astype(np.float32)[:, None].repeat(dim, 1)
    t.insert_or_assign(keys, vals)
    assert t.size() == key_num and t.capacity() == init
    t.reserve(init // 2)
    assert t.capacity() == init
    t.reserve(init)
    assert t.capacity() == init
    t.reserve(init + 1)
    assert t.capacity() == init * 2
    assert t.load_factor() == np.float32(key_num / (init * 2))
    target = init * 2
    while target <= init * 16:
        t.reserve(target)
        assert t.capacity() == target and t.size() == key_num
        v, f, _ = t.find(keys)
        assert f.all() and (v == vals).all()
        target *= 2


def test_reserve_full_table_defragmentation():
    """tests/test_reserve.cpp:193-300: a completely full table doubles to load
    factor 0.5 and every key is still found with its value."""
    dim, init = 4, 128 * 8
    t = O.OracleTable(init, init * 2, dim=dim, strategy=O.LRU, max_load_factor=1e30)
    rng = np.random.default_rng(5)
    for step in range(6):
        k = rng.choice(1 << 50, init, replace=False).astype(np.uint64) + 1
        t.set_clock(step + 1)
        t.insert_or_assign(k, np.ones((init, dim), np.float32))
    assert t.size() == init
    keys, _, _, _, vals = t.get_state()
    live = keys[keys < 0xFFFFFFFFFFFFFFFC]
    t.reserve(init + 1)
    assert t.capacity() == init * 2 and t.load_factor() == 0.5
    assert t.contains(live).all()


def test_export_batch_offsets():
    """tests/test_export_batch.cpp:115-250: full scan exports every inserted
    key with its value; an offset scan exports a subset; an empty table
    exports nothing; offset >= capacity exports nothing."""
    dim, cap, n = 8, 128 * 1024, 5000
    t = O.OracleTable(cap, cap, dim=dim, strategy=O.LRU)
    assert len(t.export_batch(cap)[0]) == 0
    keys = np.arange(1, n + 1, dtype=np.uint64)
    vals = (keys.astype(np.float64) * 1e-5).astype(np.float32)[:, None].repeat(dim, 1)
    t.insert_or_assign(keys, vals)
    ek, ev, _ = t.export_batch(cap)
    assert len(ek) == n and set(ek.tolist()) == set(keys.tolist())
    ref = {int(k): vals[i] for i, k in enumerate(keys)}
    for k, v in zip(ek, ev):
        assert (ref[int(k)] == v).all()
    part, _, _ = t.export_batch(cap, offset=cap // 2)
    assert 0 < len(part) < n
    assert len(t.export_batch(10, offset=cap)[0]) == 0


def test_insert_and_evict_reference_map():
    """tests/test_reserve.cpp:320-420 pattern: every inserted key is either in
    the table with its value or was reported evicted with its value."""
    dim, cap, batch = 4, 128 * 16, 512
    t = O.OracleTable(cap, cap, dim=dim, strategy=O.LRU)
    live = {}
    off = 0
    for step in range(12):
        keys = np.arange(off, off + batch, dtype=np.uint64)
        vals = keys.astype(np.float32)[:, None].repeat(dim, 1)
        t.set_clock(step + 1)
        ek, ev, _, _ = t.insert_and_evict(keys, vals)
        for k, v in zip(keys, vals):
            live[int(k)] = v
        for k, v in zip(ek, ev):
            assert (live.pop(int(k)) == v).all()
        off += batch
    keys = np.array(list(live.keys()), np.uint64)
    v, f, _ = t.find(keys)
    assert f.all() and t.size() == len(live)
    assert (v == np.array([live[int(k)] for k in keys])).all()


def test_accum_or_assign_rules():
    """accum_or_assign_kernel.h:108-153: accum adds to existing keys, assign
    inserts new keys, mismatched cases change nothing."""
    t = _table(O.LRU, 128 * 8, 4)
    k = np.array([10, 20], np.uint64)
    t.insert_or_assign(k[:1], np.full((1, 4), 1.5, np.float32))
    t.accum_or_assign(np.array([10, 20, 30, 10], np.uint64),
                      np.array([[2] * 4, [5] * 4, [7] * 4, [9] * 4], np.float32),
                      np.array([1, 1, 0, 0], np.uint8))
    v, f, _ = t.find(np.array([10, 20, 30], np.uint64))
    assert f.tolist() == [True, False, True]
    assert (v[0] == 3.5).all() and (v[2] == 7).all()


def test_multithreaded_oracle_equals_single_threaded():
    rng = np.random.default_rng(9)
    cap, dim = 128 * 256, 4
    keys = rng.integers(1, 1 << 62, 20000).astype(np.uint64)
    vals = rng.random((20000, dim)).astype(np.float32)
    sc = rng.integers(1, 1 << 40, 20000).astype(np.uint64)
    a = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED, threads=1)
    b = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED, threads=8)
    a.insert_or_assign(keys, vals, sc)
    b.insert_or_assign(keys, vals, sc)
    for x, y in zip(a.get_state(), b.get_state()):
        assert (x == y).all()


# ------------------------------------- erase, insert_or_assign, accum, assign
def test_erase_in_full_bucket():
    """tests/test_erase.cpp:73-150 (test_erase_in_full_bucket): one bucket
    (capacity 128), Lru: keys 1..1024 in one call, then the last key again,
    leave the bucket full with the last key in it; erasing it leaves 127;
    inserting it again fills the bucket and changes no other key's
    presence."""
    t = O.OracleTable(128, 128, dim=8, strategy=O.LRU)
    keys = np.arange(1, 1025, dtype=np.uint64)
    vals = np.zeros((1024, 8), np.float32)
    t.set_clock(100)
    t.insert_or_assign(keys, vals)
    t.set_clock(200)
    t.insert_or_assign(keys[-1:], vals[:1])
    assert t.size() == 128
    before = t.contains(keys)
    assert before[-1] and before.sum() == 128
    t.erase(keys[-1:])
    assert t.size() == 127
    t.set_clock(300)
    res = t.insert_or_assign(keys[-1:], vals[:1])
    assert res[0] == O.R_OCCUPIED_RECLAIMED  # the tombstone (score 0) is the victim
    assert t.size() == 128
    assert (t.contains(keys) == before).all()


def test_erase_then_insert_and_evict_reuses_tombstones():
    """tests/test_erase.cpp:289-375 (test_erase_with_insert_and_evict): a full
    one-bucket table (keys 1..128, Lru); erase 10 keys (size 118);
    insert_and_evict of the same 10 keys reports nothing evicted (tombstones
    are not reported), the size is back to 128 and the keys are found."""
    t = O.OracleTable(128, 128, dim=8, strategy=O.LRU)
    keys = np.arange(1, 129, dtype=np.uint64)
    t.set_clock(10)
    t.insert_or_assign(keys, np.zeros((128, 8), np.float32))
    assert t.size() == 128
    t.erase(keys[:10])
    assert t.size() == 118
    t.set_clock(20)
    ek, _, _, _ = t.insert_and_evict(keys[:10], np.ones((10, 8), np.float32))
    assert len(ek) == 0
    assert t.size() == 128
    assert t.contains(keys[:10]).all()


def test_insert_or_assign_evict():
    """tests/test_insert_or_assign.cpp:230-267 (test_evict): one bucket
    (capacity 128), Lru, 1024 keys 0..1023 with values key*1e-5 in one call:
    size 128, and every key found carries its own value."""
    t = O.OracleTable(128, 128, dim=8, strategy=O.LRU)
    keys = np.arange(0, 1024, dtype=np.uint64)
    vals = (keys.astype(np.float64) * 1e-5).astype(np.float32)[:, None].repeat(8, 1)
    t.set_clock(1)
    t.insert_or_assign(keys, vals)
    assert t.size() == 128
    v, f, _ = t.find(keys)
    assert f.sum() == 128
    assert (v[f] == vals[f]).all()


def test_insert_or_assign_repeated_keys():
    """tests/test_insert_or_assign.cpp:454-560 (test_repeat_key_basic): keys
    i // 10 for i < 1024 (103 distinct keys, 10 occurrences each, every
    occurrence with its own value), unique_key = false: size 103, every key
    found, its value one of its occurrences' values."""
    dim, n, rep = 8, 1024, 10
    t = O.OracleTable(128 * 1024, 128 * 1024, dim=dim, strategy=O.LRU)
    keys = (np.arange(n) // rep).astype(np.uint64)
    vals = ((np.arange(n) + 1).astype(np.float64) * 1e-5).astype(np.float32)[:, None].repeat(dim, 1)
    t.insert_or_assign(keys, vals)
    assert t.size() == (n + rep - 1) // rep
    uniq = np.unique(keys)
    v, f, _ = t.find(uniq)
    assert f.all()
    for k, row in zip(uniq, v):
        occ = vals[keys == k]
        assert any((row == o).all() for o in occ)


def test_accum_or_assign_basic_when_full():
    """tests/test_accum_or_assign.cpp:1659-1723 (test_basic_when_full),
    Customized, as many random keys as slots, all assigns: erasing every key
    empties the table, and assigning them again gives the same size."""
    cap, dim = 128 * 64, 8
    rng = np.random.default_rng(31)
    keys = np.unique(rng.integers(0, 1 << 63, cap + 64, dtype=np.uint64))[:cap]
    rng.shuffle(keys)
    t = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED)
    vals = np.full((cap, dim), 1.0, np.float32)
    acc = np.zeros(cap, np.uint8)
    t.accum_or_assign(keys, vals, acc, keys.copy())
    first = t.size()
    assert 0 < first <= cap
    t.erase(keys)
    assert t.size() == 0
    t.accum_or_assign(keys, vals, acc, keys.copy())
    assert t.size() == first


def test_accum_or_assign_values_check():
    """tests/test_accum_or_assign.cpp:2204-2232 with CheckAccumOrAssignValues
    :99-195, Lru, auto-grow from 1024 slots to U, batches of U + 13 random
    keys from [0, 16 (U + 13)) with values key*1e-5, the accum flags taken
    from a find of the batch: after each call every live key holds its old
    value plus its delta (present and in the batch), its delta (new and in
    the batch) or its old value (not in the batch); the size equals the
    exported count."""
    U, dim = 8192, 8
    B = U + 13
    t = O.OracleTable(1024, U, dim=dim, strategy=O.LRU)
    rng = np.random.default_rng(32)
    for rnd in range(6):
        keys = np.unique(rng.integers(0, 16 * B, 2 * B, dtype=np.uint64))
        rng.shuffle(keys)
        keys = keys[:B]
        vals = (keys.astype(np.float64) * 1e-5).astype(np.float32)[:, None].repeat(dim, 1)
        _, found, _ = t.find(keys)
        k0, v0, _ = t.export_batch(t.capacity())
        assert len(k0) == t.size()
        before = {int(k): v[0] for k, v in zip(k0, v0)}
        t.set_clock(rnd + 1)
        t.accum_or_assign(keys, vals, found.astype(np.uint8))
        k1, v1, _ = t.export_batch(t.capacity())
        assert len(k1) == t.size()
        batch = {int(k): v[0] for k, v in zip(keys, vals)}
        for k, row in zip(k1.tolist(), v1):
            if k in before:
                exp = np.float32(before[k] + batch[k]) if k in batch else before[k]
            else:
                assert k in batch
                exp = batch[k]
            assert (row == exp).all(), k


def test_assign_scores_partial_keys():
    """tests/test_assign_scores.cpp:301-394 (partial_keys_exist), Lfu: keys
    1..500 inserted with scores = keys; assign_scores of keys 1..1000 with
    scores 5000 + i keeps the size at 500, adds to the present keys' scores
    (Lfu hit rule) and inserts nothing."""
    t = O.OracleTable(128 * 1024, 128 * 1024, dim=8, strategy=O.LFU)
    ins = np.arange(1, 501, dtype=np.uint64)
    t.insert_or_assign(ins, np.zeros((500, 8), np.float32), ins.copy())
    upd = np.arange(1, 1001, dtype=np.uint64)
    sc = (5000 + np.arange(1000)).astype(np.uint64)
    t.assign_scores(upd, sc)
    assert t.size() == 500
    _, f, s = t.find(upd)
    assert f[:500].all() and not f[500:].any()
    assert (s[:500] == ins + sc[:500]).all()


def test_assign_scores_multiple_updates_and_lru():
    """tests/test_assign_scores.cpp:681-751 (multiple_updates, Lfu: every key
    stays found through repeated updates with scores (t+1)*1000 + i, the Lfu
    rule adding each) and :1030-1108 (lru_strategy: assign_scores without
    scores moves every Lru score forward)."""
    n = 1024
    keys = np.arange(1, n + 1, dtype=np.uint64)
    t = O.OracleTable(128 * 1024, 128 * 1024, dim=8, strategy=O.LFU)
    t.insert_or_assign(keys, np.zeros((n, 8), np.float32), keys.copy())
    total = keys.copy()
    for step in range(5):
        sc = ((step + 1) * 1000 + np.arange(n)).astype(np.uint64)
        t.assign_scores(keys, sc)
        total += sc
        _, f, s = t.find(keys)
        assert f.all() and (s == total).all()
    lru = O.OracleTable(128 * 1024, 128 * 1024, dim=8, strategy=O.LRU)
    lru.set_clock(1000)
    lru.insert_or_assign(keys, np.zeros((n, 8), np.float32))
    _, _, s0 = lru.find(keys)
    lru.set_clock(5000)
    lru.assign_scores(keys)
    _, f, s1 = lru.find(keys)
    assert f.all() and (s1 >= s0).all() and (s1 > s0).any()
