"""Reference test expectations replayed on the CUDA table (GPU): duplicate
keys in one batch, score rules per strategy, argument checks, hybrid
HBM + host value storage, and the bounded device lock wait."""
import time

import numpy as np
import pytest
import torch

import hkv_b200 as H
from hkv_gpu import GpuOps, dev, host, make_table, zeros_u64
from hkv_testutil import keys_for_bucket, random_keys

pytestmark = pytest.mark.gpu

CUST = H.EvictStrategy.kCustomized


def full_bucket(g, rng, cap, scores):
    old = keys_for_bucket(rng, cap, 0, 128)
    c = g.insert_and_evict(old, np.zeros((128, g.dim), np.float32),
                           np.asarray(scores, np.uint64))
    assert len(c[0]) == 0
    return old


def test_nonunique_duplicate_existing_key():
    """tests/test_insert_and_evict.cpp:1179-1246."""
    g = GpuOps(make_table(128 * 64, dim=4), 4)
    g.insert_and_evict(np.array([1001], np.uint64), np.ones((1, 4), np.float32),
                       np.array([10], np.uint64))
    vals = np.array([[10 + r] * 4 for r in range(4)], np.float32)
    ek, _, _ = g.insert_and_evict(np.full(4, 1001, np.uint64), vals,
                                  np.array([101, 102, 103, 104], np.uint64), unique=False)
    assert len(ek) == 0 and g.t.size() == 1
    v, f, s = g.find(np.array([1001], np.uint64))
    assert f[0] and (tuple(v[0]), int(s[0])) in {(tuple(vals[r]), 101 + r) for r in range(4)}


def test_nonunique_duplicate_new_key_empty_bucket():
    """tests/test_insert_and_evict.cpp:1248-1303."""
    g = GpuOps(make_table(128 * 64, dim=4), 4)
    vals = np.array([[20 + r] * 4 for r in range(5)], np.float32)
    sc = np.array([201, 202, 203, 204, 205], np.uint64)
    ek, _, _ = g.insert_and_evict(np.full(5, 909090, np.uint64), vals, sc, unique=False)
    assert len(ek) == 0 and g.t.size() == 1
    v, f, s = g.find(np.array([909090], np.uint64))
    assert f[0] and (tuple(v[0]), int(s[0])) in {(tuple(vals[r]), int(sc[r])) for r in range(5)}


def test_nonunique_full_bucket_accept_once():
    """tests/test_insert_and_evict.cpp:1305-1370."""
    rng = np.random.default_rng(3)
    cap = 128 * 4
    g = GpuOps(make_table(cap, dim=4), 4)
    old = full_bucket(g, rng, cap, np.arange(128))
    k = keys_for_bucket(rng, cap, 0, 1, exclude=old)
    ek, _, _ = g.insert_and_evict(np.repeat(k, 4), np.arange(16, dtype=np.float32).reshape(4, 4),
                                  np.full(4, 10000, np.uint64), unique=False)
    assert len(ek) == 1 and int(ek[0]) in set(old.tolist())
    assert g.t.size() == 128 and g.contains(k).all()


def test_nonunique_full_bucket_refused_per_input():
    """tests/test_insert_and_evict.cpp:1372-1438."""
    rng = np.random.default_rng(4)
    cap = 128 * 4
    g = GpuOps(make_table(cap, dim=4), 4)
    full_bucket(g, rng, cap, np.arange(1000, 1128))
    k = keys_for_bucket(rng, cap, 0, 1)
    vals = np.array([[40 + r] * 4 for r in range(3)], np.float32)
    ek, ev, es = g.insert_and_evict(np.repeat(k, 3), vals, np.ones(3, np.uint64), unique=False)
    assert len(ek) == 3 and g.t.size() == 128
    assert sorted(tuple(r) for r in ev) == sorted(tuple(r) for r in vals)
    assert (es == 1).all()


def test_reject_admission_reports_inputs():
    """tests/test_insert_and_evict.cpp:679-767."""
    rng = np.random.default_rng(5)
    cap, dim = 128 * 4, 4
    g = GpuOps(make_table(cap, dim=dim), dim)
    high = full_bucket(g, rng, cap, np.arange(500, 628))
    low = keys_for_bucket(rng, cap, 0, 64, exclude=high)
    lv = np.arange(64 * dim, dtype=np.float32).reshape(64, dim)
    ek, ev, es = g.insert_and_evict(low, lv, np.arange(64, dtype=np.uint64))
    assert len(ek) == 64 and set(ek.tolist()) == set(low.tolist())
    order = {int(k): i for i, k in enumerate(low)}
    for k, v, s in zip(ek, ev, es):
        assert (v == lv[order[int(k)]]).all() and s == order[int(k)]
    assert g.contains(high).all() and not g.contains(low).any()


@pytest.mark.parametrize("unique", [True, False])
def test_find_or_insert_duplicates_lfu_sum(unique):
    """Lfu: every occurrence of a key adds its score (score_functor.h:157-160);
    with unique_key=false the duplicates of a batch merge to the sum."""
    g = GpuOps(make_table(128 * 64, dim=4, strategy=H.EvictStrategy.kLfu), 4)
    k = np.array([77, 78], np.uint64)
    g.find_or_insert(k, np.full((2, 4), 3, np.float32), np.array([5, 6], np.uint64))
    if unique:
        keys = k
        sc = np.array([1, 2], np.uint64)
    else:
        keys = np.array([77, 78, 77, 77, 78], np.uint64)
        sc = np.array([1, 2, 10, 100, 20], np.uint64)
    out = g.find_or_insert(keys, np.zeros((len(keys), 4), np.float32), sc, unique=unique)
    assert (out == 3).all()  # every occurrence reads the stored value back
    _, f, s = g.find(k)
    assert f.all()
    exp = [5 + sc[keys == 77].sum(), 6 + sc[keys == 78].sum()]
    assert s.tolist() == exp


def test_find_or_insert_new_duplicates_read_first_value():
    g = GpuOps(make_table(128 * 64, dim=4, strategy=CUST), 4)
    keys = np.array([9, 9, 9], np.uint64)
    vals = np.array([[1] * 4, [2] * 4, [3] * 4], np.float32)
    out = g.find_or_insert(keys, vals, np.array([4, 5, 6], np.uint64), unique=False)
    assert (out == 1).all() and g.t.size() == 1


def test_insert_or_assign_duplicates_last_value_wins():
    g = GpuOps(make_table(128 * 64, dim=4, strategy=CUST), 4)
    keys = np.array([9, 8, 9, 9], np.uint64)
    vals = np.array([[1] * 4, [7] * 4, [2] * 4, [3] * 4], np.float32)
    g.insert_or_assign(keys, vals, np.array([4, 1, 5, 6], np.uint64), unique=False)
    v, f, s = g.find(np.array([9, 8], np.uint64))
    assert f.all() and (v[0] == 3).all() and s.tolist() == [6, 1]


@pytest.mark.parametrize("strategy", [H.EvictStrategy.kLru, H.EvictStrategy.kLfu,
                                      H.EvictStrategy.kEpochLru, H.EvictStrategy.kEpochLfu,
                                      H.EvictStrategy.kCustomized])
def test_find_or_insert_strategy_scores(strategy):
    """tests/test_find_or_insert_evict_strategies.cpp:576-623."""
    rng = np.random.default_rng(6)
    n = 2000
    g = GpuOps(make_table(128 * 64, dim=4, strategy=strategy, epoch=123), 4)
    keys = random_keys(rng, n)
    scores = rng.integers(1, 1000, n).astype(np.uint64)
    sc = None if strategy in (H.EvictStrategy.kLru, H.EvictStrategy.kEpochLru) else scores
    g.find_or_insert(keys, np.zeros((n, 4), np.float32), sc)
    _, _, s1 = g.find(keys)
    time.sleep(0.005)  # > 2^20 ns so the EpochLru clock part moves
    g.find_or_insert(keys, np.zeros((n, 4), np.float32), sc)
    _, f, s2 = g.find(keys)
    assert f.all()
    lo = np.uint64(0xFFFFFFFF)
    if strategy == H.EvictStrategy.kLfu:
        assert (s2 == 2 * scores).all()
    elif strategy == H.EvictStrategy.kEpochLfu:
        assert ((s2 >> np.uint64(32)) == 123).all() and ((s2 & lo) == 2 * scores).all()
    elif strategy == H.EvictStrategy.kCustomized:
        assert (s2 == scores).all()
    elif strategy == H.EvictStrategy.kLru:
        assert (s2 > s1).all()
    else:
        assert ((s2 >> np.uint64(32)) == 123).all() and ((s2 & lo) > (s1 & lo)).all()


def test_strategy_argument_checks():
    """check_evict_strategy, hkv_hashtable.h:3270-3298."""
    lru = make_table(128 * 8, dim=4, strategy=H.EvictStrategy.kLru)
    k = dev(np.array([1, 2], np.uint64))
    v = dev(np.zeros((2, 4), np.float32))
    s = dev(np.array([1, 2], np.uint64))
    with pytest.raises(H.HkvException):
        lru.insert_or_assign(2, k, v, s)
    lfu = make_table(128 * 8, dim=4, strategy=H.EvictStrategy.kLfu)
    with pytest.raises(H.HkvException):
        lfu.insert_or_assign(2, k, v, None)
    elfu = make_table(128 * 8, dim=4, strategy=H.EvictStrategy.kEpochLfu)
    with pytest.raises(H.HkvException):  # epoch never set
        elfu.insert_or_assign(2, k, v, s)
    # ignore_evict_strategy runs the Customized rule instead
    lru.insert_or_assign(2, k, v, s, ignore_evict_strategy=True)
    assert lru.size() == 2


def test_options_checks():
    """init option checks, hkv_hashtable.h:991-1008."""
    t = H.HashTable()
    with pytest.raises(H.HkvException):  # bucket size not a power of two
        t.init(H.HashTableOptions(init_capacity=1024, max_capacity=1024, dim=4,
                                  max_bucket_size=100))
    t = H.HashTable()
    with pytest.raises(H.HkvUnsupported):  # valid there, 128 only here
        t.init(H.HashTableOptions(init_capacity=1024, max_capacity=1024, dim=4,
                                  max_bucket_size=64))


def test_empty_batches_and_capacity_rule():
    t = make_table(1000, dim=4, max_capacity=1000)
    # init*2 > max: ceil(max/128) buckets (table.h:301-303)
    assert t.capacity() == 1024 and t.bucket_count() == 8
    g = GpuOps(t, 4)
    g.insert_or_assign(np.zeros(0, np.uint64), np.zeros((0, 4), np.float32),
                       np.zeros(0, np.uint64))
    assert t.size() == 0
    t2 = make_table(128 * 5, dim=4, max_capacity=128 * 1000)
    # init*2 <= max: power of two buckets >= init (table.h:304-309)
    assert t2.bucket_count() == 8


def test_non_power_of_two_capacity():
    """Capacity = ceil(max/128)*128 need not be a power of two; hashed %
    capacity uses the magic-number division (table.h:106-127)."""
    from hkv_oracle import OracleTable, CUSTOMIZED
    rng = np.random.default_rng(8)
    cap = 128 * 100
    g = GpuOps(make_table(cap, dim=4, max_capacity=cap), 4)
    o = OracleTable(cap, cap, dim=4, strategy=CUSTOMIZED)
    keys = random_keys(rng, 9000)
    vals = rng.random((9000, 4)).astype(np.float32)
    sc = rng.integers(1, 1 << 30, 9000).astype(np.uint64)
    g.insert_or_assign(keys, vals, sc)
    o.insert_or_assign(keys, vals, sc)
    _, f, _ = g.find(keys)
    _, of, _ = o.find(keys)
    assert g.t.capacity() == cap and (f == of).all()


def test_hybrid_values_in_host_memory():
    """max_hbm_for_vectors smaller than the values: later slices live in
    mapped pinned host memory (table.h:143-184) and are read zero-copy."""
    from hkv_oracle import OracleTable, CUSTOMIZED
    rng = np.random.default_rng(9)
    cap, dim = 128 * 4096, 32
    bucket_bytes = 128 * dim * 4
    t = make_table(cap, dim=dim, max_hbm=bucket_bytes * 1024)
    assert not t.is_pure_hbm_mode()
    g = GpuOps(t, dim)
    o = OracleTable(cap, cap, dim=dim, strategy=CUSTOMIZED, threads=8)
    keys = random_keys(rng, 300000)
    vals = rng.random((len(keys), dim)).astype(np.float32)
    sc = rng.integers(1, 1 << 40, len(keys)).astype(np.uint64)
    g.insert_or_assign(keys, vals, sc)
    o.insert_or_assign(keys, vals, sc)
    gv, gf, gs = g.find(keys)
    ov, of, os_ = o.find(keys)
    assert (gf == of).all() and (gv[gf] == ov[of]).all() and (gs[gf] == os_[of]).all()
    # insert_and_evict is refused outside pure-HBM mode (hkv_hashtable.h:1293-1295)
    with pytest.raises(RuntimeError):
        g.insert_and_evict(keys[:10], vals[:10], sc[:10])


def test_lock_wait_times_out_with_error():
    """A slot left LOCKED (planted by the test) makes accum_or_assign's wait
    run out after ~1 s: the call reports HkvTimeout instead of hanging, and
    the table stays usable once the slot is released."""
    rng = np.random.default_rng(10)
    cap, dim = 128 * 4, 4
    g = GpuOps(make_table(cap, dim=dim, strategy=H.EvictStrategy.kLru), dim)
    k = keys_for_bucket(rng, cap, 0, 1)
    g.insert_or_assign(k, np.ones((1, dim), np.float32))
    keys, scores, digests, sizes, values = g.t.get_state()
    slot = int(np.nonzero(keys == k[0])[0][0])
    keys[slot] = np.uint64(0xFFFFFFFFFFFFFFFD)  # LOCKED_KEY
    g.t.set_state(keys=keys)
    t0 = time.time()
    g.t.accum_or_assign(1, dev(k), dev(np.ones((1, dim), np.float32)),
                        dev(np.array([True])), None)
    with pytest.raises(H.HkvTimeout):
        g.t.check_device_error()
    assert time.time() - t0 < 30
    keys[slot] = k[0]
    g.t.set_state(keys=keys)
    g.t.check_device_error()
    g.accum_or_assign(k, np.ones((1, dim), np.float32), np.array([True]))
    v, f, _ = g.find(k)
    assert f[0] and (v[0] == 2).all()


def test_half_values_accum():
    g = GpuOps(make_table(128 * 8, dim=8, strategy=H.EvictStrategy.kLru,
                          value_dtype="float16"), 8, np.float16)
    k = np.array([3, 4], np.uint64)
    g.insert_or_assign(k, np.full((2, 8), 1.5, np.float16))
    g.accum_or_assign(k, np.full((2, 8), 0.25, np.float16), np.array([True, True]))
    v, f, _ = g.find(k)
    assert f.all() and (v == np.float16(1.75)).all()


def test_int64_keys():
    t = make_table(128 * 8, dim=4, strategy=CUST, key_dtype="int64")
    keys = torch.tensor([-5, 7, -(2 ** 62)], dtype=torch.int64, device="cuda")
    t.insert_or_assign(3, keys, torch.ones((3, 4), device="cuda"),
                       torch.tensor([1, 2, 3], dtype=torch.int64, device="cuda"))
    f = torch.zeros(3, dtype=torch.bool, device="cuda")
    t.contains(3, keys, f)
    assert f.all().item()


def test_api_lock_serialises_host_threads():
    """options.api_lock (reference group_lock.h): inserts from several host
    threads on their own streams, with finds running beside them, give the
    table that one thread would build."""
    import threading

    dim, cap = 8, 128 * 256
    t = H.HashTable(H.EvictStrategy.kLru)
    t.init(H.HashTableOptions(init_capacity=cap, max_capacity=cap,
                              max_hbm_for_vectors=1 << 30, dim=dim, api_lock=True))
    rng = np.random.default_rng(77)
    keys = np.unique(rng.integers(1, 1 << 62, 40000, dtype=np.uint64))[:16000]
    vals = rng.standard_normal((len(keys), dim)).astype(np.float32)
    parts = np.array_split(np.arange(len(keys)), 4)
    errors = []

    def writer(idx):
        try:
            s = torch.cuda.Stream()
            for chunk in np.array_split(idx, 8):
                t.insert_or_assign(len(chunk), dev(keys[chunk]), dev(vals[chunk]), stream=s)
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    def reader():
        try:
            s = torch.cuda.Stream()
            out = torch.zeros((4000, dim), device="cuda")
            f = torch.zeros(4000, dtype=torch.bool, device="cuda")
            for _ in range(8):
                t.find(4000, dev(keys[:4000]), out, f, stream=s)
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    th = [threading.Thread(target=writer, args=(p,)) for p in parts]
    th += [threading.Thread(target=reader) for _ in range(2)]
    for x in th:
        x.start()
    for x in th:
        x.join(timeout=120)
    assert not errors and not any(x.is_alive() for x in th)
    torch.cuda.synchronize()
    assert t.size() == len(keys)
    v, f, _ = GpuOps(t, dim).find(keys)
    assert f.all() and (v == vals).all()
