"""CUDA table vs the CPU oracle on the same seeded inputs (GPU).

Exactness rules:
* find / contains / export: bit-exact (export as a set);
* a batch whose keys touch distinct buckets: the whole raw table state
  (keys, scores, digests, bucket sizes, values) is bit-identical slot by slot
  to the oracle run from the same starting state (imported from the GPU);
* batches with several keys per bucket under Customized scores: the set of
  live (key, score, value) is identical (per bucket it is the streaming
  top-128, which does not depend on the order of the keys).
"""
import numpy as np
import pytest
import torch

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import GpuOps, dev, host, make_table
from hkv_testutil import bucket_of, live_set, one_key_per_bucket, random_keys

pytestmark = pytest.mark.gpu

STRATS = {"customized": (H.EvictStrategy.kCustomized, O.CUSTOMIZED),
          "lfu": (H.EvictStrategy.kLfu, O.LFU),
          "epoch_lfu": (H.EvictStrategy.kEpochLfu, O.EPOCH_LFU)}


def oracle_from_gpu(g, cap, dim, ostrat, epoch=None, max_capacity=None, lf=0.5):
    o = O.OracleTable(cap, max_capacity or cap, dim=dim, strategy=ostrat,
                      max_load_factor=lf, threads=8)
    if epoch is not None:
        o.set_global_epoch(epoch)
    keys, scores, digests, sizes, values = g.t.get_state()
    o.set_state(keys, scores, digests, sizes, np.ascontiguousarray(values))
    return o


def assert_same_state(g, o, compare_scores=True):
    gk, gs, gd, gz, gv = g.t.get_state()
    ok, os_, od, oz, ov = o.get_state()
    assert (gk == ok).all(), f"keys differ at {np.nonzero(gk != ok)[0][:8]}"
    assert (gd == od).all(), f"digests differ at {np.nonzero(gd != od)[0][:8]}"
    assert (gz == oz).all(), f"sizes differ at {np.nonzero(gz != oz)[0][:8]}"
    live = gk < np.uint64(0xFFFFFFFFFFFFFFFC)
    assert (gv[live] == ov[live]).all()
    if compare_scores:
        assert (gs[live] == os_[live]).all(), f"scores differ at {np.nonzero((gs != os_) & live)[0][:8]}"


def test_smoke_find_after_insert():
    rng = np.random.default_rng(1)
    g = GpuOps(make_table(128 * 64, dim=8), 8)
    keys = random_keys(rng, 3000)
    vals = rng.random((3000, 8)).astype(np.float32)
    sc = rng.integers(1, 1 << 40, 3000).astype(np.uint64)
    g.insert_or_assign(keys, vals, sc)
    v, f, s = g.find(keys)
    o = O.OracleTable(128 * 64, dim=8, strategy=O.CUSTOMIZED)
    o.insert_or_assign(keys, vals, sc)
    ov, of, os_ = o.find(keys)
    assert (f == of).all()
    assert (v[f] == ov[of]).all() and (s[f] == os_[of]).all()
    g.t.check_device_error()


def test_config1_customized_parity():
    """1Mi slots (8192 buckets), dim 8, Customized;
    16 x 65,536 insert_or_assign, find of 65,536 keys (half resident, half
    fresh), export_batch."""
    rng = np.random.default_rng(20261201)
    cap, dim, batch = 1 << 20, 8, 65536
    g = GpuOps(make_table(cap, dim=dim), dim)
    o = O.OracleTable(cap, dim=dim, strategy=O.CUSTOMIZED, threads=8)
    allk = random_keys(rng, 16 * batch)
    for b in range(16):
        k = allk[b * batch:(b + 1) * batch]
        v = rng.random((batch, dim)).astype(np.float32)
        s = rng.integers(0, 1 << 63, batch, dtype=np.uint64)
        g.insert_or_assign(k, v, s)
        o.insert_or_assign(k, v, s)
    gs = live_set(*[x for i, x in enumerate(g.t.get_state()) if i != 2 and i != 3])
    os_ = live_set(*[x for i, x in enumerate(o.get_state()) if i != 2 and i != 3])
    assert len(gs) == len(os_) == g.t.size() == o.size()
    assert gs == os_
    resident = np.array(sorted(os_.keys()), np.uint64)
    q = np.concatenate([rng.choice(resident, batch // 2, replace=False),
                        random_keys(np.random.default_rng(99), batch // 2, lo=1 << 63,
                                    hi=(1 << 64) - 8)])
    rng.shuffle(q)
    gv, gf, gsc = g.find(q, init_value=-7.0)
    ov = np.full((len(q), dim), -7.0, np.float32)
    ov, of, osc = o.find(q, values=ov)
    assert (gf == of).all() and gf.sum() == batch // 2
    assert (gv == ov).all()  # misses keep the caller's values
    assert (gsc[gf] == osc[of]).all()
    ek, ev, es = g.export(cap)
    assert len(ek) == len(os_)
    assert {int(k): (int(s), v.tobytes()) for k, s, v in zip(ek, es, ev)} == os_
    g.t.check_device_error()


@pytest.mark.parametrize("name", list(STRATS))
@pytest.mark.parametrize("tie_scores", [False, True])
def test_exact_state_distinct_buckets(name, tie_scores):
    """Each batch touches each bucket at most once: after every batch the
    GPU state equals the oracle's slot for slot (placement, digests, the
    16-lane victim tie-break, tombstone reuse, score rules)."""
    hs, os_ = STRATS[name]
    rng = np.random.default_rng(7 + tie_scores)
    cap, dim = 128 * 64, 4
    epoch = 5 if name == "epoch_lfu" else None
    g = GpuOps(make_table(cap, dim=dim, strategy=hs, epoch=epoch), dim)
    # fill with contention (several keys per bucket) up to full buckets
    pre = random_keys(rng, int(cap * 1.3))
    hi = 4 if tie_scores else 1 << 40
    for part in np.array_split(pre, 4):
        g.insert_or_assign(part, rng.random((len(part), dim)).astype(np.float32),
                           rng.integers(1, hi, len(part)).astype(np.uint64))
    g.erase(pre[:200])  # tombstones
    o = oracle_from_gpu(g, cap, dim, os_, epoch)
    assert_same_state(g, o)
    nb = cap // 128
    resident = o.get_state()[0]
    resident = resident[resident < np.uint64(0xFFFFFFFFFFFFFFFC)]
    for step in range(3):
        buckets = rng.permutation(nb)
        fresh = one_key_per_bucket(rng, cap, buckets[: nb // 2])
        hits = []
        for b in buckets[nb // 2:]:
            r = resident[bucket_of(resident, cap) == np.uint64(b)]
            if len(r):
                hits.append(r[rng.integers(len(r))])
        keys = np.concatenate([fresh, np.array(hits, np.uint64)])
        vals = rng.random((len(keys), dim)).astype(np.float32)
        sc = rng.integers(1, hi, len(keys)).astype(np.uint64)
        g.insert_or_assign(keys, vals, sc)
        o.insert_or_assign(keys, vals, sc)
        assert_same_state(g, o)
        resident = o.get_state()[0]
        resident = resident[resident < np.uint64(0xFFFFFFFFFFFFFFFC)]
    g.t.check_device_error()


def test_exact_state_lru_distinct_buckets():
    """Lru: the oracle clock is set above every stored score, so admission
    and victims match; written scores are device clocks and are checked to
    exceed everything stored before."""
    rng = np.random.default_rng(31)
    cap, dim = 128 * 64, 4
    g = GpuOps(make_table(cap, dim=dim, strategy=H.EvictStrategy.kLru), dim)
    pre = random_keys(rng, int(cap * 1.2))
    for part in np.array_split(pre, 3):
        g.insert_or_assign(part, rng.random((len(part), dim)).astype(np.float32))
    o = oracle_from_gpu(g, cap, dim, O.LRU)
    before = g.t.get_state()[1].max()
    o.set_clock(int(before) + 1)
    nb = cap // 128
    keys = one_key_per_bucket(rng, cap, np.arange(nb))
    vals = rng.random((nb, dim)).astype(np.float32)
    g.insert_or_assign(keys, vals)
    o.insert_or_assign(keys, vals)
    assert_same_state(g, o, compare_scores=False)
    gk, gs = g.t.get_state()[:2]
    written = np.isin(gk, keys)
    assert (gs[written] > before).all()


@pytest.mark.parametrize("name", list(STRATS))
def test_find_or_insert_exact(name):
    hs, os_ = STRATS[name]
    rng = np.random.default_rng(41)
    cap, dim = 128 * 32, 8
    epoch = 9 if name == "epoch_lfu" else None
    g = GpuOps(make_table(cap, dim=dim, strategy=hs, epoch=epoch), dim)
    pre = random_keys(rng, int(cap * 1.1))
    g.insert_or_assign(pre, rng.random((len(pre), dim)).astype(np.float32),
                       rng.integers(1, 1 << 30, len(pre)).astype(np.uint64))
    o = oracle_from_gpu(g, cap, dim, os_, epoch)
    nb = cap // 128
    res = o.get_state()[0]
    res = res[res < np.uint64(0xFFFFFFFFFFFFFFFC)]
    hits = np.array([res[bucket_of(res, cap) == np.uint64(b)][0] for b in range(0, nb, 2)],
                    np.uint64)
    fresh = one_key_per_bucket(rng, cap, np.arange(1, nb, 2))
    keys = np.concatenate([hits, fresh])
    vals = rng.random((len(keys), dim)).astype(np.float32)
    sc = rng.integers(1, 1 << 30, len(keys)).astype(np.uint64)
    gout = g.find_or_insert(keys, vals, sc)
    oout, _ = o.find_or_insert(keys, vals, sc)
    assert (gout == oout).all()
    assert_same_state(g, o)


# dim 8 rows fit the registers of a 4-lane tile and are written out after the
# rounds; dim 64 rows are copied out while the victim's slot is held
@pytest.mark.parametrize("dim", [8, 64])
def test_insert_and_evict_matches_oracle(dim):
    rng = np.random.default_rng(51)
    cap = 128 * 32
    g = GpuOps(make_table(cap, dim=dim), dim)
    pre = random_keys(rng, cap)
    g.insert_or_assign(pre, rng.random((cap, dim)).astype(np.float32),
                       rng.integers(1000, 1 << 30, cap).astype(np.uint64))
    o = oracle_from_gpu(g, cap, dim, O.CUSTOMIZED)
    nb = cap // 128
    keys = one_key_per_bucket(rng, cap, np.arange(nb))
    vals = rng.random((nb, dim)).astype(np.float32)
    sc = np.where(rng.random(nb) < 0.5, rng.integers(0, 999, nb),
                  rng.integers(1 << 31, 1 << 40, nb)).astype(np.uint64)
    gk, gv, gs = g.insert_and_evict(keys, vals, sc)
    ok, ov, os_, _ = o.insert_and_evict(keys, vals, sc)
    assert len(gk) == len(ok) > 0
    assert {int(k): (int(s), v.tobytes()) for k, s, v in zip(gk, gs, gv)} == \
        {int(k): (int(s), v.tobytes()) for k, s, v in zip(ok, os_, ov)}
    assert_same_state(g, o)


@pytest.mark.parametrize("dim", [4, 32, 64])
def test_insert_and_evict_every_key_accounted_lru(dim):
    """tests/test_reserve.cpp:320-420 pattern under contention (LRU, LF -> 1):
    every inserted key is in the table with its value or was reported
    evicted with its value; size matches."""
    rng = np.random.default_rng(61)
    cap, batch = 128 * 256, 8192
    g = GpuOps(make_table(cap, dim=dim, strategy=H.EvictStrategy.kLru), dim)
    live = {}
    for step in range(12):
        keys = random_keys(rng, batch)
        vals = rng.random((batch, dim)).astype(np.float32)
        ek, ev, _ = g.insert_and_evict(keys, vals)
        for k, v in zip(keys.tolist(), vals):
            live[k] = v
        for k, v in zip(ek.tolist(), ev):
            assert (live.pop(k) == v).all()
    keys = np.array(list(live), np.uint64)
    v, f, _ = g.find(keys)
    assert f.all() and g.t.size() == len(live)
    assert (v == np.stack([live[k] for k in keys.tolist()])).all()
    g.t.check_device_error()


# dim 8 and 64: rows added four floats per 16-byte access; dim 5: one float
# at a time. Random float rows: the sums must match the oracle's bit for bit.
@pytest.mark.parametrize("dim", [8, 5, 64])
def test_accum_or_assign_exact(dim):
    rng = np.random.default_rng(71)
    cap = 128 * 32
    g = GpuOps(make_table(cap, dim=dim), dim)
    pre = random_keys(rng, cap // 2)
    g.insert_or_assign(pre, rng.standard_normal((len(pre), dim)).astype(np.float32),
                       rng.integers(1, 1 << 30, len(pre)).astype(np.uint64))
    o = oracle_from_gpu(g, cap, dim, O.CUSTOMIZED)
    nb = cap // 128
    res = pre
    hits = np.array([res[bucket_of(res, cap) == np.uint64(b)][0] for b in range(0, nb, 2)],
                    np.uint64)
    fresh = one_key_per_bucket(rng, cap, np.arange(1, nb, 2))
    keys = np.concatenate([hits, fresh, hits[:5], fresh[:5]])
    vals = rng.standard_normal((len(keys), dim)).astype(np.float32)
    acc = np.concatenate([np.ones(len(hits)), np.zeros(len(fresh)),
                          np.zeros(5), np.ones(5)]).astype(np.uint8)
    # the trailing mismatched entries (assign on existing / accum on new)
    # are no-ops; they share buckets with earlier keys only through keys
    # already processed, so keep them in a second call
    sc = rng.integers(1, 1 << 30, len(keys)).astype(np.uint64)
    m = len(hits) + len(fresh)
    g.accum_or_assign(keys[:m], vals[:m], acc[:m].astype(bool), sc[:m])
    o.accum_or_assign(keys[:m], vals[:m], acc[:m], sc[:m])
    assert_same_state(g, o)
    g.accum_or_assign(keys[m:], vals[m:], acc[m:].astype(bool), sc[m:])
    o.accum_or_assign(keys[m:], vals[m:], acc[m:], sc[m:])
    assert_same_state(g, o)


def test_accum_duplicates_serialise():
    """accum_or_assign has no unique_key flag: duplicate keys of one batch
    each add their delta (the reference serialises them on the key lock)."""
    cap, dim = 128 * 16, 4
    g = GpuOps(make_table(cap, dim=dim, strategy=H.EvictStrategy.kLru), dim)
    k = np.array([5, 6], np.uint64)
    g.insert_or_assign(k, np.zeros((2, dim), np.float32))
    keys = np.repeat(k, 50)
    g.accum_or_assign(keys, np.ones((100, dim), np.float32), np.ones(100, bool))
    v, f, _ = g.find(k)
    assert f.all() and (v == 50).all()
    g.t.check_device_error()


@pytest.mark.parametrize("name", ["customized", "lfu", "epoch_lfu"])
def test_assign_scores_exact(name):
    hs, os_ = STRATS[name]
    rng = np.random.default_rng(81)
    cap, dim = 128 * 32, 4
    epoch = 3 if name == "epoch_lfu" else None
    g = GpuOps(make_table(cap, dim=dim, strategy=hs, epoch=epoch), dim)
    pre = random_keys(rng, cap // 2)
    g.insert_or_assign(pre, np.zeros((len(pre), dim), np.float32),
                       rng.integers(1, 1 << 20, len(pre)).astype(np.uint64))
    o = oracle_from_gpu(g, cap, dim, os_, epoch)
    q = np.concatenate([pre[::3], random_keys(rng, 500, lo=1 << 62)])
    sc = rng.integers(1, 1 << 20, len(q)).astype(np.uint64)
    g.assign_scores(q, sc)
    o.assign_scores(q, sc)
    assert_same_state(g, o)


def test_erase_exact():
    rng = np.random.default_rng(91)
    cap, dim = 128 * 32, 4
    g = GpuOps(make_table(cap, dim=dim), dim)
    pre = random_keys(rng, cap)
    g.insert_or_assign(pre, np.zeros((cap, dim), np.float32),
                       rng.integers(1, 1 << 20, cap).astype(np.uint64))
    o = oracle_from_gpu(g, cap, dim, O.CUSTOMIZED)
    q = np.concatenate([pre[::2], random_keys(rng, 500, lo=1 << 62)])
    g.erase(q)
    o.erase(q)
    assert_same_state(g, o)
    assert g.t.size() == o.size()
    assert not g.contains(pre[::2]).any()


def test_contains_and_reserved_keys():
    rng = np.random.default_rng(101)
    g = GpuOps(make_table(128 * 16, dim=4), 4)
    keys = random_keys(rng, 1000)
    g.insert_or_assign(keys, np.zeros((1000, 4), np.float32), np.ones(1000, np.uint64))
    res = np.array([0xFFFFFFFFFFFFFFFC, 0xFFFFFFFFFFFFFFFD, 0xFFFFFFFFFFFFFFFE,
                    0xFFFFFFFFFFFFFFFF], np.uint64)
    g.insert_or_assign(res, np.ones((4, 4), np.float32), np.ones(4, np.uint64))
    assert g.t.size() == 1000
    assert g.contains(keys).all() and not g.contains(res).any()
    _, f, _ = g.find(res)
    assert not f.any()


def test_export_batch_offsets_and_counter():
    rng = np.random.default_rng(111)
    cap, dim = 128 * 1024, 8
    g = GpuOps(make_table(cap, dim=dim, strategy=H.EvictStrategy.kLru), dim)
    assert len(g.export(cap)[0]) == 0
    keys = np.arange(1, 5001, dtype=np.uint64)
    vals = (keys.astype(np.float64) * 1e-5).astype(np.float32)[:, None].repeat(dim, 1)
    g.insert_or_assign(keys, vals)
    o = oracle_from_gpu(g, cap, dim, O.LRU)
    ek, ev, _ = g.export(cap)
    assert len(ek) == 5000 and set(ek.tolist()) == set(keys.tolist())
    ref = {int(k): v for k, v in zip(keys, vals)}
    assert all((ref[int(k)] == v).all() for k, v in zip(ek, ev))
    for off, n in [(cap // 2, cap), (1000, 3000), (cap - 7, 100), (cap, 10)]:
        gk, gv, gs = g.export(n, off)
        ok, ov, os_ = o.export_batch(n, off)
        assert sorted(gk.tolist()) == sorted(ok.tolist())
    # device-counter overload sets (not accumulates) the counter
    d = torch.full((1,), 12345, dtype=torch.int64, device="cuda")
    k = torch.zeros(cap, dtype=torch.int64, device="cuda")
    v = torch.zeros((cap, dim), dtype=torch.float32, device="cuda")
    g.t.export_batch(cap, 0, k, v, None, d_counter=d)
    torch.cuda.synchronize()
    assert int(d.item()) == 5000


@pytest.mark.parametrize("nb,erased", [(64, 300), (4096, 20000)])
def test_reserve_exact_layout(nb, erased):
    """reserve doubles the buckets and rehashes with the reference's
    algorithm (rehash_kernel.h:30-207): the GPU layout after reserve equals
    the oracle's slot for slot, from the same starting state (reclaimed
    slots of erased keys included)."""
    rng = np.random.default_rng(121 + nb)
    cap, dim = 128 * nb, 4
    g = GpuOps(make_table(cap, dim=dim, max_capacity=cap * 8, max_load_factor=1.0), dim)
    pre = random_keys(rng, int(cap * 0.9))
    g.insert_or_assign(pre, rng.random((len(pre), dim)).astype(np.float32),
                       rng.integers(1, 1 << 30, len(pre)).astype(np.uint64))
    g.erase(pre[:erased])
    o = oracle_from_gpu(g, cap, dim, O.CUSTOMIZED, max_capacity=cap * 8, lf=1.0)
    present = pre[g.contains(pre)]  # the batch overfilled some buckets
    g.t.reserve(cap * 4)
    o.reserve(cap * 4)
    assert g.t.capacity() == o.capacity() == cap * 4
    assert_same_state(g, o)
    assert g.contains(present).all()


@pytest.mark.parametrize("dim", [5, 33, 136])
def test_reserve_rows_of_any_width(dim):
    """reserve's row moves at row widths that take each copy path of the
    rehash: 20-byte rows (4-byte vectors, several rows per warp pass),
    132-byte rows (33 vectors) and 544-byte rows (34 16-byte vectors), the
    latter two a warp per row; two doublings, the second in place; layout
    and values equal the oracle's slot for slot."""
    rng = np.random.default_rng(700 + dim)
    cap = 128 * 32
    g = GpuOps(make_table(cap, dim=dim, max_capacity=cap * 4, max_load_factor=1.0), dim)
    pre = random_keys(rng, int(cap * 0.9))
    g.insert_or_assign(pre, rng.standard_normal((len(pre), dim)).astype(np.float32),
                       rng.integers(1, 1 << 30, len(pre)).astype(np.uint64))
    g.erase(pre[:200])
    o = oracle_from_gpu(g, cap, dim, O.CUSTOMIZED, max_capacity=cap * 4, lf=1.0)
    g.t.reserve(cap * 4)
    o.reserve(cap * 4)
    assert g.t.capacity() == o.capacity() == cap * 4
    assert_same_state(g, o)


def test_reserve_into_host_slices():
    """BASELINE config 4's reserve, scaled down: max_hbm_for_vectors holds
    exactly the first value slice, so the slices a doubling appends go to
    mapped pinned host memory (table.h:143-184, :360-377;
    hkv_hashtable.h:2873-2935), low bucket indices keep HBM. The layout after
    reserve equals the oracle's slot for slot, values included, and every
    key reads back its row through find."""
    rng = np.random.default_rng(133)
    cap, dim = 128 * 64, 4
    bucket_bytes = 128 * dim * 4
    g = GpuOps(make_table(cap, dim=dim, max_capacity=cap * 8, max_load_factor=1.0,
                          max_hbm=bucket_bytes * 64), dim)
    assert g.t.is_pure_hbm_mode()  # the initial buckets fit
    pre = random_keys(rng, int(cap * 0.95))
    vals = rng.random((len(pre), dim)).astype(np.float32)
    g.insert_or_assign(pre, vals, rng.integers(1, 1 << 30, len(pre)).astype(np.uint64))
    o = oracle_from_gpu(g, cap, dim, O.CUSTOMIZED, max_capacity=cap * 8, lf=1.0)
    present = pre[g.contains(pre)]
    g.t.reserve(cap * 4)
    o.reserve(cap * 4)
    assert g.t.capacity() == o.capacity() == cap * 4
    assert not g.t.is_pure_hbm_mode()  # the appended slices are host memory
    assert_same_state(g, o)
    got, f, _ = g.find(present)
    ov, of, _ = o.find(present)
    assert f.all() and of.all() and (got == ov).all()
    # rows in host slices are written through too
    newk = random_keys(rng, 2000, lo=1 << 62)
    nv = rng.random((2000, dim)).astype(np.float32)
    g.insert_or_assign(newk, nv, np.full(2000, 1 << 31, np.uint64))
    o.insert_or_assign(newk, nv, np.full(2000, 1 << 31, np.uint64))
    gk, gs, _, gz, gvals = g.t.get_state()
    ok, os_, _, oz, ovals = o.get_state()
    assert (gz == oz).all()  # several keys per bucket: compare the live set, not slots
    assert live_set(gk, gs, gvals) == live_set(ok, os_, ovals)


def test_reserve_full_table():
    """tests/test_reserve.cpp:193-300: a full table doubles to LF 0.5 with
    every key still found."""
    rng = np.random.default_rng(131)
    cap, dim = 128 * 128, 4
    g = GpuOps(make_table(cap, dim=dim, max_capacity=cap * 2, max_load_factor=1e30,
                          strategy=H.EvictStrategy.kLru), dim)
    for _ in range(5):
        g.insert_or_assign(random_keys(rng, cap), np.ones((cap, dim), np.float32))
    assert g.t.size() == cap
    gk = g.t.get_state()[0]
    live = gk[gk < np.uint64(0xFFFFFFFFFFFFFFFC)]
    o = oracle_from_gpu(g, cap, dim, O.LRU, max_capacity=cap * 2, lf=1e30)
    g.t.reserve(cap + 1)
    o.reserve(cap + 1)
    assert g.t.capacity() == cap * 2 and abs(g.t.load_factor() - 0.5) < 1e-7
    assert g.contains(live).all()
    assert_same_state(g, o)


def test_auto_grow_matches_oracle():
    """Insert-like calls grow the table while fast_load_factor exceeds
    max_load_factor (hkv_hashtable.h:1103-1106, :3229-3268)."""
    rng = np.random.default_rng(141)
    init, dim = 128 * 16, 4
    g = GpuOps(make_table(init, dim=dim, max_capacity=init * 64), dim)
    o = O.OracleTable(init, init * 64, dim=dim, strategy=O.CUSTOMIZED)
    for step in range(8):
        k = random_keys(rng, 1500)
        v = rng.random((1500, dim)).astype(np.float32)
        s = rng.integers(1, 1 << 30, 1500).astype(np.uint64)
        g.insert_or_assign(k, v, s)
        o.insert_or_assign(k, v, s)
        assert g.t.capacity() == o.capacity()
        assert g.t.size() == o.size()
