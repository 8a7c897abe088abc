"""The reference's bucket walks on the GPU, on layouts where they decide the
result.

find_without_lock (find_utils.h:31-86) visits groups of four slots from the
key's start group; inside a group digest hits come before empty slots, and
empties before the start position count only after the walk wraps. A
digest-empty slot holding EMPTY_KEY reached before a key's slot ends a lookup
(find, find*, contains, assign_scores). The unique-key upserts
(insert_or_assign_kernel.h:105-183, find_or_insert_kernel.h:100-179,
insert_and_evict_kernel.h:419-496) walk the same groups and claim such an
EMPTY slot before they reach the key, placing a second copy. find_and_lock
(find_utils.h:94-147, accum_or_assign) walks 32-slot windows from the start
position: a key in a later window than an EMPTY slot is not reached. erase
(remove_kernel.h:79-110) tombstones the first holder of the key in every
group, so it removes both copies.

The public API never empties a slot in front of a placed key, so the tests
plant one: a displaced key's start slot is emptied (key word, digest, score
and the bucket's size) through the raw-state entry point, and every
operation is compared with the oracle on that state, slot for slot."""
import numpy as np
import pytest
import torch

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import GpuOps, dev, host, make_table
from hkv_testutil import keys_for_bucket, murmur3_np, one_key_per_bucket

pytestmark = pytest.mark.gpu

EMPTY = np.uint64(0xFFFFFFFFFFFFFFFF)
RESERVED = np.uint64(0xFFFFFFFFFFFFFFFC)


def digest_of(k):
    return np.uint8((int(murmur3_np(np.array([k], np.uint64))[0]) >> 32) & 0xFF)


def start_of(k):
    return int(murmur3_np(np.array([k], np.uint64))[0]) & 127


def planted(rng, cap, dim, bucket=3, nkeys=100, min_lin=0):
    """A bucket of nkeys keys with the start slot of one displaced key emptied.
    The hidden key sits in a later group than its start slot, at least min_lin
    slots after it. Returns the table, its oracle copy, the bucket's remaining
    keys, the hidden key and the emptied slot."""
    nb = cap // 128
    for b in [bucket] + [x for x in range(nb) if x != bucket]:
        g = GpuOps(make_table(cap, dim=dim, strategy=H.EvictStrategy.kCustomized), dim)
        ks = keys_for_bucket(rng, cap, b, nkeys)
        g.insert_or_assign(ks, rng.standard_normal((nkeys, dim)).astype(np.float32),
                           rng.integers(1, 1 << 30, nkeys).astype(np.uint64))
        keys, scores, digests, sizes, values = g.t.get_state()
        base = b * 128
        hidden = None
        for q in range(128):
            k = keys[base + q]
            if k >= RESERVED:
                continue
            p = start_of(k)
            # a later group than the start slot, which holds another key
            if ((q >> 2) - (p >> 2)) & 31 and (q - p) & 127 >= min_lin \
                    and keys[base + p] < RESERVED:
                hidden, e = k, p
                break
        if hidden is not None:
            break
    assert hidden is not None
    gone = keys[base + e]
    keys[base + e] = EMPTY
    digests[base + e] = digest_of(EMPTY)
    scores[base + e] = 0
    sizes[b] -= 1
    g.t.set_state(keys=keys, scores=scores, digests=digests, sizes=sizes)
    o = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED, threads=1)
    keys, scores, digests, sizes, values = g.t.get_state()
    o.set_state(keys, scores, digests, sizes, np.ascontiguousarray(values))
    rest = ks[ks != gone]
    return g, o, rest, hidden, base + e


def same_state(g, o):
    gk, gs, gd, gz, gv = g.t.get_state()
    ok, os_, od, oz, ov = o.get_state()
    assert (gk == ok).all() and (gd == od).all() and (gz == oz).all()
    live = gk < RESERVED
    assert (gs[live] == os_[live]).all()
    assert (gv[live] == ov[live]).all()


def test_lookups_stop_at_a_planted_empty_slot():
    rng = np.random.default_rng(201)
    cap, dim = 128 * 8, 4
    g, o, rest, hidden, _ = planted(rng, cap, dim)
    gv, gf, gs = g.find(rest)
    ov, of, os_ = o.find(rest)[:3]
    np.testing.assert_array_equal(gf, of)
    assert not gf[rest == hidden].any()  # the rule did apply
    np.testing.assert_array_equal(gv[gf], ov[of])
    np.testing.assert_array_equal(gs[gf], os_[of])
    np.testing.assert_array_equal(g.contains(rest), of)
    # find* (reference find_ptr_with_digest_kernel.h) walks the same way
    n = len(rest)
    ptrs = torch.zeros(n, dtype=torch.int64, device="cuda")
    pf = torch.zeros(n, dtype=torch.bool, device="cuda")
    g.t.find_ptr(n, dev(rest), ptrs, pf)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(pf).astype(bool), of)
    assert ((host(ptrs) != 0) == of).all()


def test_assign_scores_applies_the_stop_rule():
    rng = np.random.default_rng(202)
    cap, dim = 128 * 8, 4
    g, o, rest, hidden, _ = planted(rng, cap, dim)
    sc = rng.integers(1, 1 << 30, len(rest)).astype(np.uint64)
    g.assign_scores(rest, sc)
    o.assign_scores(rest, sc)
    same_state(g, o)
    keys, scores = g.t.get_state()[:2]
    slot = int(np.nonzero(keys == hidden)[0][0])
    assert scores[slot] != sc[rest == hidden][0]  # hidden key left alone


def test_accum_and_erase_walk_the_whole_bucket():
    rng = np.random.default_rng(203)
    cap, dim = 128 * 8, 4
    g, o, rest, hidden, _ = planted(rng, cap, dim)
    delta = rng.standard_normal((len(rest), dim)).astype(np.float32)
    acc = np.ones(len(rest), bool)
    sc = rng.integers(1, 1 << 30, len(rest)).astype(np.uint64)
    before = g.t.get_state()
    g.accum_or_assign(rest, delta, acc, sc)
    o.accum_or_assign(rest, delta, acc.astype(np.uint8), sc)
    same_state(g, o)
    slot = int(np.nonzero(before[0] == hidden)[0][0])
    assert (g.t.get_state()[4][slot] != before[4][slot]).any()  # walked past the empty slot
    g.erase(rest[::2])
    o.erase(rest[::2])
    same_state(g, o)
    g.t.check_device_error()


def copies(g, key):
    return np.nonzero(g.t.get_state()[0] == np.uint64(key))[0]


@pytest.mark.parametrize("op", ["insert_or_assign", "find_or_insert", "insert_and_evict"])
def test_upserts_claim_an_empty_slot_ahead_of_the_key(op):
    """The group walk reaches the emptied start slot before the hidden key's
    own slot: the upsert places a second copy there, as the reference does.
    A second call then finds that copy first (its group comes first), and
    erase removes both copies."""
    rng = np.random.default_rng({"insert_or_assign": 211, "find_or_insert": 212,
                                 "insert_and_evict": 213}[op])
    cap, dim = 128 * 8, 4
    g, o, rest, hidden, e = planted(rng, cap, dim)
    old_slot = int(copies(g, hidden)[0])
    # the hidden key and fresh keys of the other buckets (no contention)
    others = one_key_per_bucket(rng, cap, [b for b in range(cap // 128) if b != e // 128],
                                exclude=rest)
    batch = np.concatenate([[hidden], others]).astype(np.uint64)
    vals = rng.standard_normal((len(batch), dim)).astype(np.float32)
    sc = rng.integers(1, 1 << 30, len(batch)).astype(np.uint64)
    if op == "insert_or_assign":
        g.insert_or_assign(batch, vals, sc)
        o.insert_or_assign(batch, vals, sc)
    elif op == "find_or_insert":
        gv = g.find_or_insert(batch, vals, sc)
        ov, _ = o.find_or_insert(batch, vals, sc)
        np.testing.assert_array_equal(gv, ov)
        np.testing.assert_array_equal(gv[0], vals[0])  # inserted, not read back
    else:
        gk, gv, gs = g.insert_and_evict(batch, vals, sc)
        ok, ov, os_, _ = o.insert_and_evict(batch, vals, sc)
        assert len(gk) == len(ok) == 0
        torch.cuda.synchronize()
    same_state(g, o)
    assert sorted(copies(g, hidden).tolist()) == sorted([e, old_slot])
    # the copy in the start group is now the first the walk reaches
    vals2 = rng.standard_normal((1, dim)).astype(np.float32)
    sc2 = np.array([7], np.uint64)
    g.insert_or_assign(batch[:1], vals2, sc2)
    o.insert_or_assign(batch[:1], vals2, sc2)
    same_state(g, o)
    gv, gf, gs = g.find(batch[:1])
    assert gf[0] and (gv[0] == vals2[0]).all() and gs[0] == 7
    sc3 = np.array([9], np.uint64)
    g.assign_scores(batch[:1], sc3)
    o.assign_scores(batch[:1], sc3)
    same_state(g, o)
    size0 = g.t.size()
    g.erase(batch[:1])
    o.erase(batch[:1])
    same_state(g, o)
    assert len(copies(g, hidden)) == 0 and g.t.size() == size0 - 2
    g.t.check_device_error()


def test_accum_window_walk_claims_an_earlier_empty_slot():
    """find_and_lock's 32-slot windows: the hidden key lies at least one window
    after its emptied start slot, so an accumulate claims the empty slot,
    finds it is not the key and gives it back (nothing accumulates), and an
    assign places a second copy there, both as in the oracle."""
    rng = np.random.default_rng(221)
    cap, dim = 128 * 8, 4
    g, o, rest, hidden, e = planted(rng, cap, dim, nkeys=124, min_lin=36)
    before = g.t.get_state()
    d = rng.standard_normal((1, dim)).astype(np.float32)
    sc = np.array([5], np.uint64)
    g.accum_or_assign([hidden], d, [True], sc)
    o.accum_or_assign([hidden], d, np.array([1], np.uint8), sc)
    same_state(g, o)
    np.testing.assert_array_equal(g.t.get_state()[4], before[4])  # nothing added
    g.accum_or_assign([hidden], d, [False], sc)
    o.accum_or_assign([hidden], d, np.array([0], np.uint8), sc)
    same_state(g, o)
    assert e in copies(g, hidden).tolist() and len(copies(g, hidden)) == 2
    # the keys of the bucket that do not pass the emptied slot accumulate
    near = np.array([k for k in rest if ((np.nonzero(before[0] == k)[0][0] % 128)
                                          - start_of(k)) % 128 < 32
                     and not (0 < (e % 128 - start_of(k)) % 128 < 32)], np.uint64)
    dd = rng.standard_normal((len(near), dim)).astype(np.float32)
    scn = rng.integers(1, 1 << 30, len(near)).astype(np.uint64)
    g.accum_or_assign(near, dd, np.ones(len(near), bool), scn)
    o.accum_or_assign(near, dd, np.ones(len(near), np.uint8), scn)
    same_state(g, o)
    g.t.check_device_error()
