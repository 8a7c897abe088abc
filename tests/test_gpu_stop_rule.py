"""The find rule's stop condition on the GPU (reference find_utils.h:58-66):
a digest-empty slot holding EMPTY_KEY that the bucket walk reaches before a
key's slot ends the walk, so lookups do not see that key. The walk visits
groups of four slots from the key's start group; inside a group, digest hits
come before empty slots, and empties before the start position count only
after the walk wraps.

Only a layout the public API does not produce (a key placed behind a slot
that later turns EMPTY) exercises the rule, so the test plants it: one slot
in front of a displaced key is emptied (key word, digest, score and the
bucket's size), then find, contains, assign_scores (which applies the rule),
accum_or_assign and erase (which do not, like the reference's
accum_or_assign_kernel.h / remove_kernel.h walks) are compared with the
oracle on that state."""
import numpy as np
import pytest
import torch

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import GpuOps, dev, host, make_table
from hkv_testutil import keys_for_bucket, murmur3_np

pytestmark = pytest.mark.gpu

EMPTY = np.uint64(0xFFFFFFFFFFFFFFFF)
RESERVED = np.uint64(0xFFFFFFFFFFFFFFFC)


def digest_of(k):
    return np.uint8((int(murmur3_np(np.array([k], np.uint64))[0]) >> 32) & 0xFF)


def planted(rng, cap, dim, bucket=3):
    """A bucket of 100 keys with the start slot of one displaced key emptied.
    Returns the table, its oracle copy, the bucket's remaining keys and the
    key hidden behind the planted slot."""
    g = GpuOps(make_table(cap, dim=dim, strategy=H.EvictStrategy.kCustomized), dim)
    ks = keys_for_bucket(rng, cap, bucket, 100)
    g.insert_or_assign(ks, rng.standard_normal((100, dim)).astype(np.float32),
                       rng.integers(1, 1 << 30, 100).astype(np.uint64))
    keys, scores, digests, sizes, values = g.t.get_state()
    base = bucket * 128
    hidden = None
    for q in range(128):
        k = keys[base + q]
        if k >= RESERVED:
            continue
        p = int(murmur3_np(np.array([k], np.uint64))[0]) & 127
        # the key sits in a later group than its start slot, and the start
        # slot holds another key (which the plant removes)
        if ((q >> 2) - (p >> 2)) & 31 and keys[base + p] < RESERVED:
            hidden, e = k, p
            break
    assert hidden is not None
    gone = keys[base + e]
    keys[base + e] = EMPTY
    digests[base + e] = digest_of(EMPTY)
    scores[base + e] = 0
    sizes[bucket] -= 1
    g.t.set_state(keys=keys, scores=scores, digests=digests, sizes=sizes)
    o = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED, threads=1)
    keys, scores, digests, sizes, values = g.t.get_state()
    o.set_state(keys, scores, digests, sizes, np.ascontiguousarray(values))
    rest = ks[ks != gone]
    return g, o, rest, hidden


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
    g, o, rest, hidden = planted(rng, cap, dim)
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
    g, o, rest, hidden = planted(rng, cap, dim)
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
    g, o, rest, hidden = planted(rng, cap, dim)
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
