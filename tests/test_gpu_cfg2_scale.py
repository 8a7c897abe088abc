"""Parity at the headline's full shape (64 Mi slots,
dim 32, kLru, load factor 1.0, 1 Mi-key batches), on the GPU.

The table is filled to load factor 1.0 on the GPU, its raw state is imported
into the oracle, and a 1 Mi-key find (half resident keys, half never
inserted) must agree bit for bit: flags, value rows and scores. Then one
insert_or_assign batch of 1 Mi keys (half resident, half new, every new key
evicting) is checked by the invariants that do not depend on thread order:
the table stays full, every input key is present with its input row, no slot
is left LOCKED, no key has two copies, and the keys that left are exactly
resident keys that were not in the batch, one per new key."""
import numpy as np
import pytest
import torch

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import dev, host, make_table

pytestmark = pytest.mark.gpu

CAP = 64 << 20
DIM = 32
BATCH = 1 << 20
RESERVED = np.uint64(0xFFFFFFFFFFFFFFFC)


def fresh_keys(gen, n, lo, device):
    """n distinct keys: counters lo.. scrambled by a bijective mixer (an odd
    multiplier and an add mod 2^64, then a logical xorshift)."""
    x = torch.arange(lo, lo + n, dtype=torch.int64, device=device)
    x = x * (0x9E3779B97F4A7C15 - (1 << 64)) + 0x632BE59BD9B4E019
    x = x ^ ((x >> 29) & ((1 << 35) - 1))
    return x


@pytest.mark.skipif(not torch.cuda.is_available()
                    or torch.cuda.get_device_properties(0).total_memory < (40 << 30),
                    reason="needs a B200-sized GPU")
def test_config2_shape_find_and_insert():
    t = make_table(CAP, dim=DIM, strategy=H.EvictStrategy.kLru, max_hbm=CAP * DIM * 4)
    vals = torch.randn((BATCH, DIM), device="cuda")
    lo = 1
    for _ in range(int(1.8 * CAP) // BATCH + 1):  # Lru keeps the most recent keys
        t.insert_or_assign(BATCH, fresh_keys(None, BATCH, lo, "cuda"), vals)
        lo += BATCH
    torch.cuda.synchronize()
    assert t.size() == CAP
    keys, scores, digests, sizes, values = t.get_state()
    live = np.nonzero(keys < RESERVED)[0]
    assert len(live) == CAP
    o = O.OracleTable(CAP, CAP, dim=DIM, strategy=O.LRU, threads=16)
    o.set_state(keys, scores, digests, sizes, np.ascontiguousarray(values))
    rng = np.random.default_rng(2026)
    resident = keys[rng.choice(live, BATCH // 2, replace=False)]
    absent = host(fresh_keys(None, BATCH // 2, lo + (1 << 40), "cuda"), np.uint64)
    q = np.concatenate([resident, absent])
    rng.shuffle(q)
    gv = torch.zeros((BATCH, DIM), device="cuda")
    gf = torch.zeros(BATCH, dtype=torch.bool, device="cuda")
    gs = torch.zeros(BATCH, dtype=torch.int64, device="cuda")
    t.find(BATCH, dev(q), gv, gf, gs)
    torch.cuda.synchronize()
    ov, of, os_ = o.find(q)
    gf = host(gf).astype(bool)
    np.testing.assert_array_equal(gf, of)
    assert gf.sum() == BATCH // 2
    np.testing.assert_array_equal(host(gv)[gf], ov[of])
    np.testing.assert_array_equal(host(gs, np.uint64)[gf], os_[of])
    del o, values, digests

    # one headline insert batch: half resident keys, half new keys
    hits = keys[rng.choice(live, BATCH // 2, replace=False)]
    new = host(fresh_keys(None, BATCH // 2, lo + (1 << 41), "cuda"), np.uint64)
    ins = np.concatenate([hits, new])
    rng.shuffle(ins)
    rows = torch.randn((BATCH, DIM), device="cuda")
    before = np.sort(keys[live])
    t.insert_or_assign(BATCH, dev(ins), rows)
    torch.cuda.synchronize()
    t.check_device_error()
    k2, s2, _, z2, v2 = t.get_state()
    assert t.size() == CAP and int(z2.sum()) == CAP
    assert not (k2 == np.uint64(0xFFFFFFFFFFFFFFFD)).any()  # no slot left LOCKED
    live_slots = np.nonzero(k2 < RESERVED)[0]
    order = np.argsort(k2[live_slots])
    after = k2[live_slots][order]
    assert len(after) == CAP and (np.diff(after) != 0).all()  # one copy per key
    pos = np.searchsorted(after, ins)
    assert (pos < CAP).all() and (after[np.minimum(pos, CAP - 1)] == ins).all()  # all present
    left = np.setdiff1d(before, after, assume_unique=True)
    assert len(left) == len(new)  # one resident key out per new key
    assert not np.isin(left, ins).any()  # and never a key of the batch
    # every input key holds its input row
    slots = live_slots[order][pos]
    np.testing.assert_array_equal(v2[slots], host(rows))
