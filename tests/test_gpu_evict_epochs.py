"""Training-style upsert with eviction (BASELINE config 3's shape, scaled
down), on the GPU: insert_and_evict of batches with repeated keys
(unique_key = false) into a full EpochLfu table, the global epoch advancing
every 10 batches, the evicted and refused tuples collected after every batch
(reference insert_and_evict_kernel.h:231-337 for repeated keys, outputs
:549-685).

Which key loses a contested slot depends on thread order, so each batch is
checked by invariants that hold for every order:
* every input key is in the table afterwards or among the batch's outputs;
* every output is a legal event: a resident key evicted (with the value and
  score it held before), an input placed or updated and then evicted by a
  later key of the batch (its merged row), or a refused input (each
  occurrence with its own row and desired score); a key can have several
  such events in one batch;
* victims are minimum-score slots: in each bucket, every key present after
  the batch scores at least as high as every victim taken from it;
* sizes are consistent and no key has two copies."""
import numpy as np
import pytest
import torch

import hkv_b200 as H
from hkv_gpu import GpuOps, make_table
from hkv_testutil import bucket_of

pytestmark = pytest.mark.gpu

RESERVED = np.uint64(0xFFFFFFFFFFFFFFFC)
LOW32 = np.uint64(0xFFFFFFFF)


def snapshot(t):
    keys, scores, _, sizes, values = t.get_state()
    live = keys < RESERVED
    return {int(k): (int(s), v.copy()) for k, s, v in zip(keys[live], scores[live],
                                                         values[live])}, keys, sizes


def test_insert_and_evict_with_repeats_across_epochs():
    cap, dim = 128 * 32, 8
    rng = np.random.default_rng(303)
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kEpochLfu, epoch=1)
    g = GpuOps(t, dim)
    # fill to load factor 1.0
    pool = np.unique(rng.integers(1, 1 << 62, 4 * cap, dtype=np.uint64))
    g.insert_or_assign(pool[:2 * cap], rng.standard_normal((2 * cap, dim)).astype(np.float32),
                       rng.integers(1, 17, 2 * cap).astype(np.uint64))
    assert t.size() == cap
    epoch = 1
    ids = np.arange(len(pool))
    weights = 1.0 / (ids + 1.0) ** 1.05  # power law over the key pool
    weights /= weights.sum()
    total_out = 0
    for b in range(30):
        if b and b % 10 == 0:
            epoch += 1
            t.set_global_epoch(epoch)
        n = 2048
        keys = pool[rng.choice(len(pool), n, p=weights)]  # repeats, hot keys first
        vals = rng.standard_normal((n, dim)).astype(np.float32)
        sc = rng.integers(1, 17, n).astype(np.uint64)
        before, _, _ = snapshot(t)
        ek, ev, es = g.insert_and_evict(keys, vals, sc, unique=False)
        total_out += len(ek)
        after, k2, z2 = snapshot(t)
        assert len(after) == int(z2.sum()) == cap  # stays full, sizes consistent
        live = k2[k2 < RESERVED]
        assert len(np.unique(live)) == len(live)  # one copy per key
        batch_keys = set(keys.tolist())
        out_keys = set(int(k) for k in ek)
        for k in batch_keys:
            assert k in after or k in out_keys, "input key neither present nor reported"
        # the merged input of each key: last occurrence's row, EpochLfu low
        # halves summed (saturating) under the current epoch
        last = {}
        summed = {}
        occ = {}
        for i, k in enumerate(keys.tolist()):
            last[k] = i
            occ.setdefault(k, []).append(i)
            summed[k] = min(summed.get(k, 0) + int(sc[i]), 0xFFFFFFFF)
        victims = {}
        # Every output is one event, and a key may have two in a batch (a
        # resident key evicted, then placed again by its own input and
        # evicted again or refused):
        #  - a resident key evicted: the value and score it held before;
        #  - an input placed or updated, then evicted by a later key of the
        #    batch: its merged row and the score the hit gave it;
        #  - a refused input: its merged row and desired score.
        for k, s_, v in zip(ek.tolist(), es.tolist(), ev):
            cands = []
            if k in before:
                cands.append((before[k][0], before[k][1]))
            if k in batch_keys:
                desired = (epoch << 32) | summed[k]
                cands.append((desired, vals[last[k]]))
                # a refused key is reported once per occurrence, each with its
                # own row and desired score (insert_and_evict_kernel.h:291-303)
                for i in occ[k]:
                    cands.append(((epoch << 32) | int(sc[i]), vals[i]))
                if k in before:
                    low = before[k][0] & 0xFFFFFFFF
                    cands.append(((epoch << 32) | min(low + summed[k], 0xFFFFFFFF),
                                  vals[last[k]]))
            assert any(s_ == cs and (v == cv).all() for cs, cv in cands), \
                f"output {k} matches no legal event"
            if k in before and k not in batch_keys:
                bkt = int(bucket_of(np.array([k], np.uint64), cap)[0])
                victims[bkt] = max(victims.get(bkt, 0), s_)
        # victims were minimum-score slots of their buckets
        if victims:
            ak = np.array(list(after.keys()), np.uint64)
            asc = np.array([after[int(k)][0] for k in ak], np.uint64)
            bk = bucket_of(ak, cap)
            for bkt, vmax in victims.items():
                assert (asc[bk == np.uint64(bkt)] >= np.uint64(vmax)).all()
    assert total_out > 0
    t.check_device_error()
