"""Writes the golden fixtures of tests/golden/ (run from the repository root:
`python tests/golden/make_golden.py`).

The reference (an Ascend NPU library) cannot run here, so the expected
outputs come from the CPU oracle in oracle/, which tests/test_oracle_kat.py
pins against the known answers of the reference's own tests. Each fixture
holds its inputs and the expected outputs of one seeded case, chosen so that
the result is independent of thread order (distinct Customized scores, or
keys that never share a bucket), which lets the CUDA path be compared
bit-for-bit: tests/test_golden.py replays every fixture on the oracle (CPU)
and through the C ABI on the GPU.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import hkv_oracle as O  # noqa: E402
from hkv_testutil import bucket_of  # noqa: E402

RESERVED_MIN = np.uint64(0xFFFFFFFFFFFFFFFC)


def live_sorted(t):
    keys, scores, _, _, values = t.get_state()
    live = keys < RESERVED_MIN
    order = np.argsort(keys[live])
    return keys[live][order], scores[live][order], values[live][order]


def fresh_keys(rng, n, exclude=()):
    out = np.unique(rng.integers(1, 1 << 63, size=n * 2, dtype=np.uint64))
    out = np.setdiff1d(out, np.asarray(exclude, np.uint64))
    return rng.permutation(out)[:n]


def case_customized_batches(rng):
    """Three insert_or_assign batches of new keys into a 32-bucket table
    (Customized, distinct scores, heavy per-bucket contention), one batch
    that only updates resident keys, then find and the table contents. (A
    batch that mixes updates of resident keys with evicting inserts into the
    same bucket has an order-dependent result, so the cases keep them apart.)"""
    cap, dim, nb, per = 128 * 32, 4, 3, 1536
    t = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED)
    pool = fresh_keys(rng, nb * per)
    scores_all = rng.permutation(np.arange(1, 10 * per, dtype=np.uint64))
    out = {"capacity": cap, "dim": dim}
    for b in range(nb):
        keys = pool[b * per:(b + 1) * per]
        vals = rng.standard_normal((per, dim)).astype(np.float32)
        sc = scores_all[b * per:(b + 1) * per]
        t.insert_or_assign(keys, vals, sc)
        out[f"keys{b}"], out[f"vals{b}"], out[f"scores{b}"] = keys, vals, sc
    res_k, _, _ = live_sorted(t)
    hk = rng.choice(res_k, 512, replace=False)
    hv = rng.standard_normal((512, dim)).astype(np.float32)
    hs = scores_all[nb * per:nb * per + 512]
    t.insert_or_assign(hk, hv, hs)
    out.update(hit_keys=hk, hit_vals=hv, hit_scores=hs)
    q = np.concatenate([rng.choice(res_k, 512, replace=False), fresh_keys(rng, 512, pool)])
    q = rng.permutation(q)
    fv, ff, fs = t.find(q)
    out.update(find_keys=q, find_values=fv, find_founds=ff, find_scores=fs)
    out["state_keys"], out["state_scores"], out["state_values"] = live_sorted(t)
    return out


def case_lfu_duplicates(rng):
    """find_or_insert with repeated keys (unique_key = false), Lfu, keys in
    distinct buckets: merged scores add, every occurrence reads one row."""
    cap, dim = 128 * 64, 4
    t = O.OracleTable(cap, cap, dim=dim, strategy=O.LFU)
    distinct, seen = [], set()
    while len(distinct) < 48:
        k = fresh_keys(rng, 1)[0]
        b = int(bucket_of(np.array([k], np.uint64), cap)[0])
        if b not in seen:
            seen.add(b)
            distinct.append(k)
    distinct = np.array(distinct, np.uint64)
    out = {"capacity": cap, "dim": dim}
    for c, (lo, hi) in enumerate(((0, 32), (16, 48))):
        keys = rng.choice(distinct[lo:hi], 400, replace=True).astype(np.uint64)
        vals = rng.standard_normal((400, dim)).astype(np.float32)
        sc = rng.integers(1, 17, 400).astype(np.uint64)
        got, _ = t.find_or_insert(keys, vals, sc)
        out[f"keys{c}"], out[f"vals{c}"], out[f"scores{c}"] = keys, vals, sc
        out[f"returned{c}"] = got
    out["state_keys"], out["state_scores"], out["state_values"] = live_sorted(t)
    return out


def case_insert_and_evict(rng):
    """insert_and_evict of new keys into a full 16-bucket table (Customized,
    distinct scores): the evicted and refused tuples as a set, then the
    table."""
    cap, dim = 128 * 16, 4
    t = O.OracleTable(cap, cap, dim=dim, strategy=O.CUSTOMIZED)
    pre = fresh_keys(rng, 3 * cap)
    scores = rng.permutation(np.arange(1, 20 * cap, dtype=np.uint64))
    pv = rng.standard_normal((len(pre), dim)).astype(np.float32)
    t.insert_or_assign(pre, pv, scores[: len(pre)])
    keys = fresh_keys(rng, 512, pre)
    vals = rng.standard_normal((len(keys), dim)).astype(np.float32)
    sc = scores[len(pre):len(pre) + len(keys)]
    ek, ev, es, _ = t.insert_and_evict(keys, vals, sc)
    order = np.argsort(ek)
    return {"capacity": cap, "dim": dim, "pre_keys": pre, "pre_vals": pv,
            "pre_scores": scores[: len(pre)], "keys": keys, "vals": vals, "scores": sc,
            "ev_keys": ek[order], "ev_vals": ev[order], "ev_scores": es[order],
            "state_keys": live_sorted(t)[0], "state_scores": live_sorted(t)[1],
            "state_values": live_sorted(t)[2]}


def case_epoch_lfu_scores_erase(rng):
    """EpochLfu: insert with epoch 3, assign_scores on a subset, erase a
    subset, then find every key."""
    cap, dim, epoch = 128 * 16, 4, 3
    t = O.OracleTable(cap, cap, dim=dim, strategy=O.EPOCH_LFU)
    t.set_global_epoch(epoch)
    keys = fresh_keys(rng, 1024)
    vals = rng.standard_normal((1024, dim)).astype(np.float32)
    sc = rng.integers(1, 1 << 40, 1024).astype(np.uint64)
    t.insert_or_assign(keys, vals, sc)
    ak = rng.choice(keys, 300, replace=False)
    asc = rng.integers(1, 1 << 33, 300).astype(np.uint64)
    t.assign_scores(ak, asc)
    rk = rng.choice(keys, 200, replace=False)
    t.erase(rk)
    fv, ff, fs = t.find(keys)
    return {"capacity": cap, "dim": dim, "epoch": epoch, "keys": keys, "vals": vals,
            "scores": sc, "assign_keys": ak, "assign_scores": asc, "erase_keys": rk,
            "find_values": fv, "find_founds": ff, "find_scores": fs,
            "state_keys": live_sorted(t)[0], "state_scores": live_sorted(t)[1],
            "state_values": live_sorted(t)[2]}


CASES = {
    "customized_batches": (case_customized_batches, 20261201),
    "lfu_duplicates": (case_lfu_duplicates, 20261202),
    "insert_and_evict": (case_insert_and_evict, 20261203),
    "epoch_lfu_scores_erase": (case_epoch_lfu_scores_erase, 20261204),
}


def main():
    for name, (fn, seed) in CASES.items():
        data = fn(np.random.default_rng(seed))
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **data)
        print(f"{path}: {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
