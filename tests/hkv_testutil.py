"""Shared helpers for the tests: vectorised Murmur3, key generators that
target buckets (the idea of the reference's tests/common/test_util.h:244-317),
and GPU/oracle comparison helpers."""
import numpy as np

U64 = np.uint64
RESERVED_LO = np.uint64(0xFFFFFFFFFFFFFFFC)


def murmur3_np(k):
    k = np.asarray(k, np.uint64).copy()
    with np.errstate(over="ignore"):
        k ^= k >> U64(33)
        k *= U64(0xFF51AFD7ED558CCD)
        k ^= k >> U64(33)
        k *= U64(0xC4CEB9FE1A85EC53)
        k ^= k >> U64(33)
    return k


def bucket_of(keys, capacity):
    """Bucket index of each key in a power-of-two table."""
    return (murmur3_np(keys) & U64(capacity - 1)) >> U64(7)


def random_keys(rng, n, lo=1, hi=(1 << 63)):
    """Distinct random non-reserved keys."""
    out = np.unique(rng.integers(lo, hi, int(n * 1.05) + 16, dtype=np.uint64))
    rng.shuffle(out)
    assert len(out) >= n
    return out[:n]


def one_key_per_bucket(rng, capacity, buckets, exclude=()):
    """For each bucket in `buckets`, one fresh random key mapping to it
    (no two keys of the batch share a bucket)."""
    want = {int(b): None for b in buckets}
    excl = set(int(x) for x in exclude)
    remaining = set(want)
    while remaining:
        cand = rng.integers(1, 1 << 63, max(4096, len(remaining) * 64 * (capacity // 128) // max(len(remaining), 1)), dtype=np.uint64)
        cand = cand[: 1 << 22]
        bk = bucket_of(cand, capacity)
        for k, b in zip(cand.tolist(), bk.tolist()):
            if b in remaining and k not in excl:
                want[b] = k
                remaining.discard(b)
                if not remaining:
                    break
    return np.array([want[int(b)] for b in buckets], np.uint64)


def keys_for_bucket(rng, capacity, bucket, count, exclude=()):
    excl = set(int(x) for x in exclude)
    out = []
    nb = capacity // 128
    while len(out) < count:
        cand = rng.integers(1, 1 << 63, 64 * nb, dtype=np.uint64)
        sel = cand[bucket_of(cand, capacity) == U64(bucket)]
        for k in sel.tolist():
            if k not in excl and k not in out:
                out.append(k)
                if len(out) == count:
                    break
    return np.array(out, np.uint64)


def live_set(keys, scores, values):
    """(key -> (score, value bytes)) of the live slots of a raw state."""
    live = keys < RESERVED_LO
    k = keys[live]
    s = scores[live]
    v = values[live]
    return {int(a): (int(b), c.tobytes()) for a, b, c in zip(k, s, v)}
