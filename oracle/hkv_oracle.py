"""ctypes binding of the CPU oracle (oracle/hkv_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product. Arrays are numpy arrays.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhkv_oracle.so")

EMPTY_KEY = 0xFFFFFFFFFFFFFFFF
RECLAIM_KEY = 0xFFFFFFFFFFFFFFFE
LOCKED_KEY = 0xFFFFFFFFFFFFFFFD
MAX_SCORE = 0xFFFFFFFFFFFFFFFF
IGNORED_EPOCH = 0xFFFFFFFFFFFFFFFF
LRU, LFU, EPOCH_LRU, EPOCH_LFU, CUSTOMIZED = range(5)
F32, F16, BF16 = 0, 1, 2
R_ILLEGAL, R_DUPLICATE, R_OCCUPIED_EMPTY, R_OCCUPIED_RECLAIMED, R_EVICT, R_REFUSED = range(6)

_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_U64 = ctypes.c_uint64


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    sig = {
        "hkvo_murmur3": (_U64, [_U64]),
        "hkvo_digest": (ctypes.c_uint8, [_U64]),
        "hkvo_empty_digest": (ctypes.c_uint8, []),
        "hkvo_reclaim_digest": (ctypes.c_uint8, []),
        "hkvo_is_reserved": (ctypes.c_int, [_U64]),
        "hkvo_magic_div": (None, [_U64, ctypes.POINTER(_U64), ctypes.POINTER(_U64)]),
        "hkvo_fast_mod": (_U64, [_U64, _U64, _U64, _U64]),
        "hkvo_desired_when_missed": (_U64, [ctypes.c_int, _P, _SZ, _U64, _U64]),
        "hkvo_score_on_write": (ctypes.c_int, [ctypes.c_int, _U64, _P, _SZ, _U64,
                                               ctypes.c_int, ctypes.POINTER(_U64)]),
        "hkvo_score_without_missed": (ctypes.c_int, [ctypes.c_int, _U64, _P, _SZ, _U64,
                                                     _U64, ctypes.POINTER(_U64)]),
        "hkvo_create": (_P, [_U64, _U64, ctypes.c_uint32, ctypes.c_uint32,
                             ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_float]),
        "hkvo_destroy": (None, [_P]),
        "hkvo_set_threads": (None, [_P, ctypes.c_int]),
        "hkvo_set_global_epoch": (None, [_P, _U64]),
        "hkvo_set_clock": (None, [_P, _U64]),
        "hkvo_capacity": (_U64, [_P]),
        "hkvo_bucket_count": (_U64, [_P]),
        "hkvo_size": (_U64, [_P]),
        "hkvo_load_factor": (ctypes.c_float, [_P]),
        "hkvo_reach_max": (ctypes.c_int, [_P]),
        "hkvo_find": (None, [_P, _SZ, _P, _P, _P, _P]),
        "hkvo_contains": (None, [_P, _SZ, _P, _P]),
        "hkvo_insert_or_assign": (None, [_P, _SZ, _P, _P, _P, ctypes.c_int, _P]),
        "hkvo_find_or_insert": (None, [_P, _SZ, _P, _P, _P, ctypes.c_int, _P]),
        "hkvo_insert_and_evict": (_SZ, [_P, _SZ, _P, _P, _P, _P, _P, _P,
                                        ctypes.c_int, _P]),
        "hkvo_accum_or_assign": (None, [_P, _SZ, _P, _P, _P, _P, ctypes.c_int, _P]),
        "hkvo_assign_scores": (None, [_P, _SZ, _P, _P]),
        "hkvo_erase": (None, [_P, _SZ, _P]),
        "hkvo_clear": (None, [_P]),
        "hkvo_export_batch": (_SZ, [_P, _SZ, _SZ, _P, _P, _P]),
        "hkvo_reserve": (None, [_P, _U64]),
        "hkvo_get_state": (None, [_P, _P, _P, _P, _P, _P]),
        "hkvo_set_state": (None, [_P, _P, _P, _P, _P, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


L = _load()


def _p(a):
    return None if a is None else a.ctypes.data


def murmur3(k: int) -> int:
    return L.hkvo_murmur3(k)


def digest(k: int) -> int:
    return L.hkvo_digest(k)


def desired_when_missed(strategy, in_scores, idx, epoch, cycle):
    arr = None if in_scores is None else np.asarray(in_scores, np.uint64)
    return L.hkvo_desired_when_missed(strategy, _p(arr), idx, epoch, cycle)


def score_on_write(strategy, old, in_scores, idx, desired, new_insert):
    arr = None if in_scores is None else np.asarray(in_scores, np.uint64)
    out = _U64(0)
    ok = L.hkvo_score_on_write(strategy, old, _p(arr), idx, desired, int(new_insert),
                               ctypes.byref(out))
    return out.value if ok else None


def score_without_missed(strategy, old, in_scores, idx, epoch, cycle):
    arr = None if in_scores is None else np.asarray(in_scores, np.uint64)
    out = _U64(0)
    ok = L.hkvo_score_without_missed(strategy, old, _p(arr), idx, epoch, cycle,
                                     ctypes.byref(out))
    return out.value if ok else None


class OracleTable:
    """Sequential CPU table with the reference's rules (test checker)."""

    def __init__(self, init_capacity, max_capacity=None, dim=8, strategy=LRU,
                 value_dtype=np.float32, max_load_factor=0.5, bucket_size=128,
                 threads=1):
        max_capacity = init_capacity if max_capacity is None else max_capacity
        self.vdt = np.dtype(value_dtype) if value_dtype != "bfloat16" else np.dtype(np.uint16)
        code = {np.dtype(np.float32): F32, np.dtype(np.float16): F16}.get(self.vdt, F32)
        if value_dtype == "bfloat16":
            code = BF16
        self.dim = dim
        self.h = L.hkvo_create(init_capacity, max_capacity, bucket_size, dim,
                               self.vdt.itemsize, code, strategy, max_load_factor)
        L.hkvo_set_threads(self.h, threads)

    def __del__(self):
        if getattr(self, "h", None):
            L.hkvo_destroy(self.h)
            self.h = None

    # configuration
    def set_threads(self, n):
        L.hkvo_set_threads(self.h, n)

    def set_global_epoch(self, e):
        L.hkvo_set_global_epoch(self.h, e)

    def set_clock(self, c):
        L.hkvo_set_clock(self.h, c)

    def capacity(self):
        return L.hkvo_capacity(self.h)

    def bucket_count(self):
        return L.hkvo_bucket_count(self.h)

    def size(self):
        return L.hkvo_size(self.h)

    def load_factor(self):
        return L.hkvo_load_factor(self.h)

    # ops
    def _k(self, keys):
        return np.ascontiguousarray(keys, np.uint64)

    def _v(self, values, n):
        return np.ascontiguousarray(values, self.vdt).reshape(n, self.dim)

    def find(self, keys, values=None, scores=None):
        keys = self._k(keys)
        n = len(keys)
        values = np.zeros((n, self.dim), self.vdt) if values is None else values
        founds = np.zeros(n, np.uint8)
        scores = np.zeros(n, np.uint64) if scores is None else scores
        L.hkvo_find(self.h, n, _p(keys), _p(values), _p(founds), _p(scores))
        return values, founds.astype(bool), scores

    def contains(self, keys):
        keys = self._k(keys)
        founds = np.zeros(len(keys), np.uint8)
        L.hkvo_contains(self.h, len(keys), _p(keys), _p(founds))
        return founds.astype(bool)

    def insert_or_assign(self, keys, values, scores=None, ignore=False):
        keys = self._k(keys)
        n = len(keys)
        values = self._v(values, n)
        sc = None if scores is None else np.ascontiguousarray(scores, np.uint64)
        res = np.zeros(n, np.uint8)
        L.hkvo_insert_or_assign(self.h, n, _p(keys), _p(values), _p(sc), int(ignore), _p(res))
        return res

    def find_or_insert(self, keys, values, scores=None, ignore=False):
        keys = self._k(keys)
        n = len(keys)
        values = np.array(self._v(values, n), copy=True)
        sc = None if scores is None else np.ascontiguousarray(scores, np.uint64)
        res = np.zeros(n, np.uint8)
        L.hkvo_find_or_insert(self.h, n, _p(keys), _p(values), _p(sc), int(ignore), _p(res))
        return values, res

    def insert_and_evict(self, keys, values, scores=None, ignore=False):
        keys = self._k(keys)
        n = len(keys)
        values = self._v(values, n)
        sc = None if scores is None else np.ascontiguousarray(scores, np.uint64)
        ek = np.zeros(max(n, 1), np.uint64)
        ev = np.zeros((max(n, 1), self.dim), self.vdt)
        es = np.zeros(max(n, 1), np.uint64)
        res = np.zeros(n, np.uint8)
        c = L.hkvo_insert_and_evict(self.h, n, _p(keys), _p(values), _p(sc), _p(ek),
                                    _p(ev), _p(es), int(ignore), _p(res))
        return ek[:c], ev[:c], es[:c], res

    def accum_or_assign(self, keys, values, accum, scores=None, ignore=False):
        keys = self._k(keys)
        n = len(keys)
        values = self._v(values, n)
        acc = np.ascontiguousarray(accum, np.uint8)
        sc = None if scores is None else np.ascontiguousarray(scores, np.uint64)
        res = np.zeros(n, np.uint8)
        L.hkvo_accum_or_assign(self.h, n, _p(keys), _p(values), _p(acc), _p(sc),
                               int(ignore), _p(res))
        return res

    def assign_scores(self, keys, scores=None):
        keys = self._k(keys)
        sc = None if scores is None else np.ascontiguousarray(scores, np.uint64)
        L.hkvo_assign_scores(self.h, len(keys), _p(keys), _p(sc))

    def erase(self, keys):
        keys = self._k(keys)
        L.hkvo_erase(self.h, len(keys), _p(keys))

    def clear(self):
        L.hkvo_clear(self.h)

    def export_batch(self, n, offset=0):
        keys = np.zeros(max(n, 1), np.uint64)
        values = np.zeros((max(n, 1), self.dim), self.vdt)
        scores = np.zeros(max(n, 1), np.uint64)
        c = L.hkvo_export_batch(self.h, n, offset, _p(keys), _p(values), _p(scores))
        return keys[:c], values[:c], scores[:c]

    def load_chunks(self, keys, values, scores, max_workspace_size=1 << 20):
        """The reference's load (hkv_hashtable.h:3125-3195) on tuples already
        read from a file: chunks of max_workspace_size // (16 + value row
        bytes) tuples, each inserted with insert_or_assign(unique_key=true,
        ignore_evict_strategy=true) after setting the global epoch to
        IGNORED_GLOBAL_EPOCH."""
        tuple_bytes = 16 + self.dim * self.vdt.itemsize
        n = max_workspace_size // tuple_bytes
        for s in range(0, len(keys), n):
            self.set_global_epoch(0xFFFFFFFFFFFFFFFF)
            self.insert_or_assign(keys[s:s + n], values[s:s + n], scores[s:s + n],
                                  ignore=True)
        return len(keys)

    def reserve(self, new_capacity):
        L.hkvo_reserve(self.h, new_capacity)

    def get_state(self):
        cap, nb = self.capacity(), self.bucket_count()
        keys = np.empty(cap, np.uint64)
        scores = np.empty(cap, np.uint64)
        digests = np.empty(cap, np.uint8)
        sizes = np.empty(nb, np.int32)
        values = np.empty((cap, self.dim), self.vdt)
        L.hkvo_get_state(self.h, _p(keys), _p(scores), _p(digests), _p(sizes), _p(values))
        return keys, scores, digests, sizes, values

    def set_state(self, keys=None, scores=None, digests=None, sizes=None, values=None):
        L.hkvo_set_state(self.h, _p(keys), _p(scores), _p(digests), _p(sizes), _p(values))
