"""Python binding of the B200 HierarchicalKV table (libhkv_b200.so, C ABI in
include/hkv_b200.h).

`HashTable` mirrors the reference's `HashTable<K, V, S, Strategy>`
(include/hkv_hashtable.h of yangzhen92/HierarchicalKV-ascend): same method
names, argument order and defaults, with torch tensors (or raw device
addresses) in place of device pointers and a torch CUDA stream in place of
the ACL stream. Errors raise `HkvException` (configuration / argument,
the reference's HKV_CHECK), `CudaException` (runtime API), `HkvTimeout`
(a device lock wait ran out) or `RuntimeError` (std::runtime_error).

The library is loaded from this directory. There is no fallback: if the
shared library is missing or cannot be loaded, importing this module fails.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

_HERE = os.path.dirname(os.path.abspath(__file__))
# HKV_B200_LIB selects another build of the same library (e.g. the
# self-checking libhkv_b200_checked.so); the default is the optimised one.
LIB_PATH = os.environ.get("HKV_B200_LIB") or os.path.join(_HERE, "libhkv_b200.so")

HKV_OK = 0
HKV_ERR_INVALID = 1
HKV_ERR_CUDA = 2
HKV_ERR_TIMEOUT = 3
HKV_ERR_UNSUPPORTED = 4
HKV_ERR_RUNTIME = 5


class EvictStrategy:
    """EvictStrategy::EvictStrategyEnum, reference hkv_hashtable.h:111-119."""

    kLru = 0
    kLfu = 1
    kEpochLru = 2
    kEpochLfu = 3
    kCustomized = 4


KEY_U64 = 0
KEY_I64 = 1
VALUE_TYPES = {"float32": 0, "float16": 1, "bfloat16": 2, "float64": 3,
               "uint32": 4, "uint16": 5, "int8": 6, "uint64": 7}
IGNORED_GLOBAL_EPOCH = 0xFFFFFFFFFFFFFFFF


class HkvException(ValueError):
    """HKV_CHECK failures (reference debug.h:53-74)."""


class CudaException(RuntimeError):
    """CUDA runtime failures (the reference's NpuException, debug.h:30-51)."""


class HkvTimeout(RuntimeError):
    """A device-side lock wait exceeded its bound."""


class HkvUnsupported(NotImplementedError):
    """Valid in the reference, not supported by this build."""


class _Options(ctypes.Structure):
    _fields_ = [
        ("init_capacity", ctypes.c_uint64),
        ("max_capacity", ctypes.c_uint64),
        ("max_hbm_for_vectors", ctypes.c_uint64),
        ("max_bucket_size", ctypes.c_uint64),
        ("dim", ctypes.c_uint64),
        ("max_load_factor", ctypes.c_float),
        ("block_size", ctypes.c_int),
        ("io_block_size", ctypes.c_int),
        ("device_id", ctypes.c_int),
        ("io_by_cpu", ctypes.c_int),
        ("use_constant_memory", ctypes.c_int),
        ("reserved_key_start_bit", ctypes.c_int),
        ("num_of_buckets_per_alloc", ctypes.c_uint64),
        ("api_lock", ctypes.c_int),
    ]


class _Predicate(ctypes.Structure):
    _fields_ = [("key_mask", ctypes.c_uint64), ("key_value", ctypes.c_uint64),
                ("score_cmp", ctypes.c_int), ("threshold", ctypes.c_uint64)]


SCORE_CMP = {None: 0, "<": 1, "<=": 2, ">": 3, ">=": 4, "==": 5}


def predicate(key_mask=0, key_value=0, score_cmp=None, threshold=0):
    """Built-in scan predicate: (key & key_mask) == key_value and
    score <score_cmp> threshold (score_cmp one of None, '<', '<=', '>', '>=',
    '==')."""
    return _Predicate(key_mask, key_value, SCORE_CMP[score_cmp], threshold)


@dataclass
class HashTableOptions:
    """HashTableOptions, reference hashtable_options.h:534-566."""

    init_capacity: int = 0
    max_capacity: int = 0
    max_hbm_for_vectors: int = 0
    max_bucket_size: int = 128
    dim: int = 64
    max_load_factor: float = 0.5
    block_size: int = 128
    io_block_size: int = 1024
    device_id: int = -1
    io_by_cpu: bool = False
    use_constant_memory: bool = False
    reserved_key_start_bit: int = 0
    num_of_buckets_per_alloc: int = 1
    api_lock: bool = False

    def _c(self) -> _Options:
        o = _Options()
        for f, _ in _Options._fields_:
            v = getattr(self, f)
            setattr(o, f, float(v) if f == "max_load_factor" else int(v))
        return o


# hkv_allocator (include/hkv_b200.h): the reference's BaseAllocator as
# callbacks on a caller's object
_ALLOC_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                             ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t, ctypes.c_uint)
_ALLOC_ASYNC_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t,
                                   ctypes.c_void_p)
_FREE_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p)
_FREE_ASYNC_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                  ctypes.c_void_p, ctypes.c_void_p)


class _Allocator(ctypes.Structure):
    _fields_ = [("user", ctypes.c_void_p), ("alloc", _ALLOC_FN),
                ("alloc_async", _ALLOC_ASYNC_FN), ("free", _FREE_FN),
                ("free_async", _FREE_ASYNC_FN)]


MEMORY_DEVICE, MEMORY_PINNED, MEMORY_HOST = 0, 1, 2

# C ABI symbols and their signatures (include/hkv_b200.h)
_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_B = ctypes.c_bool
_U64 = ctypes.c_uint64
SIGNATURES = {
    "hkv_options_init": (None, [ctypes.POINTER(_Options)]),
    "hkv_last_error": (ctypes.c_char_p, []),
    "hkv_table_create": (ctypes.c_int, [ctypes.POINTER(_Options), ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)]),
    "hkv_table_create_with_allocator": (ctypes.c_int, [ctypes.POINTER(_Options), ctypes.c_int,
                                                       ctypes.c_int, ctypes.c_int,
                                                       ctypes.POINTER(_Allocator),
                                                       ctypes.POINTER(_P)]),
    "hkv_table_destroy": (ctypes.c_int, [_P]),
    "hkv_set_max_capacity": (ctypes.c_int, [_P, _SZ]),
    "hkv_insert_or_assign": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _B, _B]),
    "hkv_insert_and_evict": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P, _P, _P, _P, _B, _B]),
    "hkv_insert_and_evict_count": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P, _P, _P,
                                                  _B, _B, ctypes.POINTER(_SZ)]),
    "hkv_accum_or_assign": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P, _B]),
    "hkv_find_or_insert": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _B, _B]),
    "hkv_assign_scores": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _B]),
    "hkv_find_or_insert_noalloc": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _B]),
    "hkv_find": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P]),
    "hkv_contains": (ctypes.c_int, [_P, _SZ, _P, _P, _P]),
    "hkv_erase": (ctypes.c_int, [_P, _SZ, _P, _P]),
    "hkv_clear": (ctypes.c_int, [_P, _P]),
    "hkv_export_batch": (ctypes.c_int, [_P, _SZ, _SZ, _P, _P, _P, _P, _P]),
    "hkv_export_batch_count": (ctypes.c_int, [_P, _SZ, _SZ, _P, _P, _P, _P,
                                              ctypes.POINTER(_SZ)]),
    "hkv_size": (ctypes.c_int, [_P, _P, ctypes.POINTER(_SZ)]),
    "hkv_capacity": (ctypes.c_int, [_P, ctypes.POINTER(_SZ)]),
    "hkv_load_factor": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_float)]),
    "hkv_dim": (ctypes.c_int, [_P, ctypes.POINTER(_SZ)]),
    "hkv_max_bucket_size": (ctypes.c_int, [_P, ctypes.POINTER(_SZ)]),
    "hkv_bucket_count": (ctypes.c_int, [_P, ctypes.POINTER(_SZ)]),
    "hkv_is_pure_hbm_mode": (ctypes.c_int, [_P, ctypes.POINTER(_B)]),
    "hkv_reserve": (ctypes.c_int, [_P, _SZ, _P]),
    "hkv_set_global_epoch": (ctypes.c_int, [_P, _U64]),
    "hkv_check_device_error": (ctypes.c_int, [_P, _P]),
    "hkv_kernel_launches": (ctypes.c_int, [ctypes.POINTER(_U64)]),
    "hkv_find_ptr": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P]),
    "hkv_erase_if": (ctypes.c_int, [_P, _P, _P, ctypes.POINTER(_SZ)]),
    "hkv_export_batch_if": (ctypes.c_int, [_P, _P, _SZ, _SZ, _P, _P, _P, _P, _P]),
    "hkv_size_if": (ctypes.c_int, [_P, _P, _P, _P]),
    "hkv_table_get_view": (ctypes.c_int, [_P, _P]),
    "hkv_find_or_insert_ptr": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P, _B, _B, _P]),
    "hkv_lock_keys": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P]),
    "hkv_unlock_keys": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P]),
    "hkv_save_files": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p,
                                      ctypes.c_char_p, _SZ, _P, ctypes.POINTER(_SZ)]),
    "hkv_load_files": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_char_p,
                                      ctypes.c_char_p, _SZ, _P, ctypes.POINTER(_SZ)]),
    "hkv_save": (ctypes.c_int, [_P, _P, _P, _SZ, _P, ctypes.POINTER(_SZ)]),
    "hkv_load": (ctypes.c_int, [_P, _P, _P, _SZ, _P, ctypes.POINTER(_SZ)]),
    "hkv_debug_get_state": (ctypes.c_int, [_P, _P, _P, _P, _P, _P]),
    "hkv_debug_set_state": (ctypes.c_int, [_P, _P, _P, _P, _P, _P]),
    "hkv_nccl_unique_id": (ctypes.c_int, [_P]),
    "hkv_sharded_create": (ctypes.c_int, [ctypes.POINTER(_Options), ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, _P, ctypes.c_int,
                                          ctypes.c_int, _SZ, ctypes.POINTER(_P)]),
    "hkv_sharded_transport": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int)]),
    "hkv_sharded_destroy": (ctypes.c_int, [_P]),
    "hkv_sharded_local": (_P, [_P]),
    "hkv_sharded_find_or_insert": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _B]),
    "hkv_sharded_find": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _P]),
    "hkv_sharded_insert_or_assign": (ctypes.c_int, [_P, _SZ, _P, _P, _P, _P, _B]),
    "hkv_sharded_size": (ctypes.c_int, [_P, _P, ctypes.POINTER(_SZ)]),
}


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads libhkv_b200.so and declares every C ABI signature."""
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        # an older build (HKV_B200_LIB) may lack newer entry points: calling
        # one then raises AttributeError; tests/test_abi.py checks that the
        # in-tree library exports every declared symbol
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load_library()
    return _LIB


def _check(status: int) -> None:
    if status == HKV_OK:
        return
    msg = (lib().hkv_last_error() or b"").decode()
    if status == HKV_ERR_INVALID:
        raise HkvException(msg)
    if status == HKV_ERR_CUDA:
        raise CudaException(msg)
    if status == HKV_ERR_TIMEOUT:
        raise HkvTimeout(msg)
    if status == HKV_ERR_UNSUPPORTED:
        raise HkvUnsupported(msg)
    raise RuntimeError(msg)


def _allocator_callbacks(allocator) -> _Allocator:
    """hkv_allocator callbacks over a Python allocator object; an exception in
    the object becomes a failed allocation (non-zero status)."""

    def alloc(_u, mt, out, size, flags):
        try:
            out[0] = int(allocator.alloc(mt, int(size), int(flags)))
            return 0
        except Exception:
            return 1

    def free(_u, mt, ptr):
        try:
            allocator.free(mt, int(ptr or 0))
            return 0
        except Exception:
            return 1

    a = _Allocator()
    a.user = None
    a.alloc = _ALLOC_FN(alloc)
    a.free = _FREE_FN(free)
    if hasattr(allocator, "alloc_async") and hasattr(allocator, "free_async"):
        def alloc_async(_u, mt, out, size, stream):
            try:
                out[0] = int(allocator.alloc_async(mt, int(size), stream or 0))
                return 0
            except Exception:
                return 1

        def free_async(_u, mt, ptr, stream):
            try:
                allocator.free_async(mt, int(ptr or 0), stream or 0)
                return 0
            except Exception:
                return 1

        a.alloc_async = _ALLOC_ASYNC_FN(alloc_async)
        a.free_async = _FREE_ASYNC_FN(free_async)
    else:
        a.alloc_async = ctypes.cast(None, _ALLOC_ASYNC_FN)
        a.free_async = ctypes.cast(None, _FREE_ASYNC_FN)
    a._keep = (alloc, free)  # the Python functions behind the callbacks
    return a


class TorchAllocator:
    """A BaseAllocator over PyTorch's CUDA caching allocator for device
    memory (so a table embedded in a PyTorch program shares torch's memory
    pool and shows in torch.cuda.memory_allocated) and pinned host memory
    from torch (pinned tensors, mapped into the device address space on
    this platform). Blocks are kept by address until freed."""

    def __init__(self, device=None):
        import torch

        self._torch = torch
        self.device = torch.cuda.current_device() if device is None else device
        self.blocks = {}

    def alloc(self, memory_type, size, flags=0):
        t = self._torch
        n = max(int(size), 1)
        if memory_type == MEMORY_DEVICE:
            buf = t.empty(n, dtype=t.uint8, device=f"cuda:{self.device}")
        elif memory_type == MEMORY_PINNED:
            buf = t.empty(n, dtype=t.uint8, pin_memory=True)
        else:
            buf = t.empty(n, dtype=t.uint8)
        addr = buf.data_ptr()
        self.blocks[addr] = buf
        return addr

    def free(self, memory_type, addr):
        self.blocks.pop(addr, None)


def kernel_launches() -> int:
    """Kernels this library has enqueued in this process (all tables)."""
    out = _U64(0)
    _check(lib().hkv_kernel_launches(ctypes.byref(out)))
    return int(out.value)


def _ptr(x):
    """Device address of a tensor (or an int address, or None)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream):
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class HashTable:
    """Mirror of the reference's HashTable<K, V, S, Strategy>.

    key_dtype: "uint64" or "int64"; value_dtype: a name in VALUE_TYPES.
    """

    def __init__(self, evict_strategy: int = EvictStrategy.kLru,
                 key_dtype: str = "uint64", value_dtype: str = "float32"):
        self.evict_strategy = evict_strategy
        self.key_dtype = key_dtype
        self.value_dtype = value_dtype
        self._h = None
        self._options = None
        self._borrowed = False

    @classmethod
    def borrow(cls, handle, evict_strategy, key_dtype="uint64", value_dtype="float32"):
        """Wraps a table handle owned elsewhere (e.g. a sharded table's local
        shard); closing the wrapper does not destroy it."""
        t = cls(evict_strategy, key_dtype, value_dtype)
        t._h = handle
        t._borrowed = True
        return t

    # -- lifecycle ---------------------------------------------------------
    def init(self, options: HashTableOptions, allocator=None) -> None:
        """HashTable::init(options, allocator), reference hkv_hashtable.h
        :962-1042. `allocator` (the reference's BaseAllocator) provides
        alloc(memory_type, size, pinned_flags) -> address and
        free(memory_type, address), and optionally alloc_async(memory_type,
        size, stream) and free_async(memory_type, address, stream); every
        allocation of the table comes from it (MEMORY_DEVICE / MEMORY_PINNED,
        see hkv_allocator in include/hkv_b200.h). It must outlive the
        table."""
        if self._h is not None:
            return
        h = ctypes.c_void_p()
        o = options._c()
        kt = KEY_I64 if self.key_dtype == "int64" else KEY_U64
        if allocator is None:
            _check(lib().hkv_table_create(ctypes.byref(o), kt, VALUE_TYPES[self.value_dtype],
                                          self.evict_strategy, ctypes.byref(h)))
        else:
            self._alloc_cbs = _allocator_callbacks(allocator)  # kept alive with the table
            _check(lib().hkv_table_create_with_allocator(
                ctypes.byref(o), kt, VALUE_TYPES[self.value_dtype], self.evict_strategy,
                ctypes.byref(self._alloc_cbs), ctypes.byref(h)))
        self._h = h.value
        self._options = options

    def close(self) -> None:
        if self._h is not None and not self._borrowed:
            _check(lib().hkv_table_destroy(self._h))
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    # -- insert-like ---------------------------------------------------------
    def insert_or_assign(self, n, keys, values, scores=None, stream=None,
                         unique_key=True, ignore_evict_strategy=False):
        _check(lib().hkv_insert_or_assign(self._h, n, _ptr(keys), _ptr(values),
                                          _ptr(scores), _stream(stream),
                                          unique_key, ignore_evict_strategy))

    def insert_and_evict(self, n, keys, values, scores, evicted_keys,
                         evicted_values, evicted_scores=None,
                         d_evicted_counter=None, stream=None, unique_key=True,
                         ignore_evict_strategy=False):
        """With d_evicted_counter: the device-counter overload (caller zeroes
        it). Without: the overload that returns the count (synchronises)."""
        if d_evicted_counter is not None:
            _check(lib().hkv_insert_and_evict(
                self._h, n, _ptr(keys), _ptr(values), _ptr(scores),
                _ptr(evicted_keys), _ptr(evicted_values), _ptr(evicted_scores),
                _ptr(d_evicted_counter), _stream(stream), unique_key,
                ignore_evict_strategy))
            return None
        cnt = ctypes.c_size_t(0)
        _check(lib().hkv_insert_and_evict_count(
            self._h, n, _ptr(keys), _ptr(values), _ptr(scores),
            _ptr(evicted_keys), _ptr(evicted_values), _ptr(evicted_scores),
            _stream(stream), unique_key, ignore_evict_strategy,
            ctypes.byref(cnt)))
        return cnt.value

    def accum_or_assign(self, n, keys, value_or_deltas, accum_or_assigns,
                        scores=None, stream=None, ignore_evict_strategy=False):
        _check(lib().hkv_accum_or_assign(self._h, n, _ptr(keys),
                                         _ptr(value_or_deltas),
                                         _ptr(accum_or_assigns), _ptr(scores),
                                         _stream(stream), ignore_evict_strategy))

    def find_or_insert(self, n, keys, values, scores=None, stream=None,
                       unique_key=True, ignore_evict_strategy=False):
        _check(lib().hkv_find_or_insert(self._h, n, _ptr(keys), _ptr(values),
                                        _ptr(scores), _stream(stream),
                                        unique_key, ignore_evict_strategy))

    def find_or_insert_noalloc(self, n, keys, values, scores=None, stream=None,
                               ignore_evict_strategy=False):
        """find_or_insert of a batch that may repeat keys, using the library's
        fixed device scratch array instead of allocating (see
        hkv_find_or_insert_noalloc in include/hkv_b200.h for its limits)."""
        _check(lib().hkv_find_or_insert_noalloc(self._h, n, _ptr(keys), _ptr(values),
                                                _ptr(scores), _stream(stream),
                                                ignore_evict_strategy))

    def assign_scores(self, n, keys, scores=None, stream=None, unique_key=True):
        _check(lib().hkv_assign_scores(self._h, n, _ptr(keys), _ptr(scores),
                                       _stream(stream), unique_key))

    assign = assign_scores

    # -- lookups -------------------------------------------------------------
    def find(self, n, keys, values, founds, scores=None, stream=None):
        _check(lib().hkv_find(self._h, n, _ptr(keys), _ptr(values),
                              _ptr(founds), _ptr(scores), _stream(stream)))

    def erase_if(self, pred, stream=None) -> int:
        """erase_if with a built-in predicate (see predicate()); returns the
        number erased."""
        out = _SZ(0)
        _check(lib().hkv_erase_if(self._h, ctypes.byref(pred), _stream(stream),
                                  ctypes.byref(out)))
        return out.value

    def export_batch_if(self, pred, n, offset, d_counter, keys, values, scores=None,
                        stream=None):
        _check(lib().hkv_export_batch_if(self._h, ctypes.byref(pred), n, offset,
                                         _ptr(d_counter), _ptr(keys), _ptr(values),
                                         _ptr(scores), _stream(stream)))

    def size_if(self, pred, d_counter, stream=None):
        _check(lib().hkv_size_if(self._h, ctypes.byref(pred), _ptr(d_counter),
                                 _stream(stream)))

    def find_ptr(self, n, keys, value_ptrs, founds=None, scores=None, stream=None):
        """find* : value_ptrs (int64 device tensor of n) receives the device
        address of each found key's value row, 0 for a missed key."""
        _check(lib().hkv_find_ptr(self._h, n, _ptr(keys), _ptr(value_ptrs),
                                  _ptr(founds), _ptr(scores), _stream(stream)))

    def find_or_insert_ptr(self, n, keys, value_ptrs, founds, scores=None,
                           stream=None, unique_key=True, ignore_evict_strategy=False,
                           locked_key_ptrs=None):
        """find_or_insert* : finds or inserts each key (find_or_insert rules)
        without copying values; value_ptrs receives each key's row address
        (0 when refused), founds whether the key was there before. With
        locked_key_ptrs the keys stay locked (their key-word addresses go
        there) until unlock_keys."""
        _check(lib().hkv_find_or_insert_ptr(self._h, n, _ptr(keys), _ptr(value_ptrs),
                                            _ptr(founds), _ptr(scores), _stream(stream),
                                            unique_key, ignore_evict_strategy,
                                            _ptr(locked_key_ptrs)))

    def lock_keys(self, n, keys, locked_key_ptrs, succeededs=None, stream=None,
                  scores=None):
        """lock_keys: locks each present key (hit score rule) and writes its
        key-word address to locked_key_ptrs (0 and False when absent)."""
        _check(lib().hkv_lock_keys(self._h, n, _ptr(keys), _ptr(locked_key_ptrs),
                                   _ptr(succeededs), _stream(stream), _ptr(scores)))

    def unlock_keys(self, n, locked_key_ptrs, keys, succeededs=None, stream=None):
        """unlock_keys: puts each key back at its locked key word."""
        _check(lib().hkv_unlock_keys(self._h, n, _ptr(locked_key_ptrs), _ptr(keys),
                                     _ptr(succeededs), _stream(stream)))

    def save(self, keys_path, values_path, scores_path,
             max_workspace_size=1 << 20, stream=None) -> int:
        """save() into the reference's LocalKVFile format (three raw binary
        files: keys, value rows, scores). Returns the number of tuples."""
        out = _SZ(0)
        _check(lib().hkv_save_files(self._h, str(keys_path).encode(),
                                    str(values_path).encode(), str(scores_path).encode(),
                                    max_workspace_size, _stream(stream), ctypes.byref(out)))
        return out.value

    def load(self, keys_path, values_path, scores_path,
             max_workspace_size=1 << 20, stream=None) -> int:
        """load() from the LocalKVFile format. Returns the number of tuples."""
        out = _SZ(0)
        _check(lib().hkv_load_files(self._h, str(keys_path).encode(),
                                    str(values_path).encode(), str(scores_path).encode(),
                                    max_workspace_size, _stream(stream), ctypes.byref(out)))
        return out.value

    def contains(self, n, keys, founds, stream=None):
        _check(lib().hkv_contains(self._h, n, _ptr(keys), _ptr(founds),
                                  _stream(stream)))

    def erase(self, n, keys, stream=None):
        _check(lib().hkv_erase(self._h, n, _ptr(keys), _stream(stream)))

    def clear(self, stream=None):
        _check(lib().hkv_clear(self._h, _stream(stream)))

    def export_batch(self, n, offset, keys, values, scores=None, stream=None,
                     d_counter=None):
        """Without d_counter returns the exported count (synchronises)."""
        if d_counter is not None:
            _check(lib().hkv_export_batch(self._h, n, offset, _ptr(d_counter),
                                          _ptr(keys), _ptr(values),
                                          _ptr(scores), _stream(stream)))
            return None
        cnt = ctypes.c_size_t(0)
        _check(lib().hkv_export_batch_count(self._h, n, offset, _ptr(keys),
                                            _ptr(values), _ptr(scores),
                                            _stream(stream), ctypes.byref(cnt)))
        return cnt.value

    # -- properties ------------------------------------------------------------
    def size(self, stream=None) -> int:
        out = ctypes.c_size_t(0)
        _check(lib().hkv_size(self._h, _stream(stream), ctypes.byref(out)))
        return out.value

    def empty(self, stream=None) -> bool:
        return self.size(stream) == 0

    def capacity(self) -> int:
        out = ctypes.c_size_t(0)
        _check(lib().hkv_capacity(self._h, ctypes.byref(out)))
        return out.value

    def load_factor(self, stream=None) -> float:
        out = ctypes.c_float(0)
        _check(lib().hkv_load_factor(self._h, _stream(stream), ctypes.byref(out)))
        return out.value

    def dim(self) -> int:
        out = ctypes.c_size_t(0)
        _check(lib().hkv_dim(self._h, ctypes.byref(out)))
        return out.value

    def max_bucket_size(self) -> int:
        out = ctypes.c_size_t(0)
        _check(lib().hkv_max_bucket_size(self._h, ctypes.byref(out)))
        return out.value

    def bucket_count(self) -> int:
        out = ctypes.c_size_t(0)
        _check(lib().hkv_bucket_count(self._h, ctypes.byref(out)))
        return out.value

    def is_pure_hbm_mode(self) -> bool:
        out = ctypes.c_bool(False)
        _check(lib().hkv_is_pure_hbm_mode(self._h, ctypes.byref(out)))
        return out.value

    def reserve(self, new_capacity, stream=None):
        _check(lib().hkv_reserve(self._h, new_capacity, _stream(stream)))

    def set_max_capacity(self, new_max_capacity):
        """set_max_capacity, reference hkv_hashtable.h:2955-2977."""
        _check(lib().hkv_set_max_capacity(self._h, new_max_capacity))

    def raw_view(self):
        """Addresses of the raw table arrays (hkv_table_view): keys, scores,
        digests, sizes, slices (device array of slice addresses), capacity,
        num_buckets, slice_shift, value_bytes."""

        class _View(ctypes.Structure):
            _fields_ = [("keys", _P), ("scores", _P), ("digests", _P), ("sizes", _P),
                        ("slices", _P), ("capacity", _U64), ("num_buckets", _U64),
                        ("bucket_size", ctypes.c_uint32), ("slice_shift", ctypes.c_uint32),
                        ("value_bytes", ctypes.c_uint32), ("dim", ctypes.c_uint32),
                        ("reclaim_digest", ctypes.c_uint8)]

        v = _View()
        _check(lib().hkv_table_get_view(self._h, ctypes.byref(v)))
        return {f: getattr(v, f) for f, _ in _View._fields_}

    def set_global_epoch(self, epoch: int):
        _check(lib().hkv_set_global_epoch(self._h, epoch))

    def check_device_error(self, stream=None):
        _check(lib().hkv_check_device_error(self._h, _stream(stream)))

    # -- test support ------------------------------------------------------
    def get_state(self):
        """Raw slot state as numpy arrays (keys, scores, digests, sizes, values)."""
        import numpy as np

        cap, nb, dim = self.capacity(), self.bucket_count(), self.dim()
        keys = np.empty(cap, np.uint64)
        scores = np.empty(cap, np.uint64)
        digests = np.empty(cap, np.uint8)
        sizes = np.empty(nb, np.int32)
        vt = np.dtype(self.value_dtype) if self.value_dtype != "bfloat16" else np.uint16
        values = np.empty(cap * dim, vt)
        _check(lib().hkv_debug_get_state(self._h, keys.ctypes.data, scores.ctypes.data,
                                         digests.ctypes.data, sizes.ctypes.data,
                                         values.ctypes.data))
        return keys, scores, digests, sizes, values.reshape(cap, dim)

    def set_state(self, keys=None, scores=None, digests=None, sizes=None, values=None):
        def p(a):
            return None if a is None else a.ctypes.data

        _check(lib().hkv_debug_set_state(self._h, p(keys), p(scores), p(digests),
                                         p(sizes), p(values)))


class ShardedHashTable:
    """One table shard per rank; collective calls route keys to their owner
    over NCCL all-to-all (no reference counterpart)."""

    TRANSPORTS = {0: "nccl", 1: "peer"}

    def __init__(self, options: HashTableOptions, rank: int, world_size: int,
                 nccl_id: bytes, evict_strategy: int = EvictStrategy.kLru,
                 key_dtype: str = "uint64", value_dtype: str = "float32",
                 max_batch: int = 1 << 20):
        """Collective. max_batch > 0 asks for the peer-memory transport
        (every call's n on every rank at most max_batch); 0 selects NCCL."""
        h = ctypes.c_void_p()
        o = options._c()
        buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        _check(lib().hkv_sharded_create(ctypes.byref(o),
                                        KEY_I64 if key_dtype == "int64" else KEY_U64,
                                        VALUE_TYPES[value_dtype], evict_strategy,
                                        buf, rank, world_size, max_batch,
                                        ctypes.byref(h)))
        self._h = h.value
        self.rank, self.world_size = rank, world_size

    @property
    def transport(self) -> str:
        out = ctypes.c_int(0)
        _check(lib().hkv_sharded_transport(self._h, ctypes.byref(out)))
        return self.TRANSPORTS[out.value]

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        _check(lib().hkv_nccl_unique_id(buf))
        return buf.raw

    def close(self):
        if self._h is not None:
            _check(lib().hkv_sharded_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def find_or_insert(self, n, keys, values, scores=None, stream=None,
                       unique_key=False):
        _check(lib().hkv_sharded_find_or_insert(self._h, n, _ptr(keys), _ptr(values),
                                                _ptr(scores), _stream(stream),
                                                unique_key))

    def find(self, n, keys, values, founds, scores=None, stream=None):
        _check(lib().hkv_sharded_find(self._h, n, _ptr(keys), _ptr(values),
                                      _ptr(founds), _ptr(scores), _stream(stream)))

    def insert_or_assign(self, n, keys, values, scores=None, stream=None,
                         unique_key=False):
        _check(lib().hkv_sharded_insert_or_assign(self._h, n, _ptr(keys), _ptr(values),
                                                  _ptr(scores), _stream(stream),
                                                  unique_key))

    def size(self, stream=None) -> int:
        out = ctypes.c_size_t(0)
        _check(lib().hkv_sharded_size(self._h, _stream(stream), ctypes.byref(out)))
        return out.value
