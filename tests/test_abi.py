"""The C ABI library loads and exports every entry point include/hkv_b200.h
declares (CPU only: nothing here touches a GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hkv_b200.h")
LIB = os.path.join(ROOT, "hierarchicalkv-ascend_b200", "libhkv_b200.so")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_\s\*]*?\b(hkv_[a-z0-9_]+)\s*\(",
                       text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_api():
    names = declared_functions()
    for must in ("hkv_table_create", "hkv_find", "hkv_insert_or_assign",
                 "hkv_insert_and_evict", "hkv_find_or_insert", "hkv_accum_or_assign",
                 "hkv_assign_scores", "hkv_erase", "hkv_export_batch", "hkv_reserve",
                 "hkv_set_global_epoch", "hkv_contains", "hkv_size"):
        assert must in names


def test_library_exports_every_declared_symbol():
    if not os.path.exists(LIB):
        pytest.fail("libhkv_b200.so is not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_signatures_cover_the_header():
    import hkv_b200

    assert set(declared_functions()) <= set(hkv_b200.SIGNATURES)
    hkv_b200.load_library()  # every declared signature resolves


def test_options_defaults_match_reference():
    """hkv_options_init gives the reference's HashTableOptions defaults
    (hashtable_options.h:535-562)."""
    import hkv_b200

    lib = hkv_b200.load_library()
    o = hkv_b200._Options()
    lib.hkv_options_init(ctypes.byref(o))
    assert o.max_bucket_size == 128 and o.dim == 64
    assert abs(o.max_load_factor - 0.5) < 1e-7 and o.device_id == -1
    assert o.block_size == 128 and o.io_block_size == 1024
    assert o.num_of_buckets_per_alloc == 1 and o.api_lock == 0
