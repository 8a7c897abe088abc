"""save / load through the reference's LocalKVFile format (GPU).

Reference: HashTable::save / load (hkv_hashtable.h:3021-3195) and
LocalKVFile (types.h:349-464): three files of raw keys, raw value rows and
raw uint64 scores, one tuple per live slot, written chunk by chunk (each
chunk is an export of max_workspace_size / tuple-size slots, in an order
that is not specified inside a chunk); load reads chunks of the same size and
inserts each with insert_or_assign(unique_key=true,
ignore_evict_strategy=true) after setting the global epoch to
IGNORED_GLOBAL_EPOCH, where it stays.
"""
import numpy as np
import pytest

import hkv_b200 as H
import hkv_oracle as O
from hkv_gpu import GpuOps, make_table
from hkv_testutil import live_set

pytestmark = pytest.mark.gpu


def read_files(base, dim):
    k = np.fromfile(f"{base}_keys", dtype=np.uint64)
    v = np.fromfile(f"{base}_values", dtype=np.float32).reshape(-1, dim)
    s = np.fromfile(f"{base}_scores", dtype=np.uint64)
    return k, v, s


def test_save_writes_every_live_tuple(tmp_path):
    rng = np.random.default_rng(11)
    dim = 8
    t = make_table(128 * 64, dim=dim, strategy=H.EvictStrategy.kCustomized)
    ops = GpuOps(t, dim)
    keys = np.unique(rng.integers(1, 1 << 62, 12000, dtype=np.uint64))[:10000]
    ops.insert_or_assign(keys, rng.standard_normal((len(keys), dim)).astype(np.float32),
                         rng.permutation(np.arange(1, len(keys) + 1, dtype=np.uint64)))
    base = tmp_path / "t"
    n = t.save(f"{base}_keys", f"{base}_values", f"{base}_scores",
               max_workspace_size=40 * 1024)  # many chunks
    k, v, s = read_files(base, dim)
    assert n == len(k) == len(v) == len(s) == t.size()
    assert len(np.unique(k)) == len(k)
    sk, ss, _, _, sv = t.get_state()
    assert live_set(k, s, v) == live_set(sk, ss, sv)


@pytest.mark.parametrize("ws", [1 << 20, 24 * 1024])
def test_load_matches_oracle(tmp_path, ws):
    rng = np.random.default_rng(12)
    dim, cap = 4, 128 * 32
    keys = np.unique(rng.integers(1, 1 << 62, 9000, dtype=np.uint64))[:8000]
    keys = rng.permutation(keys)
    vals = rng.standard_normal((len(keys), dim)).astype(np.float32)
    scores = rng.permutation(np.arange(1, 3 * len(keys), dtype=np.uint64))[:len(keys)]
    base = tmp_path / "f"
    keys.tofile(f"{base}_keys")
    vals.tofile(f"{base}_values")
    scores.tofile(f"{base}_scores")
    # an Lru table: load ignores the strategy and uses the file's scores
    t = make_table(cap, dim=dim, strategy=H.EvictStrategy.kLru)
    n = t.load(f"{base}_keys", f"{base}_values", f"{base}_scores", max_workspace_size=ws)
    assert n == len(keys)
    t.check_device_error()
    o = O.OracleTable(cap, cap, dim=dim, strategy=O.LRU)
    o.load_chunks(keys, vals, scores, ws)
    gk, gs, _, gz, gv = t.get_state()
    ok, osc, _, oz, ov = o.get_state()
    assert (gz == oz).all()
    assert live_set(gk, gs, gv) == live_set(ok, osc, ov)


def test_round_trip_and_epoch(tmp_path):
    rng = np.random.default_rng(13)
    dim = 16
    a = make_table(128 * 64, dim=dim, strategy=H.EvictStrategy.kEpochLfu, epoch=5)
    ops = GpuOps(a, dim)
    keys = np.unique(rng.integers(1, 1 << 62, 6000, dtype=np.uint64))[:5000]
    ops.insert_or_assign(keys, rng.standard_normal((len(keys), dim)).astype(np.float32),
                         rng.integers(1, 1000, len(keys)).astype(np.uint64))
    base = tmp_path / "r"
    assert a.save(f"{base}_keys", f"{base}_values", f"{base}_scores") == len(keys)
    b = make_table(128 * 64, dim=dim, strategy=H.EvictStrategy.kEpochLfu, epoch=5)
    assert b.load(f"{base}_keys", f"{base}_values", f"{base}_scores") == len(keys)
    ak, as_, _, _, av = a.get_state()
    bk, bs, _, _, bv = b.get_state()
    assert live_set(ak, as_, av) == live_set(bk, bs, bv)
    # load leaves the global epoch at IGNORED_GLOBAL_EPOCH: an EpochLfu insert
    # is refused until the caller sets an epoch again
    with pytest.raises(H.HkvException):
        GpuOps(b, dim).insert_or_assign(keys[:4], np.zeros((4, dim), np.float32),
                                        np.ones(4, np.uint64))
    b.set_global_epoch(6)
    GpuOps(b, dim).insert_or_assign(keys[:4], np.zeros((4, dim), np.float32),
                                    np.ones(4, np.uint64))


def test_save_load_argument_checks(tmp_path):
    t = make_table(128 * 8, dim=8)
    with pytest.raises(H.HkvException):  # smaller than one tuple
        t.save(tmp_path / "k", tmp_path / "v", tmp_path / "s", max_workspace_size=16)
    with pytest.raises(RuntimeError):  # no such files
        t.load(tmp_path / "nok", tmp_path / "nov", tmp_path / "nos")
