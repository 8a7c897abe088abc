"""Golden fixtures (tests/golden/*.npz, written by tests/golden/make_golden.py):
the oracle must reproduce them (CPU), and the CUDA path through the C ABI
must give the same values, flags, scores and table contents bit for bit
(GPU). Each case is one whose result does not depend on thread order."""
import os

import numpy as np
import pytest

import hkv_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
RESERVED_MIN = np.uint64(0xFFFFFFFFFFFFFFFC)


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def sorted_live(keys, scores, values):
    live = keys < RESERVED_MIN
    order = np.argsort(keys[live])
    return keys[live][order], scores[live][order], values[live][order]


def assert_state(got, g):
    k, s, v = got
    np.testing.assert_array_equal(k, g["state_keys"])
    np.testing.assert_array_equal(s, g["state_scores"])
    np.testing.assert_array_equal(v, g["state_values"])


# ------------------------------------------------------------------- drivers
class OracleDriver:
    def __init__(self, cap, dim, strategy, epoch=None):
        self.t = O.OracleTable(cap, cap, dim=dim, strategy=strategy)
        if epoch is not None:
            self.t.set_global_epoch(epoch)

    def insert_or_assign(self, k, v, s):
        self.t.insert_or_assign(k, v, s)

    def find_or_insert_dups(self, k, v, s):
        return self.t.find_or_insert(k, v, s)[0]

    def insert_and_evict(self, k, v, s):
        ek, ev, es, _ = self.t.insert_and_evict(k, v, s)
        return ek, ev, es

    def find(self, k):
        return self.t.find(k)

    def assign_scores(self, k, s):
        self.t.assign_scores(k, s)

    def erase(self, k):
        self.t.erase(k)

    def state(self):
        keys, scores, _, _, values = self.t.get_state()
        return sorted_live(keys, scores, values)


class GpuDriver:
    def __init__(self, cap, dim, strategy, epoch=None):
        import hkv_b200 as H
        from hkv_gpu import GpuOps, make_table

        hs = {O.LRU: H.EvictStrategy.kLru, O.LFU: H.EvictStrategy.kLfu,
              O.EPOCH_LRU: H.EvictStrategy.kEpochLru, O.EPOCH_LFU: H.EvictStrategy.kEpochLfu,
              O.CUSTOMIZED: H.EvictStrategy.kCustomized}[strategy]
        self.t = make_table(cap, dim=dim, strategy=hs, epoch=epoch)
        self.ops = GpuOps(self.t, dim)

    def insert_or_assign(self, k, v, s):
        self.ops.insert_or_assign(k, v, s)

    def find_or_insert_dups(self, k, v, s):
        return self.ops.find_or_insert(k, v, s, unique=False)

    def insert_and_evict(self, k, v, s):
        return self.ops.insert_and_evict(k, v, s)

    def find(self, k):
        return self.ops.find(k)

    def assign_scores(self, k, s):
        self.ops.assign_scores(k, s)

    def erase(self, k):
        self.ops.erase(k)

    def state(self):
        self.t.check_device_error()
        keys, scores, _, _, values = self.t.get_state()
        return sorted_live(keys, scores, values)


# --------------------------------------------------------------------- cases
def run_customized_batches(D):
    g = load("customized_batches")
    d = D(int(g["capacity"]), int(g["dim"]), O.CUSTOMIZED)
    for b in range(3):
        d.insert_or_assign(g[f"keys{b}"], g[f"vals{b}"], g[f"scores{b}"])
    d.insert_or_assign(g["hit_keys"], g["hit_vals"], g["hit_scores"])
    fv, ff, fs = d.find(g["find_keys"])
    np.testing.assert_array_equal(ff, g["find_founds"])
    np.testing.assert_array_equal(fv[ff], g["find_values"][ff])
    np.testing.assert_array_equal(fs[ff], g["find_scores"][ff])
    assert_state(d.state(), g)


def run_lfu_duplicates(D):
    g = load("lfu_duplicates")
    d = D(int(g["capacity"]), int(g["dim"]), O.LFU)
    for c in range(2):
        got = d.find_or_insert_dups(g[f"keys{c}"], g[f"vals{c}"], g[f"scores{c}"])
        np.testing.assert_array_equal(got, g[f"returned{c}"])
    assert_state(d.state(), g)


def run_insert_and_evict(D):
    g = load("insert_and_evict")
    d = D(int(g["capacity"]), int(g["dim"]), O.CUSTOMIZED)
    d.insert_or_assign(g["pre_keys"], g["pre_vals"], g["pre_scores"])
    ek, ev, es = d.insert_and_evict(g["keys"], g["vals"], g["scores"])
    order = np.argsort(ek)
    np.testing.assert_array_equal(ek[order], g["ev_keys"])
    np.testing.assert_array_equal(ev[order], g["ev_vals"])
    np.testing.assert_array_equal(es[order], g["ev_scores"])
    assert_state(d.state(), g)


def run_epoch_lfu_scores_erase(D):
    g = load("epoch_lfu_scores_erase")
    d = D(int(g["capacity"]), int(g["dim"]), O.EPOCH_LFU, epoch=int(g["epoch"]))
    d.insert_or_assign(g["keys"], g["vals"], g["scores"])
    d.assign_scores(g["assign_keys"], g["assign_scores"])
    d.erase(g["erase_keys"])
    fv, ff, fs = d.find(g["keys"])
    np.testing.assert_array_equal(ff, g["find_founds"])
    np.testing.assert_array_equal(fv[ff], g["find_values"][ff])
    np.testing.assert_array_equal(fs[ff], g["find_scores"][ff])
    assert_state(d.state(), g)


CASES = [run_customized_batches, run_lfu_duplicates, run_insert_and_evict,
         run_epoch_lfu_scores_erase]


@pytest.mark.parametrize("case", CASES, ids=lambda f: f.__name__[4:])
def test_oracle_reproduces_golden(case):
    case(OracleDriver)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda f: f.__name__[4:])
def test_cuda_path_matches_golden(case):
    case(GpuDriver)
