"""A caller's allocator (reference allocator.h BaseAllocator, taken by
HashTable::init, hkv_hashtable.h:962-978) supplies every allocation of the
table: the bucket arrays and value slices at creation and at each doubling,
host value slices as mapped pinned memory, and per-call scratch. Checked
through the Python binding with a counting allocator and with the PyTorch
caching-allocator adapter (GPU)."""
import numpy as np
import pytest
import torch

import hkv_b200 as H
from hkv_gpu import GpuOps, dev
from hkv_testutil import random_keys

pytestmark = pytest.mark.gpu


class Counting:
    """Device and pinned blocks from torch, recorded by address."""

    def __init__(self):
        self.blocks = {}
        self.calls = {"alloc": 0, "free": 0, "alloc_async": 0, "free_async": 0}
        self.flags = []

    def alloc(self, mt, size, flags=0):
        self.calls["alloc"] += 1
        n = max(size, 1)
        if mt == H.MEMORY_DEVICE:
            t = torch.empty(n, dtype=torch.uint8, device="cuda")
        else:
            t = torch.empty(n, dtype=torch.uint8, pin_memory=True)
            self.flags.append((size, flags))
        self.blocks[t.data_ptr()] = (mt, size, t)
        return t.data_ptr()

    def free(self, mt, addr):
        self.calls["free"] += 1
        assert addr in self.blocks and self.blocks[addr][0] == mt
        del self.blocks[addr]

    def owns(self, addr, length, mt=H.MEMORY_DEVICE):
        return any(m == mt and a <= addr and addr + length <= a + s
                   for a, (m, s, _) in self.blocks.items())

    def bytes(self, mt):
        return sum(s for m, s, _ in self.blocks.values() if m == mt)


class CountingAsync(Counting):
    """Also takes per-call scratch stream-ordered (alloc_async/free_async)."""

    def alloc_async(self, mt, size, stream):
        self.calls["alloc_async"] += 1
        return Counting.alloc(self, mt, size)

    def free_async(self, mt, addr, stream):
        self.calls["free_async"] += 1
        torch.cuda.synchronize()  # scratch may still be read on `stream`
        Counting.free(self, mt, addr)


def table_with(alloc, cap=128 * 64, max_cap=128 * 256, dim=16, max_hbm=1 << 30):
    t = H.HashTable(H.EvictStrategy.kLru)
    t.init(H.HashTableOptions(init_capacity=cap, max_capacity=max_cap,
                              max_hbm_for_vectors=max_hbm, dim=dim,
                              max_load_factor=1.0), allocator=alloc)
    return t


@pytest.mark.parametrize("kind", [Counting, CountingAsync])
def test_every_table_allocation_comes_from_the_allocator(kind):
    a = kind()
    cap, dim = 128 * 64, 16
    t = table_with(a, cap, dim=dim)
    v = t.raw_view()
    assert a.owns(v["keys"], cap * 8) and a.owns(v["scores"], cap * 8)
    assert a.owns(v["digests"], cap) and a.owns(v["sizes"], (cap // 128) * 4)
    assert a.owns(v["slices"], 8)
    # the value slice (one slice of every bucket's rows) is one of its blocks
    assert any(m == H.MEMORY_DEVICE and s == cap * dim * 4 for m, s, _ in a.blocks.values())
    assert a.bytes(H.MEMORY_DEVICE) >= cap * (8 + 8 + 1 + dim * 4)
    g = GpuOps(t, dim)
    rng = np.random.default_rng(5)
    keys = random_keys(rng, 3000)
    vals = rng.standard_normal((3000, dim)).astype(np.float32)
    g.insert_or_assign(keys, vals, unique=False)  # the duplicate merge takes scratch
    if kind is CountingAsync:
        assert a.calls["alloc_async"] > 0 and a.calls["free_async"] == a.calls["alloc_async"]
    assert t.size() == 3000
    dev_before = a.bytes(H.MEMORY_DEVICE)
    frees_before = a.calls["free"]
    t.reserve(2 * cap)
    assert t.capacity() == 2 * cap
    v2 = t.raw_view()
    assert a.owns(v2["keys"], 2 * cap * 8) and a.owns(v2["scores"], 2 * cap * 8)
    assert a.calls["free"] >= frees_before + 4  # the old bucket arrays went back
    assert a.bytes(H.MEMORY_DEVICE) > dev_before
    got, f, _ = g.find(keys)
    assert f.all() and (got == vals).all()
    t.set_max_capacity(128 * 1024)
    t.reserve(128 * 512)
    assert t.capacity() == 128 * 512
    got, f, _ = g.find(keys)
    assert f.all() and (got == vals).all()
    t.close()
    assert not a.blocks  # every block went back


def test_host_value_slices_are_mapped_pinned_memory():
    a = Counting()
    cap, dim = 128 * 64, 16
    t = table_with(a, cap, cap, dim=dim, max_hbm=0)
    assert not t.is_pure_hbm_mode()
    assert any(size >= cap * dim * 4 and flags & 1 for size, flags in a.flags)  # cudaHostAllocMapped
    g = GpuOps(t, dim)
    rng = np.random.default_rng(6)
    keys = random_keys(rng, 2000)
    vals = rng.standard_normal((2000, dim)).astype(np.float32)
    g.insert_or_assign(keys, vals)
    got, f, _ = g.find(keys)
    assert f.all() and (got == vals).all()
    t.close()
    assert not a.blocks


def test_torch_allocator_adapter():
    a = H.TorchAllocator()
    before = torch.cuda.memory_allocated()
    cap, dim = 128 * 256, 32
    t = table_with(a, cap, cap, dim=dim)
    # the table's bytes show in torch's own accounting
    assert torch.cuda.memory_allocated() - before >= cap * (8 + 8 + 1 + dim * 4)
    g = GpuOps(t, dim)
    rng = np.random.default_rng(7)
    keys = random_keys(rng, 5000)
    vals = rng.standard_normal((5000, dim)).astype(np.float32)
    g.insert_or_assign(keys, vals)
    got, f, _ = g.find(keys)
    assert f.all() and (got == vals).all()
    t.close()
    assert not a.blocks
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before


def test_a_failing_allocator_fails_the_call():
    class Refuses(Counting):
        def alloc(self, mt, size, flags=0):
            if size > 1 << 22:  # a 16 MiB value slice, after the bucket arrays
                raise MemoryError("no")
            return Counting.alloc(self, mt, size, flags)

    a = Refuses()
    with pytest.raises(H.CudaException):
        table_with(a, 128 * 4096, 128 * 4096, dim=64)
    assert not a.blocks  # what was taken before the failure went back


def test_a_reserve_that_fails_leaves_the_table_as_it_was():
    """The second new value slice is refused: reserve raises, every block it
    took goes back, and the table keeps its capacity, size and contents."""

    class RefusesSecondSlice(Counting):
        armed = False
        seen = 0

        def alloc(self, mt, size, flags=0):
            if self.armed and size == 64 * 128 * 16 * 4:  # one 64-bucket value slice
                self.seen += 1
                if self.seen == 2:
                    raise MemoryError("no")
            return Counting.alloc(self, mt, size, flags)

    a = RefusesSecondSlice()
    cap, dim = 128 * 64, 16
    t = table_with(a, cap, 128 * 256, dim=dim)
    rng = np.random.default_rng(77)
    keys = np.unique(rng.integers(1, 1 << 62, 6000, dtype=np.uint64))[:5000]
    vals = rng.standard_normal((len(keys), dim)).astype(np.float32)
    t.insert_or_assign(len(keys), torch.from_numpy(keys.view(np.int64)).cuda(),
                       torch.from_numpy(vals).cuda())
    torch.cuda.synchronize()
    size_before = t.size()
    held = set(a.blocks)
    a.armed = True
    with pytest.raises(H.CudaException):
        t.reserve(128 * 256)
    a.armed = False
    assert set(a.blocks) == held  # the call's new arrays and slices went back
    assert t.capacity() == cap and t.size() == size_before
    got = torch.zeros((len(keys), dim), device="cuda")
    f = torch.zeros(len(keys), dtype=torch.bool, device="cuda")
    t.find(len(keys), torch.from_numpy(keys.view(np.int64)).cuda(), got, f)
    torch.cuda.synchronize()
    ok = f.cpu().numpy()
    assert ok.sum() == size_before
    assert (got.cpu().numpy()[ok] == vals[ok]).all()
    # and it can still grow
    t.reserve(128 * 256)
    assert t.capacity() == 128 * 256 and t.size() == size_before
    t.close()
