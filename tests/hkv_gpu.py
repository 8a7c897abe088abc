"""GPU-side helpers for the `gpu` tests: numpy <-> CUDA tensors and table
construction through the Python binding of the C ABI."""
import numpy as np
import torch

import hkv_b200 as H


def dev(a, dtype=None):
    """numpy -> CUDA tensor (uint64 travels as int64 bits)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    t = torch.from_numpy(a.copy())
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t, dtype=None):
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def zeros_u64(n):
    return torch.zeros(max(n, 1), dtype=torch.int64, device="cuda")


def make_table(capacity, dim=8, strategy=H.EvictStrategy.kCustomized,
               max_capacity=None, max_hbm=1 << 34, max_load_factor=0.5,
               value_dtype="float32", key_dtype="uint64", epoch=None):
    t = H.HashTable(strategy, key_dtype=key_dtype, value_dtype=value_dtype)
    t.init(H.HashTableOptions(init_capacity=capacity,
                              max_capacity=capacity if max_capacity is None else max_capacity,
                              max_hbm_for_vectors=max_hbm, dim=dim,
                              max_load_factor=max_load_factor))
    if epoch is not None:
        t.set_global_epoch(epoch)
    return t


class GpuOps:
    """Convenience wrappers returning numpy results."""

    def __init__(self, table, dim, vdtype=np.float32):
        self.t = table
        self.dim = dim
        self.vdt = vdtype

    def insert_or_assign(self, keys, values, scores=None, unique=True, ignore=False):
        n = len(keys)
        self.t.insert_or_assign(n, dev(keys), dev(np.asarray(values, self.vdt)),
                                None if scores is None else dev(np.asarray(scores, np.uint64)),
                                unique_key=unique, ignore_evict_strategy=ignore)
        torch.cuda.synchronize()

    def find(self, keys, init_value=0.0):
        n = len(keys)
        vals = torch.full((max(n, 1), self.dim), init_value, dtype=torch.float32
                          if self.vdt == np.float32 else torch.float16, device="cuda")
        founds = torch.zeros(max(n, 1), dtype=torch.bool, device="cuda")
        scores = zeros_u64(n)
        self.t.find(n, dev(keys), vals, founds, scores)
        torch.cuda.synchronize()
        return (host(vals)[:n], host(founds)[:n].astype(bool),
                host(scores, np.uint64)[:n])

    def contains(self, keys):
        n = len(keys)
        founds = torch.zeros(max(n, 1), dtype=torch.bool, device="cuda")
        self.t.contains(n, dev(keys), founds)
        torch.cuda.synchronize()
        return host(founds)[:n].astype(bool)

    def find_or_insert(self, keys, values, scores=None, unique=True, ignore=False):
        n = len(keys)
        v = dev(np.asarray(values, self.vdt))
        self.t.find_or_insert(n, dev(keys), v,
                              None if scores is None else dev(np.asarray(scores, np.uint64)),
                              unique_key=unique, ignore_evict_strategy=ignore)
        torch.cuda.synchronize()
        return host(v)

    def insert_and_evict(self, keys, values, scores=None, unique=True, ignore=False):
        n = len(keys)
        ek = zeros_u64(n)
        ev = torch.zeros((max(n, 1), self.dim), dtype=torch.float32, device="cuda")
        es = zeros_u64(n)
        c = self.t.insert_and_evict(n, dev(keys), dev(np.asarray(values, self.vdt)),
                                    None if scores is None else dev(np.asarray(scores, np.uint64)),
                                    ek, ev, es, unique_key=unique,
                                    ignore_evict_strategy=ignore)
        return (host(ek, np.uint64)[:c], host(ev)[:c], host(es, np.uint64)[:c])

    def accum_or_assign(self, keys, values, accum, scores=None):
        n = len(keys)
        self.t.accum_or_assign(n, dev(keys), dev(np.asarray(values, self.vdt)),
                               dev(np.asarray(accum, bool)),
                               None if scores is None else dev(np.asarray(scores, np.uint64)))
        torch.cuda.synchronize()

    def assign_scores(self, keys, scores=None):
        n = len(keys)
        self.t.assign_scores(n, dev(keys),
                             None if scores is None else dev(np.asarray(scores, np.uint64)))
        torch.cuda.synchronize()

    def erase(self, keys):
        self.t.erase(len(keys), dev(keys))
        torch.cuda.synchronize()

    def export(self, n, offset=0):
        k = zeros_u64(n)
        v = torch.zeros((max(n, 1), self.dim), dtype=torch.float32, device="cuda")
        s = zeros_u64(n)
        c = self.t.export_batch(n, offset, k, v, s)
        return host(k, np.uint64)[:c], host(v)[:c], host(s, np.uint64)[:c]
