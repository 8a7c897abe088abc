"""Python restatement of the sharded table's exchange protocol (test
infrastructure; the product is hierarchicalkv-ascend_b200/csrc/hkv_sharded.cu).

Per collective call every rank:
  1. merges duplicate keys of its batch (first occurrence represents a key,
     Lfu scores are summed),
  2. routes each distinct key to owner = (Murmur3(key) >> 40) % world,
  3. exchanges counts, then keys, scores and value rows (all-to-all),
  4. applies the operation on its own shard to what it received, merging
     keys that several ranks sent (earlier ranks first),
  5. sends result rows back and scatters them to every occurrence.
"""
import numpy as np
import torch
import torch.distributed as dist

from hkv_testutil import murmur3_np


def owner(keys, world):
    return ((murmur3_np(keys) >> np.uint64(40)) % np.uint64(world)).astype(np.int64)


def merge(keys, scores):
    """first-occurrence representatives, inverse map, summed scores"""
    uk, first, inv = np.unique(keys, return_index=True, return_inverse=True)
    order = np.argsort(first, kind="stable")
    rank_of = np.empty_like(order)
    rank_of[order] = np.arange(len(order))
    ukeys = uk[order]
    rep = first[order]
    uid = rank_of[inv]
    us = None
    if scores is not None:
        us = np.zeros(len(ukeys), np.uint64)
        np.add.at(us, uid, scores.astype(np.uint64))
    return ukeys, rep, uid, us


def _a2a(send, counts_send, counts_recv, dtype, width=1):
    recv = torch.empty((int(sum(counts_recv)), width), dtype=dtype)
    s = torch.from_numpy(np.ascontiguousarray(send)).reshape(-1, width)
    dist.all_to_all_single(recv, s, [int(c) for c in counts_recv],
                           [int(c) for c in counts_send])
    return recv.numpy()


def sharded_find_or_insert(shard, keys, values, scores):
    """One collective Lfu find_or_insert; `shard` is this rank's OracleTable.
    Returns the values as the caller's buffer holds them afterwards."""
    world = dist.get_world_size()
    ukeys, rep, uid, us = merge(keys, scores)
    dest = owner(ukeys, world)
    order = np.argsort(dest, kind="stable")
    cs = np.bincount(dest, minlength=world)
    cr = torch.empty(world, dtype=torch.int64)
    dist.all_to_all_single(cr, torch.from_numpy(cs.astype(np.int64)))
    cr = cr.numpy()
    dim = values.shape[1]
    rk = _a2a(ukeys[order].view(np.int64), cs, cr, torch.int64).reshape(-1).view(np.uint64)
    rs = _a2a(us[order].view(np.int64), cs, cr, torch.int64).reshape(-1).view(np.uint64)
    rv = _a2a(values[rep[order]], cs, cr, torch.float32, dim)
    out, _ = shard.find_or_insert(rk, rv, rs) if len(rk) else (rv, None)
    back = _a2a(out, cr, cs, torch.float32, dim)
    urows = np.empty((len(ukeys), dim), np.float32)
    urows[order] = back
    return urows[uid]
