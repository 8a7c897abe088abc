"""The sharded table on every visible GPU (one process per GPU), over both
transports (peer memory and NCCL), gives what one table gives for the
concatenation of the ranks' batches, and each shard holds only the keys it
owns (gpu; skipped with fewer than 2 GPUs)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from test_sharded_cpu import _batches

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _unique_batch(world, rank, seed=500):
    rng = np.random.default_rng(seed)
    pool = np.unique(rng.integers(1, 1 << 62, 2500, dtype=np.uint64))
    out = []
    for r in range(world):
        k = rng.choice(pool, 1500, replace=False).astype(np.uint64)
        out.append((k, rng.standard_normal((1500, 4)).astype(np.float32),
                    rng.integers(1, 17, 1500).astype(np.uint64)))
    return out[rank]


def _rank(rank, world, port, outdir, max_batch):
    import sys
    from datetime import timedelta

    for p in (os.path.join(ROOT, "tests"), os.path.join(ROOT, "oracle"),
              os.path.join(ROOT, "hierarchicalkv-ascend_b200")):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    import hkv_b200 as H
    from sharded_protocol import owner

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    uid = [H.ShardedHashTable.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    opts = H.HashTableOptions(init_capacity=128 * 64, max_capacity=128 * 64,
                              max_hbm_for_vectors=1 << 30, dim=4, device_id=rank)
    t = H.ShardedHashTable(opts, rank, world, uid[0], H.EvictStrategy.kLfu,
                           max_batch=max_batch)
    transport = t.transport
    results = []
    for step in range(3):
        k, v, s = _batches(world, step)[rank]
        dv = torch.from_numpy(v).cuda()
        t.find_or_insert(len(k), torch.from_numpy(k.view(np.int64)).cuda(), dv,
                         torch.from_numpy(s.view(np.int64)).cuda())
        torch.cuda.synchronize()
        results.append(dv.cpu().numpy())
    # unique-key insert_or_assign (distinct within a rank, shared across ranks)
    uk, uv, us = _unique_batch(world, rank)
    t.insert_or_assign(len(uk), torch.from_numpy(uk.view(np.int64)).cuda(),
                       torch.from_numpy(uv).cuda(), torch.from_numpy(us.view(np.int64)).cuda(),
                       unique_key=True)
    torch.cuda.synchronize()
    # unique-key find_or_insert: some keys new, some inserted just above; a
    # key several ranks send is inserted by the lowest rank and found by the
    # others
    fk, fvals, fsc = _unique_batch(world, rank, seed=501)
    fk[: len(fk) // 2] = uk[: len(fk) // 2]
    fdv = torch.from_numpy(fvals).cuda()
    t.find_or_insert(len(fk), torch.from_numpy(fk.view(np.int64)).cuda(), fdv,
                     torch.from_numpy(fsc.view(np.int64)).cuda(), unique_key=True)
    torch.cuda.synchronize()
    fio = fdv.cpu().numpy()
    # collective find of every rank's first batch
    k0, _, _ = _batches(world, 0)[rank]
    fv = torch.zeros((len(k0), 4), device="cuda")
    ff = torch.zeros(len(k0), dtype=torch.bool, device="cuda")
    fs = torch.zeros(len(k0), dtype=torch.int64, device="cuda")
    t.find(len(k0), torch.from_numpy(k0.view(np.int64)).cuda(), fv, ff, fs)
    total = t.size()
    local = H.HashTable.borrow(H.lib().hkv_sharded_local(t._h), H.EvictStrategy.kLfu)
    keys, scores, _, _, vals = local.get_state()
    live = keys < np.uint64(0xFFFFFFFFFFFFFFFC)
    own_ok = bool((owner(keys[live], world) == rank).all())
    np.savez(os.path.join(outdir, f"r{rank}.npz"), *results, keys=keys[live],
             scores=scores[live], fv=fv.cpu().numpy(), ff=ff.cpu().numpy(),
             fs=fs.cpu().numpy().view(np.uint64), total=np.array([total]),
             own_ok=np.array([own_ok]), transport=np.array([transport]), fio=fio)
    dist.barrier()
    t.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport,max_batch", [("peer", 4096), ("nccl", 0)])
def test_sharded_gpus_match_one_table(tmp_path, transport, max_batch):
    """One rank per visible GPU (2, 4 or 8)."""
    import sys

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import hkv_oracle as O

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path), max_batch),
                             nprocs=world, join=False, start_method="spawn")
    while not ctx.join(timeout=180):
        pass
    res = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    assert all(str(r["transport"][0]) == transport for r in res)
    assert all(bool(r["own_ok"][0]) for r in res)
    # as many slots as the shards together: no bucket of either overflows
    one = O.OracleTable(world * 128 * 64, world * 128 * 64, dim=4, strategy=O.LFU)
    for step in range(3):
        bs = _batches(world, step)
        out, _ = one.find_or_insert(np.concatenate([b[0] for b in bs]),
                                    np.concatenate([b[1] for b in bs]),
                                    np.concatenate([b[2] for b in bs]))
        off = 0
        for r in range(world):
            n = len(bs[r][0])
            assert (res[r][f"arr_{step}"] == out[off:off + n]).all(), (step, r)
            off += n
    ub = [_unique_batch(world, r) for r in range(world)]
    one.insert_or_assign(np.concatenate([b[0] for b in ub]), np.concatenate([b[1] for b in ub]),
                         np.concatenate([b[2] for b in ub]))
    fb = []
    for r in range(world):
        fk, fvals, fsc = _unique_batch(world, r, seed=501)
        fk[: len(fk) // 2] = ub[r][0][: len(fk) // 2]
        fb.append((fk, fvals, fsc))
    out, _ = one.find_or_insert(np.concatenate([b[0] for b in fb]),
                                np.concatenate([b[1] for b in fb]),
                                np.concatenate([b[2] for b in fb]))
    off = 0
    for r in range(world):
        n = len(fb[r][0])
        assert (res[r]["fio"] == out[off:off + n]).all(), ("unique find_or_insert", r)
        off += n
    gk = np.concatenate([r["keys"] for r in res])
    gs = np.concatenate([r["scores"] for r in res])
    _, f, s = one.find(gk)
    assert f.all() and (s == gs).all()
    assert int(res[0]["total"][0]) == one.size() == len(gk)
    for r in range(world):
        k0 = _batches(world, 0)[r][0]
        ov, of, osc = one.find(k0)
        assert (res[r]["ff"] == of).all() and (res[r]["fv"] == ov).all()
        assert (res[r]["fs"][of] == osc[of]).all()
