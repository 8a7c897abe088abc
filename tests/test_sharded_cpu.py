"""World-size-2 gloo run of the sharded exchange protocol on CPU: two ranks,
each with an oracle shard, together give what one table gives for the
concatenation of their batches (no GPU)."""
import os
import socket

import numpy as np
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _batches(world, step):
    rng = np.random.default_rng(100 + step)
    pool = np.unique(rng.integers(1, 1 << 62, 3000, dtype=np.uint64))
    out = []
    for r in range(world):
        k = rng.choice(pool, 2000, replace=True).astype(np.uint64)
        v = rng.standard_normal((2000, 4)).astype(np.float32)
        s = rng.integers(1, 17, 2000).astype(np.uint64)
        out.append((k, v, s))
    return out


def _rank(rank, world, port, outdir):
    import sys

    for p in (os.path.join(ROOT, "tests"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist

    import hkv_oracle as O
    from sharded_protocol import owner, sharded_find_or_insert

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shard = O.OracleTable(128 * 64, 128 * 64, dim=4, strategy=O.LFU)
    results = []
    for step in range(3):
        k, v, s = _batches(world, step)[rank]
        results.append(sharded_find_or_insert(shard, k, v.copy(), s))
    keys, scores, _, _, vals = shard.get_state()
    live = keys < np.uint64(0xFFFFFFFFFFFFFFFC)
    assert (owner(keys[live], world) == rank).all()  # shards hold own keys only
    np.savez(os.path.join(outdir, f"r{rank}.npz"), *results, keys=keys[live],
             scores=scores[live], vals=vals[live])
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_match_one_table(tmp_path):
    import sys

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import hkv_oracle as O

    world = 2
    ctx = mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)),
                             nprocs=world, join=False, start_method="spawn")
    while not ctx.join(timeout=120):
        pass
    one = O.OracleTable(128 * 128, 128 * 128, dim=4, strategy=O.LFU)
    res = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    for step in range(3):
        bs = _batches(world, step)
        keys = np.concatenate([b[0] for b in bs])
        vals = np.concatenate([b[1] for b in bs])
        sc = np.concatenate([b[2] for b in bs])
        out, _ = one.find_or_insert(keys, vals, sc)
        off = 0
        for r in range(world):
            n = len(bs[r][0])
            assert (res[r][f"arr_{step}"] == out[off:off + n]).all()
            off += n
    gk = np.concatenate([r["keys"] for r in res])
    gs = np.concatenate([r["scores"] for r in res])
    _, f, s = one.find(gk)
    assert f.all() and (s == gs).all() and one.size() == len(gk)
