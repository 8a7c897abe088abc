"""Benchmark: B-KV/s of find + insert_or_assign (dim 32, load factor 1.0).

Workload (BASELINE config 2 at LF 1.0, one shard per GPU): uint64 keys,
float32 values of dim 32, 64 Mi slots per GPU, EvictStrategy::kLru, the
table filled to load factor 1.0. One step = find of 1 Mi keys (100% hits)
+ insert_or_assign of 1 Mi keys (50% resident keys, 50% new keys that evict
the least recently used). value = keys of all steps on all GPUs / time.

N = 1 runs the table directly. N > 1 runs the sharded table: every rank
submits its own batches; keys and rows travel to their owner GPU and results
come back over NVLink, by plain peer loads of the other ranks' memory in this
library's own kernels (the peer transport), or by NCCL send/recv where peer
mappings are unavailable (weak scaling: per-GPU table and batch fixed).

`--impl reference` times the reference's algorithm on the host CPU instead
(the reference needs an Ascend NPU and CANN, neither exists here, so its CPU
restatement in oracle/ stands in for it), with every host thread.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "hierarchicalkv-ascend_b200")
ORACLE = os.path.join(ROOT, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "B-KV/s for find & insert_or_assign (dim 32, LF 1.0) at 1/2/4/8 B200; %HBM peak"
UNIT = "B-KV/s"
DIM = 32
VALUE_BYTES = DIM * 4
CAPACITY = 64 << 20          # slots per GPU
BATCH = 1 << 20              # keys per call
PREFILL_FACTOR = 1.6         # inserted keys / capacity to reach LF 1.0 under LRU
HOT = 4 << 20                # most recent prefill keys, source of hits
# algorithmic bytes per key: the key, one 128-byte digest line per bucket
# probe, the 8-byte key compare, the value row read and written, and for an
# evicting insert the 1 KiB score scan
FIND_HIT_BYTES = 145 + 2 * VALUE_BYTES                 # 401
INSERT_HIT_BYTES = 160 + 2 * VALUE_BYTES               # 416
INSERT_EVICT_BYTES = 1185 + 2 * VALUE_BYTES            # 1441
INSERT_MIX_BYTES = 0.5 * (INSERT_HIT_BYTES + INSERT_EVICT_BYTES)  # 928.5


_T0 = time.time()


def log(msg):
    print(f"[bench {time.time() - _T0:7.1f}s] {msg}", file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# --------------------------------------------------------------------------
# key generation on the device: key = Murmur3 finalizer(counter), a bijection
# of uint64, so keys are distinct by construction (int64 bit patterns).
# --------------------------------------------------------------------------
def fmix_t(x):
    import torch

    def srl(v, s):
        return (v >> s) & ((1 << (64 - s)) - 1)

    c1 = 0xFF51AFD7ED558CCD - (1 << 64)
    c2 = 0xC4CEB9FE1A85EC53 - (1 << 64)
    x = x ^ srl(x, 33)
    x = x * c1
    x = x ^ srl(x, 33)
    x = x * c2
    x = x ^ srl(x, 33)
    return x


def key_of(counters):
    import torch

    k = fmix_t(counters)
    # the four reserved keys are -4..-1 as int64; move the (p = 2^-62) hits
    return torch.where(k >= -4, k - 8, k)


def keys_from_counters(start, n, device):
    import torch

    return key_of(torch.arange(start, start + n, dtype=torch.int64, device=device))


def owner_t(keys, world):
    """Owner rank as the sharded table computes it: (Murmur3(key) >> 40) % W."""
    h = fmix_t(keys)
    return ((h >> 40) & ((1 << 24) - 1)) % world


# --------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed
    region (read-only queries)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"hkv_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                rows.append(parts)
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [r for r in rows if r[4].isdigit() and int(r[4]) > 0] or rows
        sm = [float(r[1]) for r in loaded if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in loaded for j in range(4)
                          if r[6 + j].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "samples_under_load": len(loaded)}


# --------------------------------------------------------------------------
def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist

    if n_gpus <= 1:
        return 0, 1, 0, None
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    return rank, world, local, dist


def build_table(world, rank, dist, capacity):
    import torch

    import hkv_b200 as H

    opts = H.HashTableOptions(init_capacity=capacity, max_capacity=capacity,
                              max_hbm_for_vectors=capacity * VALUE_BYTES * 2,
                              dim=DIM, max_load_factor=1.0)
    if world == 1:
        t = H.HashTable(H.EvictStrategy.kLru)
        t.init(opts)
        return t, t
    uid = [H.ShardedHashTable.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    opts.device_id = torch.cuda.current_device()
    s = H.ShardedHashTable(opts, rank, world, uid[0], H.EvictStrategy.kLru,
                           max_batch=0 if os.environ.get("HKV_SHARDED_NCCL") else BATCH)
    log(f"rank {rank}: sharded transport {s.transport}")
    return s, H.HashTable.borrow(H.lib().hkv_sharded_local(s._h), H.EvictStrategy.kLru)


def prefill(local, rank, world, device, capacity):
    """Fill each shard to load factor 1.0 with the keys it owns (every rank
    generates the same global key stream and keeps its own keys)."""
    import torch

    total = int(capacity * world * PREFILL_FACTOR)
    chunk = 4 << 20
    vals = torch.randn((chunk, DIM), device=device)
    start = 0
    while start < total:
        n = min(chunk, total - start)
        k = keys_from_counters(start, n, device)
        if world > 1:
            k = k[owner_t(k, world) == rank]
        m = k.numel()
        local.insert_or_assign(m, k, vals[:m])
        start += n
        if (start // chunk) % 8 == 0 or start >= total:
            torch.cuda.synchronize()
            log(f"prefill {start}/{total} keys")
    torch.cuda.synchronize()
    return total


def prepare_batches(steps, rank, world, total_prefill, device, seed, capacity):
    """Per step: a find batch of resident (hot) keys and an insert batch of
    half hot keys, half never-seen keys. Hot keys are the most recent prefill
    keys of the global stream."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed + rank)
    nhot = min(HOT, capacity // 8) * world
    hot_start = total_prefill - nhot
    fresh_base = total_prefill + rank * (steps + 1) * BATCH
    finds, inserts, vals = [], [], []
    for s in range(steps):
        idx = torch.randint(0, nhot, (BATCH,), generator=g, device=device)
        finds.append(key_of(hot_start + idx))
        perm = torch.randperm(nhot, generator=g, device=device)[: BATCH // 2]
        hot_keys = key_of(hot_start + perm)
        fresh = keys_from_counters(fresh_base + s * BATCH // 2, BATCH // 2, device)
        ins = torch.cat([hot_keys, fresh])
        ins = ins[torch.randperm(BATCH, generator=g, device=device)]
        inserts.append(ins)
        vals.append(torch.rand((BATCH, DIM), generator=g, device=device))
    torch.cuda.synchronize()
    return finds, inserts, vals


def kernel_timeline(step, n, dist, rank, world, label):
    """Per-kernel device time of n calls of step(i) on this rank (torch
    profiler, CUPTI activity records), printed by every rank in rank order as
    one JSON line each. Diagnostics only: a profiled run is never a bench
    value."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for i in range(n):
            step(i)
        torch.cuda.synchronize()
    acc = {}
    for e in prof.events():
        if e.device_type.name != "CUDA":
            continue
        name = e.name.replace("void ", "").replace("hkvb::", "")
        name = name.replace("(anonymous namespace)::", "").split("(")[0][:80]
        c, t = acc.get(name, (0, 0.0))
        acc[name] = (c + 1, t + e.device_time_total)
    rows = sorted(acc.items(), key=lambda kv: -kv[1][1])
    line = {"timeline": label, "rank": rank, "world": world, "calls": n,
            "us_per_call": {k: round(t / n, 1) for k, (c, t) in rows},
            "launches_per_call": {k: round(c / n, 2) for k, (c, t) in rows}}
    for r in range(world):
        if r == rank:
            print(json.dumps(line), flush=True)
        if dist:
            dist.barrier()


def run_gpu(args):
    import numpy as np
    import torch

    import hkv_b200 as H

    rank, world, local_rank, dist = dist_setup(args.gpus)
    device = torch.device("cuda", torch.cuda.current_device())
    cap = args.capacity
    log(f"rank {rank}/{world}: table of {cap} slots")
    table, local = build_table(world, rank, dist, cap)
    transport = table.transport if world > 1 else "none"
    total = prefill(local, rank, world, device, cap)
    lf = local.load_factor()
    log(f"prefill done, load factor {lf:.4f}")
    steps, warm = args.steps, args.warmup
    n_e2e = min(steps, 20)  # the e2e steps get batches of their own, after the timed ones
    finds, inserts, vals = prepare_batches(steps + warm + n_e2e, rank, world, total, device,
                                           1234, cap)
    log("batches ready")
    out_vals = torch.empty((BATCH, DIM), device=device)
    founds = [torch.zeros(BATCH, dtype=torch.bool, device=device) for _ in range(steps + warm)]
    stream = torch.cuda.current_stream()

    def step(i, ev=None):
        if ev is not None:
            ev[0].record(stream)
        table.find(BATCH, finds[i], out_vals, founds[i])
        if ev is not None:
            ev[1].record(stream)
        table.insert_or_assign(BATCH, inserts[i], vals[i], unique_key=True)
        if ev is not None:
            ev[2].record(stream)

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    log("warmup done")
    if args.timeline:
        kernel_timeline(lambda i: table.find(BATCH, finds[warm + i], out_vals,
                                             founds[warm + i]),
                        steps, dist, rank, world, "config 2 find")
        kernel_timeline(lambda i: table.insert_or_assign(BATCH, inserts[warm + i],
                                                         vals[warm + i], unique_key=True),
                        steps, dist, rank, world, "config 2 insert_or_assign")
        if world > 1:
            table.close()
        del table, local, finds, inserts, vals, founds, out_vals
        torch.cuda.empty_cache()
        if not args.no_config5:
            config5_leg(rank, world, dist, device, timeline=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if dist:
        dist.barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.05)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches0 = H.kernel_launches()
    t0.record(stream)
    for i in range(steps):
        step(warm + i, evs[i])
    t1.record(stream)
    torch.cuda.synchronize()
    launches = H.kernel_launches() - launches0
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1)
    log(f"timed {steps} steps: {ms:.3f} ms")
    find_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    ins_ms = sum(e[1].elapsed_time(e[2]) for e in evs)
    hit = float(torch.stack(founds[warm:]).float().mean().item())
    if dist:
        tt = torch.tensor([ms, find_ms, ins_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, find_ms, ins_ms = [float(x) for x in tt.tolist()]
        tl = torch.tensor([launches], dtype=torch.int64, device=device)
        dist.all_reduce(tl)  # launches of all ranks
        launches = int(tl.item())
    e2e_line = e2e(table, finds, inserts, vals, warm + steps, n_e2e, dist, device)
    log("e2e done")
    local.check_device_error()  # a lock or peer wait that ran out fails the run
    # the headline table goes before config 5's leg (its shard takes ~70 GB)
    if world > 1:
        table.close()
    del table, local, finds, inserts, vals, founds, out_vals
    torch.cuda.empty_cache()
    cfg5 = None
    if not args.no_config5:
        cfg5 = config5_leg(rank, world, dist, device)
        log("config 5 leg done")
    keys_total = 2 * BATCH * steps * world
    value = keys_total / (ms * 1e-3) / 1e9

    result = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": round(ms / steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u64 keys / f32 values", "data": "synthetic (seeded device keys)",
        "config": {"workload": "BASELINE config 2 at load factor 1.0: find 1 Mi keys "
                               "(100% hits) + insert_or_assign 1 Mi keys (50% hits, "
                               "50% new keys evicting LRU) per step",
                   "capacity_per_gpu": cap, "dim": DIM, "batch": BATCH,
                   "strategy": "kLru", "load_factor": round(lf, 4),
                   "find_hit_rate": round(hit, 4),
                   "parallelism": "single table" if world == 1 else
                   f"sharded x{world} ({transport} transport)",
                   "l2": "table 9.2 GB/GPU >> 126 MB L2; every step uses its own input batches"},
    }
    if rank == 0:
        find_keys_s = BATCH * steps / (find_ms * 1e-3)
        ins_keys_s = BATCH * steps / (ins_ms * 1e-3)
        result["ops"] = {
            "find": {"bkvs": round(find_keys_s / 1e9, 4),
                     "bkvs_2^30": round(find_keys_s / 2 ** 30, 4),
                     "ms_per_call": round(find_ms / steps, 4)},
            "insert_or_assign": {"bkvs": round(ins_keys_s / 1e9, 4),
                                 "bkvs_2^30": round(ins_keys_s / 2 ** 30, 4),
                                 "ms_per_call": round(ins_ms / steps, 4)}}
        peak, kind = peaks()
        rf = {}
        for name, per_key, t_ms in (("find", FIND_HIT_BYTES, find_ms),
                                    ("insert_or_assign", INSERT_MIX_BYTES, ins_ms)):
            ach = per_key * BATCH / (t_ms / steps * 1e-3) / 1e9
            rf[name] = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                        "unit": "GB/s", "frac": round(ach / peak, 4),
                        "algorithmic_bytes_per_key": per_key, "peak_kind": kind}
        dom = "insert_or_assign" if ins_ms >= find_ms else "find"
        roof = dict(rf[dom])
        roof["kernel"] = dom
        roof["traffic"] = traffic_from_profiles(dom)
        result["roofline"] = roof
        result["roofline_by_op"] = rf
        result["clocks"] = clocks
        result["gpu_launches"] = launches
        result["e2e"] = e2e_line
        if cfg5 is not None:
            result["config5"] = cfg5
        if world == 1 and args.save_load:
            result["save_load"] = save_load_times(device)
            log("save/load done")
        if world == 1:
            if not args.no_cpu_baseline:
                result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
                log("cpu baseline done")
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def traffic_from_profiles(kernel):
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if not os.path.exists(p):
        return None
    d = json.load(open(p))
    v = d.get(kernel)
    return None if v is None else v.get("bytes_per_launch")


def e2e(table, finds, inserts, vals, first, steps, dist=None, device=None):
    """Same step through the public API with host buffers: every step copies
    its find keys, insert keys and insert values from pinned host memory,
    runs find + insert_or_assign, and copies the found values and flags back,
    all inside the timed region. Steps are pipelined the way a caller would
    drive the API: host-to-device copies on one stream, the table calls on a
    second, device-to-host copies on a third, with two buffer sets, so the
    copies of neighbouring steps overlap each other (both directions of the
    host link) and the kernels. On N ranks every rank runs it on its own
    batches; the time is the maximum over ranks and the value counts the keys
    of all ranks."""
    import torch

    world = dist.get_world_size() if dist else 1
    hk = [f.cpu().pin_memory() for f in finds[first:first + steps]]
    hi = [f.cpu().pin_memory() for f in inserts[first:first + steps]]
    hv = [v.cpu().pin_memory() for v in vals[first:first + steps]]
    out_h = [torch.empty((BATCH, DIM)).pin_memory() for _ in range(2)]
    fnd_h = [torch.empty(BATCH, dtype=torch.bool).pin_memory() for _ in range(2)]
    bufs = [dict(k=torch.empty(BATCH, dtype=torch.int64, device="cuda"),
                 i=torch.empty(BATCH, dtype=torch.int64, device="cuda"),
                 v=torch.empty((BATCH, DIM), device="cuda"),
                 o=torch.empty((BATCH, DIM), device="cuda"),
                 f=torch.empty(BATCH, dtype=torch.bool, device="cuda")) for _ in range(2)]
    s_in, s_run, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()  # noqa: E731
    loaded = [ev(), ev()]
    ran = [ev(), ev()]
    drained = [ev(), ev()]
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()  # the ranks start the timed region together
        torch.cuda.synchronize()
    a.record(s_in)
    for i in range(steps):
        x = i % 2
        B = bufs[x]
        if i >= 2:
            s_in.wait_event(ran[x])      # the table calls of step i-2 read B
        with torch.cuda.stream(s_in):
            B["k"].copy_(hk[i], non_blocking=True)
            B["i"].copy_(hi[i], non_blocking=True)
            B["v"].copy_(hv[i], non_blocking=True)
        loaded[x].record(s_in)
        s_run.wait_event(loaded[x])
        if i >= 2:
            s_run.wait_event(drained[x])  # step i-2's outputs have left B
        table.find(BATCH, B["k"], B["o"], B["f"], stream=s_run.cuda_stream)
        table.insert_or_assign(BATCH, B["i"], B["v"], stream=s_run.cuda_stream,
                               unique_key=True)
        ran[x].record(s_run)
        s_out.wait_event(ran[x])
        with torch.cuda.stream(s_out):
            out_h[x].copy_(B["o"], non_blocking=True)
            fnd_h[x].copy_(B["f"], non_blocking=True)
        drained[x].record(s_out)
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_run)
    b.record(s_out)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    if dist:
        tt = torch.tensor([ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    h2d = BATCH * 8 * 2 + BATCH * VALUE_BYTES
    d2h = BATCH * VALUE_BYTES + BATCH
    peak = pinned_copy_peaks()
    up = h2d * steps / (ms * 1e-3) / 1e9
    down = d2h * steps / (ms * 1e-3) / 1e9
    return {"value": round(2 * BATCH * steps * world / (ms * 1e-3) / 1e9, 4), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "pipelined": "H2D / table calls / D2H on three streams, two buffer sets",
            # the step's copies against the host link's measured peak (both
            # directions at once, as the pipeline runs them)
            "host_link": {"h2d_gbs": round(up, 1), "d2h_gbs": round(down, 1),
                          "peak_h2d_gbs": peak["h2d_duplex"], "peak_d2h_gbs": peak["d2h_duplex"],
                          "frac": round(max(up / peak["h2d_duplex"], down / peak["d2h_duplex"]), 4),
                          "peak_kind": "measured pinned cudaMemcpyAsync, 256 MiB each way "
                                       "concurrently on two streams"}}


def pinned_copy_peaks(nbytes=256 << 20, reps=3):
    """Pinned host <-> device cudaMemcpyAsync bandwidth on this GPU (best of
    `reps`): each direction alone, and both at once on two streams."""
    import torch

    hb = [torch.empty(nbytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    db = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    out = {"h2d": 0.0, "d2h": 0.0, "h2d_duplex": 0.0, "d2h_duplex": 0.0}
    for _ in range(reps):
        for name, dst, src in (("h2d", db[0], hb[0]), ("d2h", hb[1], db[1])):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record()
            dst.copy_(src, non_blocking=True)
            b.record()
            torch.cuda.synchronize()
            out[name] = max(out[name], nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize()
        ev[0].record(s1)
        ev[2].record(s2)
        with torch.cuda.stream(s1):
            db[0].copy_(hb[0], non_blocking=True)
        with torch.cuda.stream(s2):
            hb[1].copy_(db[1], non_blocking=True)
        ev[1].record(s1)
        ev[3].record(s2)
        torch.cuda.synchronize()
        out["h2d_duplex"] = max(out["h2d_duplex"],
                                nbytes / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9)
        out["d2h_duplex"] = max(out["d2h_duplex"],
                                nbytes / (ev[2].elapsed_time(ev[3]) * 1e-3) / 1e9)
    return {k: round(v, 1) for k, v in out.items()}


def save_load_times(device, capacity=8 << 20):
    """save() and load() of a full table through the LocalKVFile format (three
    raw files in a temporary directory), host wall time around each call
    (both synchronise)."""
    import shutil
    import tempfile

    import torch

    import hkv_b200 as H

    opts = H.HashTableOptions(init_capacity=capacity, max_capacity=capacity,
                              max_hbm_for_vectors=capacity * VALUE_BYTES * 2, dim=DIM,
                              max_load_factor=1.0)
    src = H.HashTable(H.EvictStrategy.kLru)
    src.init(opts)
    vals = torch.rand((4 << 20, DIM), device=device)
    for start in range(0, capacity, 4 << 20):
        src.insert_or_assign(4 << 20, keys_from_counters(start, 4 << 20, device), vals)
    torch.cuda.synchronize()
    n_live = src.size()
    d = tempfile.mkdtemp(prefix="hkv_save_")
    try:
        paths = [os.path.join(d, x) for x in ("keys", "values", "scores")]
        t0 = time.perf_counter()
        n_saved = src.save(*paths, max_workspace_size=64 << 20)
        t_save = time.perf_counter() - t0
        dst = H.HashTable(H.EvictStrategy.kLru)
        dst.init(opts)
        t0 = time.perf_counter()
        n_loaded = dst.load(*paths, max_workspace_size=64 << 20)
        t_load = time.perf_counter() - t0
        ok = n_saved == n_loaded == n_live == dst.size()
    finally:
        shutil.rmtree(d, ignore_errors=True)
    tb = 16 + VALUE_BYTES
    return {"tuples": n_saved, "tuple_bytes": tb, "workspace_bytes": 64 << 20,
            "save_s": round(t_save, 3), "load_s": round(t_load, 3),
            "save_gbs": round(n_saved * tb / t_save / 1e9, 3),
            "load_gbs": round(n_loaded * tb / t_load / 1e9, 3), "counts_match": ok}


# --------------------------------------------------------------------------
# --suite: every table operation on the config-2 table (one GPU, load factor
# 1.0), each timed with CUDA events over its own inputs and set against its
# algorithmic bytes per key (per slot for export_batch and reserve; dim 32,
# 128-byte rows). Not the headline metric; run on request.
# --------------------------------------------------------------------------
SUITE_BYTES = {
    "find_hit": 401,            # key 8, digest line 128, key 8, row 128 in + out, found 1
    "find_miss": 141,           # key 8, digest line 128, found 1, ~0.5 false digest hits
    "contains_hit": 145,        # key 8, digest line 128, key 8, found 1
    "insert_or_assign": 928.5,  # 50 % hits (416), 50 % evicting misses (1441)
    "find_or_insert": 928.5,    # same mix; hits copy the row out, misses in
    "insert_and_evict": 1064.5,  # evicting misses also write the victim out (+272)
    "accum_or_assign": 537,     # hits: key, flag, digest line, key, delta + row in, row out, score
    "assign_scores": 152,       # hits: key, digest line, key, score out
    "erase": 165,               # hits: key, digest line, key, key + score + digest + size out
    "export_batch": 288,        # per live slot: key, row, score in; key, row, score out
    "reserve": 290,             # per old slot: key, score, digest, row read once and written once
}


def run_suite(args):
    import torch

    import hkv_b200 as H

    dev = torch.device("cuda", 0)
    cap = args.capacity
    steps, warm = args.steps, args.warmup
    table, local = build_table(1, 0, None, cap)
    total = prefill(local, 0, 1, dev, cap)
    nb = steps + warm
    finds, inserts, vals = prepare_batches(4 * nb, 0, 1, total, dev, 11, cap)
    n = BATCH
    misses = [keys_from_counters((1 << 40) + i * BATCH, BATCH, dev) for i in range(nb)]
    out = torch.empty((n, DIM), device=dev)
    founds = torch.zeros(n, dtype=torch.bool, device=dev)
    ev_keys = torch.empty(n, dtype=torch.int64, device=dev)
    ev_vals = torch.empty((n, DIM), device=dev)
    ev_scores = torch.empty(n, dtype=torch.int64, device=dev)
    counter = torch.zeros(1, dtype=torch.int64, device=dev)
    flags = torch.ones(n, dtype=torch.bool, device=dev)
    ins_i = [0]

    def next_insert():
        i = ins_i[0]
        ins_i[0] += 1
        return inserts[i], vals[i]

    ops = {
        "find_hit": lambda i: table.find(n, finds[i], out, founds),
        "find_miss": lambda i: table.find(n, misses[i], out, founds),
        "contains_hit": lambda i: table.contains(n, finds[i], founds),
        "insert_or_assign": lambda i: table.insert_or_assign(n, *next_insert(), unique_key=True),
        "find_or_insert": lambda i: table.find_or_insert(n, *next_insert(), unique_key=True),
        "insert_and_evict": lambda i: (counter.zero_(), table.insert_and_evict(
            n, *next_insert(), None, ev_keys, ev_vals, ev_scores, counter, unique_key=True)),
        "accum_or_assign": lambda i: table.accum_or_assign(n, finds[i], vals[i], flags),
        "assign_scores": lambda i: table.assign_scores(n, finds[i]),
    }
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    peak, peak_kind = peaks()
    rows = []

    def record(name, ms, units, launches):
        b = SUITE_BYTES[name]
        gbs = units * b / (ms * 1e-3) / 1e9
        rows.append({"op": name, "ms_per_call": round(ms, 4),
                     "bkvs": round(units / (ms * 1e-3) / 1e9, 4), "bytes_per_unit": b,
                     "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                     "gpu_launches_per_call": launches})
        log(f"{name:18s} {ms * 1000:9.1f} us  {rows[-1]['bkvs']:7.3f} B/s  {gbs:7.0f} GB/s")

    for name, fn in ops.items():
        for i in range(warm):
            fn(i)
        torch.cuda.synchronize()
        l0 = H.kernel_launches()
        ev0.record()
        for i in range(warm, nb):
            fn(i)
        ev1.record()
        torch.cuda.synchronize()
        record(name, ev0.elapsed_time(ev1) / steps, n, (H.kernel_launches() - l0) / steps)
    # erase resident keys, then put them back (untimed) so the table stays full
    times = []
    for i in range(nb):
        k = finds[i]
        torch.cuda.synchronize()
        ev0.record()
        table.erase(n, k)
        ev1.record()
        torch.cuda.synchronize()
        if i >= warm:
            times.append(ev0.elapsed_time(ev1))
        table.insert_or_assign(n, k, vals[i], unique_key=True)
    record("erase", statistics.median(times), n, 1)
    # export the whole table in 8 Mi-slot pieces
    piece = min(8 << 20, cap)
    ek = torch.empty(piece, dtype=torch.int64, device=dev)
    evv = torch.empty((piece, DIM), device=dev)
    es = torch.empty(piece, dtype=torch.int64, device=dev)
    live = table.size()
    torch.cuda.synchronize()
    ev0.record()
    for off in range(0, cap, piece):
        table.export_batch(piece, off, ek, evv, es, d_counter=counter)
    ev1.record()
    torch.cuda.synchronize()
    record("export_batch", ev0.elapsed_time(ev1), live, cap // piece)
    table.check_device_error()
    # reserve: a growable table (max = 2 x capacity) at load factor 0.75
    # doubles once (rehash of every slot)
    del table, local
    grow = H.HashTable(H.EvictStrategy.kLru)
    grow.init(H.HashTableOptions(init_capacity=cap, max_capacity=2 * cap,
                                 max_hbm_for_vectors=2 * cap * VALUE_BYTES, dim=DIM,
                                 max_load_factor=1.0))
    fill = cap * 3 // 4
    for st in range(0, fill, n):  # n-row value batches
        m = min(n, fill - st)
        grow.insert_or_assign(m, keys_from_counters((1 << 41) + st, m, dev), vals[0][:m])
    torch.cuda.synchronize()
    l0 = H.kernel_launches()
    ev0.record()
    grow.reserve(2 * cap)
    ev1.record()
    torch.cuda.synchronize()
    assert grow.capacity() == 2 * cap
    record("reserve", ev0.elapsed_time(ev1), cap, H.kernel_launches() - l0)
    grow.check_device_error()
    print(json.dumps({"suite": rows, "capacity": cap, "dim": DIM, "batch": n,
                      "strategy": "kLru", "load_factor_before": 1.0,
                      "steps": steps, "warmup": warm,
                      "peak_gbs": peak, "peak_kind": peak_kind}),
          flush=True)


# --------------------------------------------------------------------------
# --workload hybrid: value rows split between HBM and pinned host memory
# (BASELINE config 4 at reduced size: 64 Mi slots, dim 128, 1/16 of the value
# bytes in HBM as in 16 GB of 256 GB, load factor 0.75). find of resident
# keys, 80 % of them in HBM-resident buckets; insert_or_assign of uniform keys
# (half resident, half new). Host-resident rows cross the host link zero-copy.
# --------------------------------------------------------------------------
def run_hybrid(args):
    import ctypes

    import torch

    import hkv_b200 as H

    class View(ctypes.Structure):
        _fields_ = [("keys", ctypes.c_void_p), ("scores", ctypes.c_void_p),
                    ("digests", ctypes.c_void_p), ("sizes", ctypes.c_void_p),
                    ("slices", ctypes.c_void_p), ("capacity", ctypes.c_uint64),
                    ("num_buckets", ctypes.c_uint64), ("bucket_size", ctypes.c_uint32),
                    ("slice_shift", ctypes.c_uint32), ("value_bytes", ctypes.c_uint32),
                    ("dim", ctypes.c_uint32), ("reclaim_digest", ctypes.c_uint8)]

    dev = torch.device("cuda", 0)
    cap = args.capacity if args.capacity != CAPACITY else 64 << 20
    dim = 128
    vb = dim * 4
    hbm = cap * vb // 16
    n = BATCH
    steps, warm = args.steps, args.warmup
    t = H.HashTable(H.EvictStrategy.kLru)
    t0 = time.time()
    t.init(H.HashTableOptions(init_capacity=cap, max_capacity=cap, max_hbm_for_vectors=hbm,
                              dim=dim, max_load_factor=1.0))
    view = View()
    H._check(H.lib().hkv_table_get_view(ctypes.c_void_p(t._h), ctypes.byref(view)))
    per_slice = 1 << view.slice_shift
    hbm_buckets = min(view.num_buckets, (hbm // (per_slice * 128 * vb)) * per_slice)
    if hbm_buckets == 0 or hbm_buckets == view.num_buckets:
        raise SystemExit("hybrid: no value slice (or every slice) fits the HBM budget "
                         "at this capacity; choose another --capacity")
    log(f"hybrid table: {cap} slots, dim {dim}, {hbm_buckets}/{view.num_buckets} buckets' "
        f"rows in HBM, created in {time.time() - t0:.1f}s")
    fill = cap * 3 // 4
    rows = torch.randn((n, dim), device=dev)
    for st in range(0, fill, n):
        m = min(n, fill - st)
        t.insert_or_assign(m, keys_from_counters(st, m, dev), rows[:m])
    torch.cuda.synchronize()
    resident = keys_from_counters(0, fill, dev)
    bucket = (fmix_t(resident) & (cap - 1)) >> 7
    in_hbm = resident[bucket < hbm_buckets]
    in_host = resident[bucket >= hbm_buckets]
    del resident, bucket
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    nh = n * 4 // 5
    finds, inserts = [], []
    for i in range(steps + warm):
        k = torch.cat([in_hbm[torch.randint(0, in_hbm.numel(), (nh,), generator=g, device=dev)],
                       in_host[torch.randint(0, in_host.numel(), (n - nh,), generator=g,
                                             device=dev)]])
        finds.append(k[torch.randperm(n, generator=g, device=dev)])
        old = keys_from_counters(0, fill, dev)[torch.randperm(fill, generator=g, device=dev)[:n // 2]]
        new = keys_from_counters(fill + i * n, n // 2, dev)
        inserts.append(torch.cat([old, new])[torch.randperm(n, generator=g, device=dev)])
    out = torch.empty((n, dim), device=dev)
    founds = torch.zeros(n, dtype=torch.bool, device=dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    # the host link's own peak (pinned cudaMemcpyAsync each way): the
    # roofline denominator for rows in host memory
    link = pinned_copy_peaks()
    log(f"pinned copy peak: {link} GB/s")
    res = {}
    for name in ("find", "insert_or_assign"):
        def call(i):
            if name == "find":
                t.find(n, finds[i], out, founds)
            else:
                t.insert_or_assign(n, inserts[i], rows)
        for i in range(warm):
            call(i)
        torch.cuda.synchronize()
        e0.record()
        for i in range(warm, warm + steps):
            call(i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        # rows that cross the host link per call: found rows of host buckets
        # (find), inserted rows of host buckets (insert, 1 - 1/16 of uniform keys)
        host_frac = (n - nh) / n if name == "find" else 1 - hbm_buckets / view.num_buckets
        link_bytes = n * host_frac * vb
        gbs = link_bytes / (ms * 1e-3) / 1e9
        peak = link["h2d"] if name == "find" else link["d2h"]  # rows read / written
        res[name] = {"ms_per_call": round(ms, 4), "bkvs": round(n / (ms * 1e-3) / 1e9, 4),
                     "host_rows_fraction": round(host_frac, 4),
                     "host_link_bytes_per_call": int(link_bytes),
                     "host_link_gbs": round(gbs, 1),
                     "roofline": {"bound": "host link", "achieved": round(gbs, 1),
                                  "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                                  "peak_kind": "measured pinned cudaMemcpyAsync, " +
                                               ("host to device" if name == "find"
                                                else "device to host")}}
        log(f"hybrid {name}: {ms * 1000:.1f} us per call, {res[name]['host_link_gbs']} GB/s "
            f"over the host link")
    hit = float(founds.float().mean().item())
    t.check_device_error()
    print(json.dumps({"workload": "hybrid (BASELINE config 4 at 64 Mi slots)", "dim": dim,
                      "capacity": cap, "max_hbm_for_vectors": hbm,
                      "hbm_bucket_fraction": round(hbm_buckets / view.num_buckets, 4),
                      "load_factor": 0.75, "batch": n, "steps": steps, "warmup": warm,
                      "find_hit_rate_last_call": round(hit, 4), "pinned_copy_gbs": link,
                      "ops": res}), flush=True)


# --------------------------------------------------------------------------
# --workload zipf: find_or_insert of power-law (Zipf-like) keys with repeats
# (unique_key = false), dim 64: 128 Mi slots, kEpochLfu, 2 Mi keys per step on
# one GPU; 256 Mi slots per GPU, kLfu, 8 Mi keys per GPU per step when
# sharded. Not the headline metric; run on request.
# --------------------------------------------------------------------------
def zipf_ids(n, s, universe, gen, device):
    """Power-law ids on [0, universe): the inverse CDF of the continuous
    density x^-s on [1, universe] (a stand-in for Zipf(s))."""
    import torch

    u = torch.rand(n, generator=gen, device=device, dtype=torch.float64)
    a = 1.0 - s
    x = ((universe ** a - 1.0) * u + 1.0) ** (1.0 / a)
    return (x.floor().to(torch.int64) - 1).clamp_(0, universe - 1)


def config5_leg(rank, world, dist, device, steps=5, warm=2, timeline=False):
    """BASELINE config 5 on this run's GPUs: one table shard of 256 Mi slots
    per GPU (dim 64, kLfu, scores 1..16), prefilled with as many keys as
    slots; each step every GPU submits 8 Mi power-law keys (a seeded
    Zipf(1.1) stand-in over 2^30 ids, repeats merged: unique_key = false) to
    find_or_insert, routed to their owner GPUs; then every shard is dumped
    with export_batch. Times are device times (CUDA events, max over
    ranks)."""
    import torch

    import hkv_b200 as H

    cap, dim, batch, s_exp = 256 << 20, 64, 8 << 20, 1.1
    strat = H.EvictStrategy.kLfu
    opts = H.HashTableOptions(init_capacity=cap, max_capacity=cap,
                              max_hbm_for_vectors=cap * dim * 8, dim=dim, max_load_factor=1.0)
    if world == 1:
        table = local = H.HashTable(strat)
        table.init(opts)
    else:
        uid = [H.ShardedHashTable.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        opts.device_id = torch.cuda.current_device()
        table = H.ShardedHashTable(opts, rank, world, uid[0], strat, max_batch=batch)
        local = H.HashTable.borrow(H.lib().hkv_sharded_local(table._h), strat)
    gen = torch.Generator(device=device)
    gen.manual_seed(5150 + rank)
    chunk = 4 << 20
    pv = torch.randn((chunk, dim), device=device)
    for st in range(0, cap * world, chunk):  # each shard keeps the keys it owns
        k = keys_from_counters((1 << 44) + st, chunk, device)
        if world > 1:
            k = k[owner_t(k, world) == rank]
        sc = torch.randint(1, 17, (k.numel(),), generator=gen, device=device)
        local.insert_or_assign(k.numel(), k, pv[:k.numel()], sc)
    del pv
    torch.cuda.synchronize()
    lf = local.load_factor()
    nb = 3  # batches cycled through the steps
    batches = []
    for _ in range(nb):
        k = key_of(zipf_ids(batch, s_exp, 1 << 30, gen, device))
        batches.append((k, torch.randn((batch, dim), generator=gen, device=device),
                        torch.randint(1, 17, (batch,), generator=gen, device=device)))
    uniq = sum(int(torch.unique(b[0]).numel()) for b in batches) / (nb * batch)
    stream = torch.cuda.current_stream()

    def step(i):
        k, v, sc = batches[i % nb]
        table.find_or_insert(batch, k, v, sc, unique_key=False)

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    if timeline:
        kernel_timeline(lambda i: step(warm + i), steps, dist, rank, world,
                        "config 5 find_or_insert")
        if world > 1:
            table.close()
        return None
    if dist:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        step(warm + i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    local.check_device_error()
    del batches
    # dump every shard: export_batch over all of its slots in 16 Mi pieces
    piece = 16 << 20
    ek = torch.empty(piece, dtype=torch.int64, device=device)
    ev = torch.empty((piece, dim), device=device)
    es = torch.empty(piece, dtype=torch.int64, device=device)
    cnt = torch.zeros(1, dtype=torch.int64, device=device)
    live = local.size()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0.record(stream)
    for off in range(0, cap, piece):
        local.export_batch(piece, off, ek, ev, es, d_counter=cnt)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    tt = torch.tensor([ms, ems], device=device)
    lt = torch.tensor([live], dtype=torch.int64, device=device)
    if dist:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dist.all_reduce(lt)
    ms, ems = (float(x) for x in tt.tolist())
    if world > 1:
        table.close()
    del table, local, ek, ev, es
    torch.cuda.empty_cache()
    keys = batch * steps * world
    # per GPU and step, the same merged-batch model as --workload zipf: merge
    # reads of keys and scores, each distinct key's find or insert (hit
    # model, 160 + 2 Vb), one output row per later occurrence; the NVLink
    # bytes of N > 1 are not counted
    peak, peak_kind = peaks()
    vb = dim * 4
    step_bytes = 16 * batch + uniq * batch * (160 + 2 * vb) + (1 - uniq) * batch * vb
    ach = step_bytes / (ms / steps * 1e-3) / 1e9
    return {"workload": "BASELINE config 5: 256 Mi slots per GPU, dim 64, kLfu (scores "
                        "1..16), 8 Mi keys per GPU per step (seeded Zipf(1.1) stand-in over "
                        "2^30 ids, repeats merged), find_or_insert routed to the owner "
                        "shard; then export_batch of every shard",
            "n_gpus": world, "load_factor_before": round(lf, 4),
            "distinct_fraction": round(uniq, 4), "steps": steps, "warmup": warm,
            "batches_cycled": nb,
            "find_or_insert_bkvs": round(keys / (ms * 1e-3) / 1e9, 4),
            "find_or_insert_bkvs_per_gpu": round(keys / world / (ms * 1e-3) / 1e9, 4),
            "ms_per_step": round(ms / steps, 4),
            "export_ms": round(ems, 3), "exported_keys": int(lt.item()),
            "export_slots_per_ns": round(cap * world / (ems * 1e-3) / 1e9, 3),
            "roofline_per_gpu": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                                 "unit": "GB/s", "frac": round(ach / peak, 4),
                                 "algorithmic_bytes_per_step": int(step_bytes),
                                 "peak_kind": peak_kind}}


def run_zipf(args):
    import torch

    import hkv_b200 as H

    rank, world, local_rank, dist = dist_setup(args.gpus)
    device = torch.device("cuda", torch.cuda.current_device())
    if world == 1:
        cap, dim, batch, s_exp, strat = 128 << 20, 64, 2 << 20, 1.05, H.EvictStrategy.kEpochLfu
    else:  # one shard per GPU
        cap, dim, batch, s_exp, strat = 256 << 20, 64, 8 << 20, 1.1, H.EvictStrategy.kLfu
    cap = min(cap, args.capacity) if args.capacity != CAPACITY else cap
    opts = H.HashTableOptions(init_capacity=cap, max_capacity=cap,
                              max_hbm_for_vectors=cap * dim * 8, dim=dim, max_load_factor=1.0)
    if world == 1:
        table = H.HashTable(strat)
        table.init(opts)
        local = table
    else:
        uid = [H.ShardedHashTable.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        opts.device_id = torch.cuda.current_device()
        table = H.ShardedHashTable(opts, rank, world, uid[0], strat, max_batch=batch)
        local = H.HashTable.borrow(H.lib().hkv_sharded_local(table._h), strat)
    epoch = 1
    if strat == H.EvictStrategy.kEpochLfu:
        local.set_global_epoch(epoch)
    gen = torch.Generator(device=device)
    gen.manual_seed(99 + rank)
    # prefill: capacity distinct keys (each rank its own part of the stream)
    chunk = 4 << 20
    pv = torch.randn((chunk, dim), device=device)
    for st in range(0, cap * world, chunk):
        k = keys_from_counters(st, chunk, device)
        if world > 1:
            k = k[owner_t(k, world) == rank]
        sc = torch.randint(1, 17, (k.numel(),), generator=gen, device=device)
        local.insert_or_assign(k.numel(), k, pv[:k.numel()], sc)
    torch.cuda.synchronize()
    log(f"zipf prefill done, load factor {local.load_factor():.3f}")
    steps, warm = args.steps, args.warmup
    nb = min(steps + warm, 8)
    batches = []
    for b in range(nb):
        ids = zipf_ids(batch, s_exp, 1 << 30, gen, device)
        k = key_of(ids)
        batches.append((k, torch.randn((batch, dim), generator=gen, device=device),
                        torch.randint(1, 17, (batch,), generator=gen, device=device)))
    uniq = sum(int(torch.unique(b[0]).numel()) for b in batches) / (nb * batch)
    peak, peak_kind = peaks()
    vb = dim * 4

    def merged_roofline(ms_step, per_step_bytes):
        ach = per_step_bytes / (ms_step * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                "frac": round(ach / peak, 4), "algorithmic_bytes_per_step": int(per_step_bytes),
                "peak_kind": peak_kind}

    def step(i):
        # values are in/out: a found key's row overwrites its input row, a
        # missing key is inserted with whatever its row holds
        nonlocal epoch
        k, v, sc = batches[i % nb]
        table.find_or_insert(batch, k, v, sc, unique_key=False)
        if strat == H.EvictStrategy.kEpochLfu and (i + 1) % 10 == 0:
            epoch += 1
            local.set_global_epoch(epoch)

    for i in range(warm):
        step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    stream = torch.cuda.current_stream()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record(stream)
    for i in range(steps):
        step(warm + i)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if dist:
        tt = torch.tensor([ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    local.check_device_error()
    ie = None
    if world == 1:
        # BASELINE config 3's second leg: insert_and_evict of the same batches
        # (repeats merged), the epoch still advancing every 10 steps, the
        # evicted and refused tuples collected each step
        ek = torch.empty(batch, dtype=torch.int64, device=device)
        ev = torch.empty((batch, dim), device=device)
        es = torch.empty(batch, dtype=torch.int64, device=device)
        cnt = torch.zeros(1, dtype=torch.int64, device=device)
        outs = []
        # fresh batches from the same power law: the hot keys are resident,
        # the tail brings keys that must evict (or be refused)
        for b in range(nb):
            ids = zipf_ids(batch, s_exp, 1 << 30, gen, device)
            batches[b] = (key_of(ids), torch.randn((batch, dim), generator=gen, device=device),
                          torch.randint(1, 17, (batch,), generator=gen, device=device))

        def evict_step(i):
            nonlocal epoch
            k, v, sc = batches[i % nb]
            cnt.zero_()
            table.insert_and_evict(batch, k, v, sc, ek, ev, es, cnt, unique_key=False)
            if strat == H.EvictStrategy.kEpochLfu and (i + 1) % 10 == 0:
                epoch += 1
                local.set_global_epoch(epoch)

        for i in range(warm):
            evict_step(i)
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(steps):
            evict_step(warm + i)
            outs.append(cnt.clone())
        t1.record(stream)
        torch.cuda.synchronize()
        ie_ms = t0.elapsed_time(t1)
        # the last step: every input key is in the table or among its outputs
        k = batches[(warm + steps - 1) % nb][0]
        found = torch.zeros(batch, dtype=torch.bool, device=device)
        table.contains(batch, k, found)
        c = int(outs[-1].item())
        reported = torch.isin(k, ek[:c])
        ok = bool((found | reported).all().item())
        local.check_device_error()
        outs_step = sum(int(o.item()) for o in outs) / steps
        u_ie = sum(int(torch.unique(b[0]).numel()) for b in batches) / nb
        # merge reads of keys and scores, each distinct key's upsert (hit
        # model, 160 + 2 Vb), and per reported tuple the eviction's score scan
        # (1025 more) and the output key, score and row
        ie_bytes = 16 * batch + u_ie * (160 + 2 * vb) + outs_step * (1025 + 16 + vb)
        ie = {"bkvs": round(batch * steps / (ie_ms * 1e-3) / 1e9, 4),
              "ms_per_step": round(ie_ms / steps, 4),
              "outputs_per_step": round(outs_step, 1),
              "distinct_fraction": round(u_ie / batch, 4),
              "every_input_present_or_reported": ok,
              "roofline": merged_roofline(ie_ms / steps, ie_bytes)}
        log(f"insert_and_evict leg: {ie}")
    if rank == 0:
        print(json.dumps({
            "metric": "B-KV/s for find_or_insert of Zipf keys with repeats (unique_key=false)",
            "value": round(batch * steps * world / (ms * 1e-3) / 1e9, 4), "unit": UNIT,
            "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 keys / f32 values",
            "data": "synthetic (power-law ids, seeded)",
            "config": {"workload": ("BASELINE config 3: 128 Mi slots, dim 64, kEpochLfu, "
                                    "2 Mi keys per step, Zipf(1.05) stand-in")
                       if world == 1 else
                       ("BASELINE config 5: 256 Mi slots per GPU, dim 64, kLfu, 8 Mi keys "
                        "per GPU per step, Zipf(1.1) stand-in, sharded peer transport"),
                       "capacity_per_gpu": cap, "dim": dim, "batch_per_gpu": batch,
                       "distinct_fraction": round(uniq, 4),
                       "batches_cycled": nb},
            # merge reads of keys and scores, each distinct key's find or
            # insert (hit model, 160 + 2 Vb), one output row per later
            # occurrence
            "roofline": merged_roofline(
                ms / steps, 16 * batch + uniq * batch * (160 + 2 * vb)
                + (1 - uniq) * batch * vb),
            "insert_and_evict": ie}), flush=True)
    if world > 1:
        table.close()
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------
# CPU arm: the reference's algorithm (oracle/ restatement) on host threads.
# --------------------------------------------------------------------------
def cpu_run(capacity, steps, warm, threads, min_seconds=0.0, max_steps=None):
    """The step of the GPU bench on the CPU oracle: prefill to LF 1.0, then
    per step a find of 1 Mi resident keys and an insert_or_assign of 1 Mi keys
    (half resident, half new). Each step's batch is drawn just before it; only
    the two calls are timed. Runs `steps` steps, or more (up to `max_steps`)
    until `min_seconds` of timed work have accumulated."""
    import numpy as np

    import hkv_oracle as O

    rng = np.random.default_rng(77)
    t = O.OracleTable(capacity, capacity, dim=DIM, strategy=O.LRU,
                      max_load_factor=1.0, threads=threads)
    total = int(capacity * PREFILL_FACTOR)
    chunk = 1 << 22
    clock = 1

    def fmix(x):
        x = np.asarray(x, np.uint64).copy()
        with np.errstate(over="ignore"):
            x ^= x >> np.uint64(33)
            x *= np.uint64(0xFF51AFD7ED558CCD)
            x ^= x >> np.uint64(33)
            x *= np.uint64(0xC4CEB9FE1A85EC53)
            x ^= x >> np.uint64(33)
        return x

    vals = rng.random((chunk, DIM)).astype(np.float32)
    for s in range(0, total, chunk):
        k = fmix(np.arange(s, min(s + chunk, total), dtype=np.uint64))
        t.set_clock(clock)
        clock += 1
        t.insert_or_assign(k, vals[:len(k)])
    hot = fmix(np.arange(max(0, total - min(HOT, capacity // 4)), total, dtype=np.uint64))
    out = np.empty((BATCH, DIM), np.float32)
    max_steps = max_steps or steps
    dt, done, s = 0.0, 0, 0
    while s < warm + max_steps and (done < steps or dt < min_seconds):
        f = hot[rng.integers(0, len(hot), BATCH)]
        fresh = fmix(np.arange(total + s * BATCH // 2, total + (s + 1) * BATCH // 2,
                               dtype=np.uint64))
        ins = np.concatenate([rng.choice(hot, BATCH // 2, replace=False), fresh])
        v = rng.random((BATCH, DIM)).astype(np.float32)
        t.set_clock(clock)
        clock += 1
        t0 = time.perf_counter()
        t.find(f, values=out)
        t.insert_or_assign(ins, v)
        if s >= warm:
            dt += time.perf_counter() - t0
            done += 1
        s += 1
    return 2 * BATCH * done / dt / 1e9, dt, t.load_factor(), done


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(seconds_hint):
    cap = 8 << 20
    threads = cpu_threads()
    v, dt, lf, done = cpu_run(cap, 3, 1, threads, min_seconds=seconds_hint, max_steps=400)
    return {"value": round(v, 5), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"oracle/ restatement, {cap >> 20} Mi slots (1/8 of the GPU table), "
                      f"dim 32, kLru, LF {lf:.3f}, {done} steps x (1 Mi find + 1 Mi "
                      f"insert_or_assign), {dt:.2f} s timed"}


def run_reference(args):
    """`--impl reference`: the reference's CPU algorithm on all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    mem_gb = 0
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable"):
                mem_gb = int(line.split()[1]) / (1 << 20)
    except OSError:
        pass
    cap = CAPACITY if mem_gb > 64 else 8 << 20
    steps = max(1, min(args.steps, 40))
    v, dt, lf, steps = cpu_run(cap, steps, min(args.warmup, 1), threads)
    out = {"metric": METRIC, "value": round(v, 5), "unit": UNIT, "impl": "reference",
           "n_gpus": args.gpus, "steps": steps, "warmup": min(args.warmup, 1),
           "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "u64 keys / f32 values",
           "data": "synthetic (seeded)",
           "config": {"workload": "BASELINE config 2 at load factor 1.0 (find 1 Mi hits "
                                  "+ insert_or_assign 1 Mi 50/50 per step)",
                      "capacity": cap, "dim": DIM, "strategy": "kLru",
                      "load_factor": round(lf, 4)},
           "cpu_baseline": {"value": round(v, 5), "unit": UNIT, "cores": threads,
                            "kind": "port",
                            "sample": f"oracle/ CPU restatement (the reference needs an "
                                      f"Ascend NPU + CANN), {cap >> 20} Mi slots, "
                                      f"{steps} steps, {dt:.2f} s"},
           "e2e": {"value": round(v, 5), "unit": UNIT, "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config5", action="store_true",
                    help="skip BASELINE config 5's leg (sharded find_or_insert of "
                         "power-law keys, then a dump of every shard)")
    ap.add_argument("--save-load", action="store_true",
                    help="also time save/load (LocalKVFile files in a temporary "
                         "directory) of an 8 Mi-slot table; adds a save_load key")
    ap.add_argument("--timeline", action="store_true",
                    help="diagnostics, not the bench line: per-kernel device times of "
                         "the headline's find and insert_or_assign calls and of config "
                         "5's find_or_insert (torch profiler), one JSON line per rank "
                         "and leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--capacity", type=int, default=CAPACITY,
                    help="slots per GPU (diagnostics; the metric uses the default)")
    ap.add_argument("--suite", action="store_true",
                    help="time every table operation on one GPU (not the headline)")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "zipf", "hybrid"],
                    help="cfg2: the headline metric; zipf: find_or_insert of "
                         "power-law keys with repeats (dim 64); hybrid: values split "
                         "between HBM and pinned host memory (dim 128)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "zipf":
        run_zipf(args)
        return
    if args.workload == "hybrid":
        run_hybrid(args)
        return
    if args.suite:
        run_suite(args)
        return
    run_gpu(args)


if __name__ == "__main__":
    main()
