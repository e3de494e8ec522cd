"""Benchmark of the Cascade block data path on B200.

Default workload (N=1): 65,536 Qwen2.5-7B-shaped KV blocks (917,504 B, fp16
N(0,1) from a seeded generator), 25 % of them byte-identical copies of 64
prefix blocks; one step = clear the store, batch_put every block in batches
of 1024 (GPU SHA-256 + dedup + scatter into the HBM slab pool), then
batch_get every stored block in a uniformly shuffled order (gather). Inputs
(60 GB) are resident in HBM before the timed region and are far larger than
L2, so no L2 flush is needed.

value  = (bytes put + bytes got) / step time  [GB/s, 1e9]
e2e    = same metric through the public API with pinned HOST buffers
         (host->device copies of the blocks and device->host copies of the
         results inside the timed region), on a bounded slice.
--impl reference: the reference's own CPU path (compute_block_id with
OpenMP + CascadeStore::put_batch/get_batch on its SHM tier), compiled from
its sources into oracle/_ref, on a bounded slice of the same workload.

With torchrun (N>1) every rank runs the same workload on its own GPU and
store (independent replicas, weak scaling); rank 0 prints max-over-ranks
timing.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "kcj-cascade-v6_b200"))
sys.path.insert(0, ROOT)

METRIC = "aggregate batch_put (incl. SHA256) + batch_get GB/s"
GB = 1e9
SHA_TRAFFIC_PER_1024_LAUNCH = 740_662_528  # bytes, ncu capture of one sha256_fused_kernel launch (roofline note)
SHA_ALU_INSTR_PER_CHUNK = 64 * 10 + 48 * 8 + 16  # integer-ALU lane-instructions per 64-byte chunk
NVLINK_PEER_GBS = 770.0  # measured peer copy per direction per GPU on this pool (nominal 900)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--blocks", type=int, default=65536)
    p.add_argument("--batch", type=int, default=1024)
    p.add_argument("--block-bytes", type=int, default=917504)
    p.add_argument("--e2e-blocks", type=int, default=4096)
    p.add_argument("--cpu-blocks", type=int, default=1024)
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="cpu_baseline: repeat passes over the sample until this much put + get time is timed")
    p.add_argument("--copy-engine", type=int, default=0)
    p.add_argument("--layout", choices=["shuffled", "stream"], default="shuffled",
                   help="where the caller's distinct blocks sit in its buffer: shuffled (the default, like the CPU "
                        "reference arm) or in the order of their first occurrence in the put stream")
    p.add_argument("--hash-sms", type=int, default=0,
                   help="SMs the pipelined puts' SHA-256 may occupy (0 = the library default: all on one GPU, "
                        "all but 8 on a DHT member)")
    p.add_argument("--no-profile", action="store_true",
                   help="no per-launch CUDA events in the store (roofline fields then come out empty)")
    p.add_argument("--pipeline-blocks", type=int, default=0,
                   help="pipelined puts: blocks hashing at once (0 = the library default, 65536)")
    p.add_argument("--hash-lanes", type=int, default=32, help="reserved; the SHA-256 kernel runs 32 chains per warp")
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--workload", default="config2", choices=["config2", "zipf", "spill", "sweep"])
    p.add_argument("--sweep-sizes", default="4096,65536,1048576,4194304,16777216")
    p.add_argument("--sweep-gib", type=float, default=16.0)
    p.add_argument("--spill-blocks", type=int, default=40000)
    p.add_argument("--spill-hbm-gb", type=float, default=120.0)
    p.add_argument("--spill-dram-gb", type=float, default=100.0)
    p.add_argument("--collective-timeout-ms", type=int, default=300000,
                   help="N>1: a DHT collective that does not finish in time fails instead of waiting")
    p.add_argument("--trace", action="store_true", help="print per-rank phase markers to stderr")
    p.add_argument("--kv-compression", action="store_true",
                   help="spill: DRAM-tier blocks in the INT8 KVCompressor format (lossy)")
    p.add_argument("--zipf-blocks-per-gpu", type=int, default=20000)
    p.add_argument("--zipf-block-bytes", type=int, default=5242880)
    p.add_argument("--zipf-batch", type=int, default=512)
    p.add_argument("--zipf-alpha", type=float, default=1.1)
    return p.parse_args()


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while running."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits", "-lms", "50"],
                                     stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7:
                try:
                    rows.append((float(parts[0]), float(parts[1]), parts[3:7]))
                except ValueError:
                    pass
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": rows[0][1],
                "sm_mhz_min": float(min(r[0] for r in rows)), "samples": len(rows), "reasons": reasons}


# --------------------------------------------------------------- workload

def workload(args, rank):
    from cascade_cpp import workloads as W
    src, is_prefix = W.dedup_mix(args.blocks, 64, 0.25, 2024 + rank)
    uniq = np.unique(src)
    return src, is_prefix, uniq


def gpu_blocks(args, rank, device):
    """Unique blocks generated on the GPU (seeded); per-position pointers."""
    import torch
    src, is_prefix, uniq = workload(args, rank)
    size = args.block_bytes
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    pool = torch.empty(len(uniq) * size, dtype=torch.uint8, device=device)
    chunk = 4096 * size // 2
    flat = pool.view(torch.float16)
    for o in range(0, flat.numel(), chunk):
        n = min(chunk, flat.numel() - o)
        flat[o:o + n] = torch.randn(n, generator=g, device=device, dtype=torch.float16)
    if getattr(args, "layout", "shuffled") == "stream":
        # distinct blocks stored in the order of their first occurrence in
        # the put stream (copies still point at their originals)
        _, first = np.unique(src, return_index=True)
        slot = np.empty(len(uniq), np.int64)
        slot[np.argsort(first)] = np.arange(len(uniq))
        pos = slot[np.searchsorted(uniq, src)]
    else:  # the distinct blocks at shuffled places, like the CPU reference arm's buffer
        pos = np.searchsorted(uniq, src)
    ptrs = np.uint64(pool.data_ptr()) + pos.astype(np.uint64) * np.uint64(size)
    return pool, ptrs.astype(np.uint64), is_prefix.astype(np.uint8)


_TRACE = {"on": False}


def trace(args, msg):
    if _TRACE["on"] or (args is not None and args.trace):
        print(f"[rank {os.environ.get('RANK', '0')} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def make_store(args, device_index, capacity, dht=False):
    import cascade_cpp
    cfg = cascade_cpp.DistributedConfig()
    cfg.collective_timeout_ms = args.collective_timeout_ms
    cfg.gpu_capacity_per_device = capacity
    cfg.dram_capacity = 0
    cfg.device = device_index
    cfg.copy_engine = args.copy_engine
    cfg.index_log2 = 18 if not dht else 20
    cfg.hash_lanes = args.hash_lanes
    cfg.pipeline_blocks = args.pipeline_blocks
    cfg.hash_sms = args.hash_sms
    cfg.profile = not getattr(args, "no_profile", False)  # per-kernel CUDA-event timing for the roofline fields
    cfg.dht = dht        # N>1: one hash-sharded store over all ranks
    return cascade_cpp.DistributedStore(cfg)


def plan_gets(keys_all, rng_seed):
    """The get side of a step: every distinct stored key once, in a uniformly
    shuffled order. Prepared from the IDs the puts returned, outside the
    timed region (the IDs are the same every step)."""
    uk = np.unique(keys_all.view(np.dtype((np.void, 16))).reshape(-1))
    order = np.random.default_rng(rng_seed).permutation(len(uk))
    return np.ascontiguousarray(uk[order].view(np.uint8).reshape(-1, 16))


def n_get_calls(keys, batch):
    """Get calls of a step; in a DHT the largest over ranks (every get is
    collective, so ranks with fewer keys join the last calls with empty
    batches)."""
    import torch
    n_get = (len(keys) + batch - 1) // batch
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        t = torch.tensor([n_get], dtype=torch.int64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        n_get = int(t.item())
    return n_get


def run_pass(store, ptrs, sizes, prefix, batch, out_buf, size, rng_seed, device_memory=True, pipelined=True,
             keys_all=None, gets=None):
    """One step: put everything in batches, then get every stored key in a
    shuffled order into out_buf (one batch at a time). Device blocks go
    through the pipelined put (each batch's SHA-256 launched at submission,
    batches placed in order; one wait at the end) and the stream-ordered get;
    host blocks through the synchronous calls. `gets` = (keys in get order,
    number of get calls) prepared beforehand (plan_gets); without it they
    are prepared from this pass's IDs between the two phases, outside both
    phase timings. Returns (put_s, get_s, put_bytes, get_bytes) measured
    with CUDA events on the current stream (the put phase ends with a host
    wait for every placement)."""
    import torch
    n = len(ptrs)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    if keys_all is None:
        keys_all = np.empty((n, 16), np.uint8)
    ev[0].record()
    for i in range(0, n, batch):
        if _TRACE["on"] and (i // batch) % 16 == 0:
            trace(None, f"  put batch {i // batch}")
        if device_memory and pipelined:
            store.put_ptrs_async(ptrs[i:i + batch], sizes[i:i + batch], keys_out=keys_all[i:i + batch],
                                 prefix=prefix[i:i + batch])
        else:
            k, _ = store.put_ptrs(ptrs[i:i + batch], sizes[i:i + batch], device_memory,
                                  prefix=prefix[i:i + batch])
            keys_all[i:i + batch] = k
    if device_memory and pipelined:
        store.wait_puts()
    ev[1].record()
    if gets is None:
        keys = plan_gets(keys_all, rng_seed)
        gets = (keys, n_get_calls(keys, batch))
    keys, n_get = gets
    base = out_buf.data_ptr() if hasattr(out_buf, "data_ptr") else out_buf.ctypes.data
    outs_b = np.uint64(base) + np.arange(batch, dtype=np.uint64) * np.uint64(size)
    caps = np.full(batch, size, np.uint64)
    got = 0
    ev[2].record()
    for j in range(n_get):
        i = j * batch
        if _TRACE["on"] and j % 16 == 0:
            trace(None, f"  get batch {j} of {len(keys)} keys")
        kk = keys[i:i + batch]
        m = len(kk)
        if device_memory and pipelined:
            s, f = store.get_ptrs_async(kk, outs_b[:m], caps[:m])
        else:
            s, f = store.get_ptrs(kk, outs_b[:m], caps[:m], device_memory)
        ok = (f & 0x0F) != 0
        got += int(s[ok].sum())
    ev[3].record()
    ev[3].synchronize()
    put_s = ev[0].elapsed_time(ev[1]) / 1e3
    get_s = ev[2].elapsed_time(ev[3]) / 1e3
    return put_s, get_s, int(sizes.sum()), got


def reduce_max(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------- baseline

def host_cpu():
    """(model name, SHA-NI present) of this host, from /proc/cpuinfo."""
    model, sha = "unknown", False
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name") and model == "unknown":
                    model = line.split(":", 1)[1].strip()
                elif line.startswith("flags"):
                    sha = sha or "sha_ni" in line.split()
    except OSError:
        pass
    return model, sha


def cpu_reference(args, n_blocks, steps=1, threads=None, min_seconds=0.0, max_passes=200, skip=0):
    """The reference's CPU path (oracle/_ref): OpenMP compute_block_id over
    the batch, CascadeStore::put_batch into its SHM tier, shuffled
    get_batch. One store serves every pass (cleared between passes, untimed,
    like the GPU step's clear). The first `skip` passes are warm-up; then at
    least `steps` timed passes, more until `min_seconds` of timed put + get
    have accumulated (at most `max_passes`); the median pass is reported.
    Returns (GB/s, details)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))
    import cascade_ref
    from cascade_cpp import workloads as W
    size = args.block_bytes
    src, is_prefix = W.dedup_mix(n_blocks, max(1, n_blocks // 64), 0.25, 77)
    uniq = np.unique(src)
    packed_u = np.empty(len(uniq) * size, np.uint8)
    for i, s in enumerate(uniq):
        packed_u[i * size:(i + 1) * size] = W.kv_block_fp16(int(s), size)
    pos = np.searchsorted(uniq, src)
    offsets = (pos * size).astype(np.uint64)
    sizes = np.full(n_blocks, size, np.uint64)
    threads = threads or os.cpu_count()
    shm = f"/dev/shm/cascade_bench_{os.getpid()}"
    cap = len(uniq) * size + (64 << 20)
    out = np.empty(len(uniq) * size, np.uint8)
    out_off = (np.arange(len(uniq)) * size).astype(np.uint64)
    # the IDs read back (untimed; the same every pass)
    all_ids = list(dict.fromkeys(cascade_ref.compute_block_ids(packed_u, out_off,
                                                               np.full(len(uniq), size, np.uint64), threads)))
    order = np.random.default_rng(5).permutation(len(all_ids))
    store = cascade_ref.CascadeStore(shm_capacity=cap, shm_path=shm)
    times, done = [], 0
    try:
        while done < skip or len(times) < steps or (sum(a + b for a, b in times) < min_seconds
                                                    and len(times) < max_passes):
            t0 = time.perf_counter()
            for i in range(0, n_blocks, args.batch):
                ids = cascade_ref.compute_block_ids(packed_u, offsets[i:i + args.batch], sizes[i:i + args.batch],
                                                    threads)
                store.put_batch(ids, packed_u, offsets[i:i + args.batch], sizes[i:i + args.batch])
            t1 = time.perf_counter()
            for i in range(0, len(order), args.batch):
                sel = order[i:i + args.batch]
                found, _ = store.get_batch([all_ids[j] for j in sel], out, out_off[:len(sel)])
                assert found == len(sel)
            t2 = time.perf_counter()
            if done >= skip:
                times.append((t1 - t0, t2 - t1))
            done += 1
            store.clear()
    finally:
        del store
        shutil.rmtree(shm, ignore_errors=True)
    put_s = float(np.median([t[0] for t in times]))
    get_s = float(np.median([t[1] for t in times]))
    put_b, get_b = n_blocks * size, len(uniq) * size
    return (put_b + get_b) / (put_s + get_s) / GB, {
        "put_gbs": put_b / put_s / GB, "get_gbs": get_b / get_s / GB, "cores": threads, "seconds": put_s + get_s,
        "passes": len(times), "pass_seconds": [a + b for a, b in times],
        "cpu_model": host_cpu()[0], "sha_ni": host_cpu()[1],
        "sample": f"{n_blocks} x {size} B blocks (25% copies), batch {args.batch}; median of {len(times)} "
                  f"passes ({sum(a + b for a, b in times):.1f} s timed)"}


# ------------------------------------------------------------------- main

def main():
    args = parse()
    _TRACE["on"] = args.trace
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        ok = os.path.exists(os.path.join(ROOT, "oracle", "_ref"))
        if not ok:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built"}))
            return
        v, det = cpu_reference(args, args.cpu_blocks, steps=args.steps, skip=args.warmup)
        el = float(np.sum(det["pass_seconds"]))  # timed put + get of the K steps (generation excluded)
        ref_config = config_dict(args)
        ref_config["workload"] += (f"; the reference's CPU path timed on a {args.cpu_blocks}-block sample of this "
                                   "stream (same block size, duplicate mix and batch) per step")
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s",
            "value_gibs": round(v * GB / 2**30, 3), "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic", "config": ref_config,
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": det["cores"], "kind": "reference",
                             "sample": det["sample"], "put_gbs": round(det["put_gbs"], 3),
                             "get_gbs": round(det["get_gbs"], 3), "cpu_model": det["cpu_model"],
                             "sha_ni": det["sha_ni"]},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    size = args.block_bytes

    if args.workload == "zipf":
        return zipf_main(args, rank, world, local, device)
    if args.workload == "spill":
        return spill_main(args, rank, world, local, device)
    if args.workload == "sweep":
        return sweep_main(args, rank, world, local, device)
    trace(args, "generating blocks")
    pool, ptrs, prefix = gpu_blocks(args, rank, device)
    sizes = np.full(len(ptrs), size, np.uint64)
    n_unique = pool.numel() // size
    # DHT (N>1): an owner holds ~1/W of every rank's unique blocks; leave
    # room for the owner imbalance of a random hash placement.
    cap = n_unique * size + (256 << 20) if world == 1 else int(n_unique * size * 1.15) + (1 << 30)
    trace(args, "creating the store")
    store = make_store(args, local, cap, dht=world > 1)
    trace(args, "store ready")
    out_buf = torch.empty(args.batch * size, dtype=torch.uint8, device=device)

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()

    keys_ref = np.empty((len(ptrs), 16), np.uint8)
    for w in range(max(args.warmup, 1)):  # (at least one: the IDs the timed steps get come from it)
        trace(args, f"warm-up pass {w}")
        store.clear()
        run_pass(store, ptrs, sizes, prefix, args.batch, out_buf, size, w, keys_all=keys_ref)
    # the get side of every timed step: all distinct IDs in a fresh shuffled
    # order per step (the IDs themselves are the same every step; each
    # step's are checked against them after the timed region)
    step_gets = []
    for s in range(args.steps):
        keys = plan_gets(keys_ref, 100 + s)
        step_gets.append((keys, n_get_calls(keys, args.batch)))
    step_keys = [np.empty_like(keys_ref) for _ in range(args.steps)]
    trace(args, "timed passes")
    st0 = store._n.stats()
    sync_all()
    put_t = get_t = 0.0
    put_b = get_b = 0
    t_ev0 = torch.cuda.Event(enable_timing=True)
    t_ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t_ev0.record()
        for s in range(args.steps):
            store.clear()
            ps, gs, pb, gb = run_pass(store, ptrs, sizes, prefix, args.batch, out_buf, size, 100 + s,
                                      keys_all=step_keys[s], gets=step_gets[s])
            put_t += ps
            get_t += gs
            put_b += pb
            get_b += gb
        t_ev1.record()
        sync_all()
    if not all(np.array_equal(k, keys_ref) for k in step_keys):
        raise SystemExit("block IDs of a timed step differ from the warm-up's")
    # clear() resets the counters: what they hold now is the last step's
    dedup_step = reduce_sum(store._n.stats().dedup_hits, world)
    elapsed = t_ev0.elapsed_time(t_ev1) / 1e3
    st1 = store._n.stats()
    remote_b = st1.peer_bytes_read - st0.peer_bytes_read  # crossed NVLink
    elapsed_max = reduce_max(elapsed, world)
    total_bytes = reduce_sum(put_b + get_b, world)
    value = total_bytes / elapsed_max / GB
    put_gbs = reduce_sum(put_b / put_t, world) / GB
    get_gbs = reduce_sum(get_b / get_t, world) / GB

    peaks = {}
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peaks = json.load(open(pk))
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"

    def d(f):
        return getattr(st1, f) - getattr(st0, f)

    # Pipelined puts keep many SHA-256 launches in flight at once (bytes and
    # launch counts come from the store; the launches overlap, so their
    # aggregate rate is the bytes hashed over the put phases' CUDA-event time
    # on this stream - a lower bound, the phases also hold the last
    # placements)
    sha_bytes_launch = d("sha_bytes") / max(d("sha_launches"), 1)
    sha_achieved = d("sha_bytes") / put_t / GB if put_t else 0.0
    clk_sum = clk.summary()
    sm_mhz = clk_sum.get("sm_mhz") or 1965.0
    n_sms = torch.cuda.get_device_properties(device).multi_processor_count
    # the integer ALU pipe: 16 lanes per cycle per sub-partition (4 per SM);
    # SHA-256 needs >= 1040 ALU lane-instructions per 64-byte chunk (64 rounds
    # x 10 rotates/LOP3, 48 schedule words x 8, 16 byte swaps)
    alu_peak = n_sms * 4 * 16 * sm_mhz * 1e6 * 64 / SHA_ALU_INSTR_PER_CHUNK / GB
    gather_s = d("gather_ns") / 1e9
    gather_alg = 2 * d("gather_bytes")
    gather_achieved = gather_alg / gather_s / GB if gather_s else 0.0
    scatter_s = d("scatter_ns") / 1e9
    scatter_achieved = 2 * d("scatter_bytes") / scatter_s / GB if scatter_s else 0.0
    launches = d("kernel_launches")

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "value_gibs": round(value * GB / 2**30, 3),
        "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed_max / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded fp16 N(0,1) KV blocks generated on the GPU)",
        "config": config_dict(args),
        "batch_put_gbs": round(put_gbs, 3), "batch_get_gbs": round(get_gbs, 3),
        "roofline": {
            "kernel": "sha256_fused_kernel", "bound": "hbm", "achieved": round(sha_achieved, 2),
            "peak": hbm_peak, "unit": "GB/s", "frac": round(sha_achieved / hbm_peak, 5),
            "peak_source": peak_src,
            # dram__bytes_read.sum + dram__bytes_write.sum of one 1024-block
            # sha256_fused_kernel launch from an ncu capture of this workload
            # (736.6 MB read + 4.1 MB written; most of the 25 % copies are
            # read from L2, not DRAM)
            "traffic": SHA_TRAFFIC_PER_1024_LAUNCH if args.batch == 1024 else None,
            "bytes_per_launch": int(sha_bytes_launch),
            "launches": int(d("sha_launches")),
            "achieved_is": "block bytes hashed / put-phase time (CUDA events on the caller's stream); up to "
                           f"{args.pipeline_blocks or '65536'} blocks hash at once in overlapping launches",
            "binding": {"pipe": "integer ALU (rotates, shifts, 3-input logic of SHA-256)",
                        "peak_gbs": round(alu_peak, 1), "frac": round(sha_achieved / alu_peak, 4),
                        "sm_mhz": sm_mhz, "sms": n_sms,
                        "peak_is": f"{n_sms} SMs x 4 x 16 lanes/cycle x clock x 64 B / "
                                   f"{SHA_ALU_INSTR_PER_CHUNK} ALU lane-instructions per chunk"},
        },
        "roofline_get": {
            "kernel": "copy (gather)", "bound": "hbm", "achieved": round(gather_achieved, 2), "peak": hbm_peak,
            "unit": "GB/s", "frac": round(gather_achieved / hbm_peak, 4), "peak_source": peak_src,
            "bytes_per_launch": int(gather_alg / max(d("gather_launches"), 1)),
        },
        "roofline_put_scatter": {"achieved": round(scatter_achieved, 2), "unit": "GB/s",
                                 "frac": round(scatter_achieved / hbm_peak, 4)},
        "gpu_launches": int(launches),
    }
    if world > 1:
        # remote gets cross NVLink: bytes received per GPU / gather time,
        # against the measured 770 GB/s peer copy per direction
        nv = remote_b / gather_s / GB if gather_s else 0.0
        nv_min = reduce_max(-nv, world) * -1.0
        line["roofline_nvlink"] = {"kernel": "copy_lsu (peer-load gather)", "bound": "nvlink",
                                   "achieved_per_gpu_min": round(nv_min, 2), "achieved_rank0": round(nv, 2),
                                   "peak": NVLINK_PEER_GBS, "unit": "GB/s",
                                   "frac": round(nv_min / NVLINK_PEER_GBS, 4),
                                   "frac_of_nominal_900": round(nv_min / 900.0, 4),
                                   "note": "remote bytes received per GPU / gather kernel time (the gather also "
                                           "moves the local 1/W from HBM)",
                                   "remote_fraction": round(remote_b / max(1, get_b), 4)}
        # every DHT collective step (count all-gathers, key/reply
        # all-to-alls, put barriers), CUDA events on the store's stream: the
        # time includes waiting for the slowest peer
        coll_ms = reduce_max(d("coll_ns") / 1e6 / args.steps, world)
        line["collectives"] = {"calls_per_step": round(d("coll_calls") / args.steps, 1),
                               "ms_per_step_max_rank": round(coll_ms, 3),
                               "share_of_step": round(coll_ms / (elapsed_max / args.steps * 1e3), 4),
                               "bytes_sent_per_step_rank0": int(d("coll_bytes") / args.steps)}
        line["config"]["parallelism"] = f"hash-sharded DHT over {world} GPUs (owner = ID mod {world})"
    line["clocks"] = clk_sum
    trace(args, "verification")
    line["verified"] = verify_run(store, ptrs, sizes, keys_ref, dedup_step, out_buf, size, local, world)
    line["roofline"]["chain_bound"] = chain_rates(store, ptrs, sizes, size, sm_mhz, n_sms, put_t,
                                                  d("sha_bytes"))

    if not args.no_sweep:
        trace(args, "batch sweep")
        sw = batch_sweep(args, store, ptrs, sizes, prefix, out_buf, size)  # collective in a DHT
        if rank == 0:
            line["sweep"] = sw
    del pool
    torch.cuda.empty_cache()
    if not args.no_e2e:
        trace(args, "e2e")
        line["e2e"] = e2e_run(args, rank, world, device, store)
    trace(args, "done")
    if rank == 0 and world == 1 and not args.no_cpu:  # the CPU baseline is an N=1 figure
        try:
            v, det = cpu_reference(args, args.cpu_blocks, steps=1, min_seconds=args.cpu_seconds)
            line["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": det["cores"],
                                    "kind": "reference", "sample": det["sample"],
                                    "put_gbs": round(det["put_gbs"], 3), "get_gbs": round(det["get_gbs"], 3),
                                    "cpu_model": det["cpu_model"], "sha_ni": det["sha_ni"]}
        except Exception as e:  # pragma: no cover
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    store.close()
    if world > 1:
        torch.distributed.destroy_process_group()
    if not line["verified"]["ok"]:
        sys.exit(3)


def chain_rates(store, ptrs, sizes, size, sm_mhz, n_sms, put_t, sha_bytes):
    """Cycles per SHA-256 round, from CUDA-event times x the median SM clock
    sampled during the timed region:
    * one chain: a synchronous 1024-block hashing call on the store (one
      producer/consumer launch, every chain alone on its two sub-partitions)
      = launch time x clock / (64-byte chunks per block x 64 rounds);
    * pipelined put: sub-partition cycles spent per 32-chain round during the
      timed put phases = put time x clock x sub-partitions / (chunks hashed /
      32 x 64); the integer ALU pipe needs 32.5 (1040 lane-instructions per
      chunk at 16 lanes per cycle, per 64 rounds)."""
    from cascade_cpp import _lib as L
    nch = (size + 9 + 63) // 64
    n = min(1024, len(ptrs))
    st0 = store._n.stats()
    store._n.hash(np.ascontiguousarray(ptrs[:n]), np.ascontiguousarray(sizes[:n]), L.CB_MEM_DEVICE)
    st1 = store._n.stats()
    if st1.sha_launches == st0.sha_launches:  # profiling off
        return None
    t_ns = (st1.sha_ns - st0.sha_ns) / (st1.sha_launches - st0.sha_launches)
    one = t_ns * 1e-9 * sm_mhz * 1e6 / (nch * 64)
    chunks = sha_bytes / size * nch
    piped = put_t * sm_mhz * 1e6 * n_sms * 4 / (chunks / 32 * 64) if chunks else None
    return {"one_chain_cycles_per_round": round(one, 2), "one_chain_design_floor": 20,
            "one_chain_launch_ms": round(t_ns / 1e6, 3), "one_chain_blocks": n,
            "pipelined_smsp_cycles_per_warp_round": round(piped, 2) if piped else None,
            "pipelined_alu_floor": SHA_ALU_INSTR_PER_CHUNK * 2 / 64,
            "how": "CUDA-event launch times x median SM MHz of the timed region"}


def verify_run(store, ptrs, sizes, keys_ref, dedup_step, out_buf, size, local, world, sample=256):
    """Checks of the run's results, on every rank (collective in a DHT):
    * IDs: a seeded sample of put positions re-hashed from their source
      blocks by the store-less hashing call equals the IDs the puts returned;
    * dedup: dedup hits per step, summed over ranks, equal the blocks put
      minus the distinct IDs over all ranks (every distinct block is stored
      exactly once cluster-wide, every other put is a hit);
    * read-back: a seeded sample of this rank's distinct IDs fetched again
      through the store re-hashes on the GPU to the requested IDs.
    Returns {"ok": bool, ...}; the caller exits non-zero when ok is false."""
    import torch
    import cascade_cpp
    from cascade_cpp import _lib as L
    rank = int(os.environ.get("RANK", "0"))
    rng = np.random.default_rng(4242 + rank)
    hasher = cascade_cpp._hasher(local)
    sel = np.sort(rng.choice(len(ptrs), min(sample, len(ptrs)), replace=False))
    dig = hasher.hash(np.ascontiguousarray(ptrs[sel]), np.ascontiguousarray(sizes[sel]), L.CB_MEM_DEVICE)
    ids_ok = bool(np.array_equal(dig[:, :16], keys_ref[sel]))
    all_keys = keys_ref
    if world > 1:
        kt = torch.from_numpy(keys_ref).cuda()
        parts = [torch.empty_like(kt) for _ in range(world)]
        torch.distributed.all_gather(parts, kt)
        all_keys = torch.cat(parts).cpu().numpy()
    distinct = len(np.unique(all_keys.view(np.dtype((np.void, 16))).reshape(-1)))
    dedup_want = len(all_keys) - distinct
    dedup_ok = abs(dedup_step - dedup_want) < 0.5
    uk = plan_gets(keys_ref, 777 + rank)[:min(sample, len(keys_ref), out_buf.numel() // size)]
    m = len(uk)
    outs = (np.uint64(out_buf.data_ptr()) + np.arange(m, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
    s, f = store.get_ptrs(uk, outs, np.full(m, size, np.uint64), True)
    found_ok = bool(((f & 0x0F) != 0).all() and (s == size).all())
    torch.cuda.synchronize()
    back = hasher.hash(outs, np.full(m, size, np.uint64), L.CB_MEM_DEVICE)
    read_ok = found_ok and bool(np.array_equal(back[:, :16], uk))
    oks = [ids_ok, dedup_ok, read_ok]
    if world > 1:
        t = torch.tensor([0 if x else 1 for x in oks], dtype=torch.int64, device="cuda")
        torch.distributed.all_reduce(t)
        oks = [int(v) == 0 for v in t.tolist()]
    return {"ok": all(oks), "ids": oks[0], "dedup": oks[1], "read_back": oks[2], "sample": int(len(sel)),
            "dedup_hits_per_step": round(dedup_step, 1), "expected_dedup_hits": int(dedup_want),
            "how": "IDs of a seeded sample re-hashed from the source blocks (store-less hashing call); dedup hits "
                   "per step summed over ranks = blocks put - distinct IDs over all ranks; a seeded sample of "
                   "distinct IDs fetched again and re-hashed on the GPU (all ranks must pass)"}


def zipf_main(args, rank, world, local, device):
    """Config 4: hash-sharded DHT of Qwen2.5-72B-shaped blocks (5,242,880 B,
    bf16 N(0,1) generated on the GPU). Every rank puts --zipf-blocks-per-gpu
    blocks (weak scaling: 20,000 per GPU = 160,000 at 8 GPUs), then each step
    every rank batch_gets --zipf-batch keys drawn from a bounded Zipf(alpha)
    over all ranks' keys (seeded rank->key permutation); ~(W-1)/W of the
    fetches are NVLink peer reads."""
    import torch
    import torch.distributed as dist
    from cascade_cpp import workloads as W
    size, nb, gb = args.zipf_block_bytes, args.zipf_blocks_per_gpu, args.zipf_batch
    cap = int(nb * size * 1.12) + (1 << 30)
    store = make_store(args, local, cap, dht=world > 1)
    pb = 256
    buf = torch.empty(pb * size, dtype=torch.uint8, device=device)
    g = torch.Generator(device=device).manual_seed(7000 + rank)
    keys = np.empty((nb, 16), np.uint8)
    t0 = time.perf_counter()
    for i in range(0, nb, pb):
        m = min(pb, nb - i)
        buf[:m * size].view(torch.bfloat16).copy_(
            torch.randn(m * size // 2, generator=g, device=device, dtype=torch.bfloat16))
        ptrs = (np.uint64(buf.data_ptr()) + np.arange(m, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
        k, _ = store.put_ptrs(ptrs, np.full(m, size, np.uint64), True)
        keys[i:i + m] = k
    torch.cuda.synchronize()
    populate_s = time.perf_counter() - t0
    del buf
    torch.cuda.empty_cache()
    if world > 1:
        kt = torch.from_numpy(keys).to(device)
        parts = [torch.empty_like(kt) for _ in range(world)]
        dist.all_gather(parts, kt)
        gkeys = torch.cat(parts).cpu().numpy()
    else:
        gkeys = keys
    total_steps = args.warmup + args.steps
    draws = W.zipf_keys(len(gkeys), total_steps * gb, args.zipf_alpha, seed=100 + rank)
    out = torch.empty(gb * size, dtype=torch.uint8, device=device)
    outs = (np.uint64(out.data_ptr()) + np.arange(gb, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
    caps = np.full(gb, size, np.uint64)
    for s in range(args.warmup):
        store.get_ptrs(gkeys[draws[s * gb:(s + 1) * gb]], outs, caps, True)
    st0 = store._n.stats()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    got = 0
    with ClockSampler(local) as clk:
        ev0.record()
        for s in range(args.warmup, total_steps):
            sz, f = store.get_ptrs(gkeys[draws[s * gb:(s + 1) * gb]], outs, caps, True)
            got += int(sz[(f & 0x0F) != 0].sum())
        ev1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    el = reduce_max(ev0.elapsed_time(ev1) / 1e3, world)
    st1 = store._n.stats()
    tot = reduce_sum(got, world)
    d = {f: getattr(st1, f) - getattr(st0, f) for f in ("remote_gpu_hits", "local_gpu_hits", "gather_ns",
                                                        "gather_bytes", "kernel_launches", "peer_bytes_read")}
    remote_b = d["peer_bytes_read"]  # fetched over NVLink (a key repeated in a batch crosses once)
    gather_s = d["gather_ns"] / 1e9
    nv = remote_b / gather_s / GB if gather_s else 0.0
    nv_min = -reduce_max(-nv, world)
    # owner egress imbalance: requests served per owner this run
    line = {
        "metric": "aggregate batch_get GB/s (config 4: DHT, Zipf keys)", "value": round(tot / el / GB, 3),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded bf16 N(0,1) blocks generated on the GPU)",
        "config": {"workload": f"config4: {nb} x {size} B Qwen2.5-72B KV blocks per GPU ({nb * world} total), "
                               f"batch_get of {gb} keys per rank per step, Zipf alpha {args.zipf_alpha}",
                   "parallelism": f"hash-sharded DHT over {world} GPUs" if world > 1 else "single store",
                   "l2": "every step reads 2.7 GB per GPU >> L2"},
        "populate_s": round(populate_s, 2),
        "remote_fraction": round(d["remote_gpu_hits"] / max(1, d["remote_gpu_hits"] + d["local_gpu_hits"]), 4),
        "nvlink_bytes_per_step": int(remote_b / max(args.steps, 1)),
        "logical_bytes_per_step": int(got / max(args.steps, 1)),
        "roofline": {"kernel": "copy_lsu (peer-load gather)", "bound": "nvlink" if world > 1 else "hbm",
                     "achieved": round(nv_min if world > 1 else 2 * d["gather_bytes"] / gather_s / GB, 2),
                     "peak": NVLINK_PEER_GBS if world > 1 else None, "unit": "GB/s",
                     "frac": round(nv_min / NVLINK_PEER_GBS, 4) if world > 1 else None,
                     "frac_of_nominal_900": round(nv_min / 900.0, 4) if world > 1 else None},
        "gpu_launches": int(d["kernel_launches"]), "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    store.close()
    if world > 1:
        dist.destroy_process_group()


def sweep_main(args, rank, world, local, device):
    """Config 5: block sizes 4 KiB, 64 KiB, 1 MiB, 4 MiB, 16 MiB of bf16
    N(0,1); each step is 512 ops, 30 % batch_put (half of them byte-identical
    copies of a block this rank put earlier) and 70 % batch_get of uniformly
    drawn keys this rank stored; 16 GiB of logical traffic per GPU per size
    (--sweep-gib). Reports GB/s and p50/p99 step latency per size. On N GPUs
    every call is a DHT collective."""
    import torch
    import cascade_cpp
    out = {}
    ops = 512
    n_put = int(round(ops * 0.3))
    n_get = ops - n_put
    for size in [int(s) for s in args.sweep_sizes.split(",")]:
        steps = max(2, int(args.sweep_gib * (1 << 30) // (ops * size)))
        uniq_needed = steps * n_put // 2 + n_put + 1
        cfg = cascade_cpp.DistributedConfig()
        cfg.gpu_capacity_per_device = int(uniq_needed * size * 1.3) + (1 << 30)
        cfg.dram_capacity = 0
        cfg.device = local
        cfg.index_log2 = max(16, int(np.ceil(np.log2(max(uniq_needed * 2.6, 2)))))
        cfg.dht = world > 1
        cfg.profile = False
        store = cascade_cpp.DistributedStore(cfg)
        g = torch.Generator(device=device).manual_seed(500 + rank)
        src = torch.randn(uniq_needed * size // 2, generator=g, device=device, dtype=torch.bfloat16).view(torch.uint8)
        base = np.uint64(src.data_ptr())
        rng = np.random.default_rng(600 + rank)
        outb = torch.empty(n_get * size, dtype=torch.uint8, device=device)
        optrs = (np.uint64(outb.data_ptr()) + np.arange(n_get, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
        caps = np.full(n_get, size, np.uint64)
        sizes = np.full(n_put, size, np.uint64)
        # seed the store with one batch of unique blocks so gets have targets;
        # source block j is stored under keys[j] (unique blocks are consecutive)
        keys = np.empty((uniq_needed, 16), np.uint8)
        p0 = (base + np.arange(n_put, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
        k, _ = store.put_ptrs(p0, sizes, True)
        keys[:n_put] = k
        nxt = n_put
        lat = []
        logical = 0
        new = n_put - n_put // 2
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        t_all = time.perf_counter()
        for s in range(steps):
            # half new blocks, half copies of blocks put earlier (50 % dedup)
            sel = np.concatenate([np.arange(nxt, nxt + new), rng.integers(0, nxt, n_put // 2)])
            ptrs = (base + sel.astype(np.uint64) * np.uint64(size)).astype(np.uint64)
            gk = keys[rng.integers(0, nxt, n_get)]
            t0 = time.perf_counter()
            k, st = store.put_ptrs(ptrs, sizes, True)
            sz, f = store.get_ptrs(gk, optrs, caps, True)
            lat.append(time.perf_counter() - t0)
            logical += n_put * size + int(sz[(f & 0x0F) != 0].sum())
            keys[nxt:nxt + new] = k[:new]
            nxt += new
        el = time.perf_counter() - t_all
        el = reduce_max(el, world)
        tot = reduce_sum(logical, world)
        lat_ms = np.array(lat) * 1e3
        out[str(size)] = {"gbs": round(tot / el / GB, 3), "steps": steps,
                          "p50_ms": round(float(np.percentile(lat_ms, 50)), 3),
                          "p99_ms": round(float(np.percentile(lat_ms, 99)), 3),
                          "dedup_hits": int(store.get_stats().dedup_hits)}
        store.close()
        del src, outb
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({
            "metric": "config 5 variable-block sweep: aggregate GB/s and p50/p99 step latency per size",
            "n_gpus": world, "unit": "GB/s", "higher_is_better": True, "scaling": "weak", "dtype": "u8",
            "data": "synthetic (seeded bf16 N(0,1) blocks generated on the GPU)",
            "config": {"workload": f"config5: 512 ops/step (30% put, half of them copies; 70% get, uniform keys), "
                                   f"{args.sweep_gib} GiB logical per GPU per size",
                       "parallelism": f"hash-sharded DHT over {world} GPUs" if world > 1 else "single store"},
            "per_size": out}), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def host_link_peaks(device, nbytes=4 << 30, reps=3):
    """Pinned host<->device copy bandwidth (copy engines), GB/s."""
    import torch
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dbuf = torch.empty(nbytes, dtype=torch.uint8, device=device)
    res = {}
    for name, dst, src in (("h2d", dbuf, h), ("d2h", h, dbuf)):
        dst.copy_(src, non_blocking=True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            dst.copy_(src, non_blocking=True)
        e1.record()
        e1.synchronize()
        res[name] = nbytes * reps / (e0.elapsed_time(e1) / 1e3) / GB
    del h, dbuf
    torch.cuda.empty_cache()
    return res


def spill_main(args, rank, world, local, device):
    """Config 3: 40,000 Qwen2.5-72B-shaped blocks (5,242,880 B bf16) into a
    120 GB HBM pool with a pinned DRAM tier; 10 % of the blocks (seeded) are
    prefix-protected. Put everything (LRU demotions to DRAM run as mapped-host
    copy kernels), then batch_get Zipf(1.1) keys; DRAM hits are promoted back
    to HBM (each promotion demotes an LRU block). Every warm-up get batch is
    checked: the bytes returned must hash (GPU SHA-256) to the requested ID.
    With --kv-compression the DRAM tier holds INT8-packed blocks (8 + size/2
    bytes) and a block that went through it reads back lossy, so the check
    keeps the originals of the first 128 distinct blocks the warm-up steps
    draw: a read of one must equal the original or its KVCompressor round
    trip."""
    import torch
    import cascade_cpp
    from cascade_cpp import workloads as W
    size, nb = args.zipf_block_bytes, args.spill_blocks
    peaks = host_link_peaks(device)
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = int(args.spill_hbm_gb * 1e9)
    cfg.dram_capacity = int(args.spill_dram_gb * 1e9)
    cfg.device = local
    cfg.profile = True
    cfg.dht = False
    cfg.index_log2 = 17
    cfg.kv_compression = bool(args.kv_compression)
    # the configuration asks for promotion to run: CascadeStore's rule (every
    # DRAM hit moves back to HBM), not DistributedStore's locality rule, under
    # which a single store's own DRAM hits are never promoted
    cfg.promote_on_hit = True
    store = cascade_cpp.DistributedStore(cfg)
    rng = np.random.default_rng(33)
    prefix = (rng.random(nb) < 0.10).astype(np.uint8)
    pb = 256
    buf = torch.empty(pb * size, dtype=torch.uint8, device=device)
    gb = args.zipf_batch
    total_steps = args.warmup + args.steps
    draws = W.zipf_keys(nb, total_steps * gb, args.zipf_alpha, seed=34)
    slot = {}
    if args.kv_compression:
        for b in draws[:args.warmup * gb]:
            if len(slot) == 128:
                break
            slot.setdefault(int(b), len(slot))
    n_keep = len(slot)
    kept = torch.empty(max(n_keep, 1) * size, dtype=torch.uint8, device=device)
    g = torch.Generator(device=device).manual_seed(33)
    keys = np.empty((nb, 16), np.uint8)
    s0 = store._n.stats()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(0, nb, pb):
        m = min(pb, nb - i)
        buf[:m * size].view(torch.bfloat16).copy_(
            torch.randn(m * size // 2, generator=g, device=device, dtype=torch.bfloat16))
        for j in range(i, i + m):
            if j in slot:
                kept[slot[j] * size:(slot[j] + 1) * size].copy_(buf[(j - i) * size:(j - i + 1) * size])
        ptrs = (np.uint64(buf.data_ptr()) + np.arange(m, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
        k, st = store.put_ptrs(ptrs, np.full(m, size, np.uint64), True, prefix=prefix[i:i + m])
        assert (st == 0).all(), "put failed"
        keys[i:i + m] = k
    torch.cuda.synchronize()
    put_s = time.perf_counter() - t0
    s1 = store._n.stats()
    del buf
    torch.cuda.empty_cache()
    # prefix protection: no prefix block may sit in DRAM while HBM holds a
    # non-prefix block
    in_dram = [store.locate(k.tobytes().hex()) for k in keys]
    pf_dram = sum(1 for j, l in enumerate(in_dram) if prefix[j] and not l.is_gpu)
    np_hbm = sum(1 for j, l in enumerate(in_dram) if not prefix[j] and l.is_gpu)
    out = torch.empty(gb * size, dtype=torch.uint8, device=device)
    outs = (np.uint64(out.data_ptr()) + np.arange(gb, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
    caps = np.full(gb, size, np.uint64)
    hasher = cascade_cpp._hasher(local)
    if n_keep:
        blocks = [kept[j * size:(j + 1) * size] for j in range(n_keep)]
        rt = cascade_cpp.KVCompressor.decompress_batch(cascade_cpp.KVCompressor.compress_batch(blocks),
                                                       [size] * n_keep)
    checked = 0
    for s in range(args.warmup):
        dk = draws[s * gb:(s + 1) * gb]
        kk = keys[dk]
        sz, f = store.get_ptrs(kk, outs, caps, True)
        assert ((f & 0x0F) != 0).all()
        if not n_keep:
            dig = hasher.hash(outs, caps, 0)  # bytes returned hash to the requested IDs
            assert np.array_equal(dig[:, :16], kk), "get returned wrong bytes"
            continue
        for j, b in enumerate(dk):
            if int(b) in slot:
                o, t = out[j * size:(j + 1) * size], slot[int(b)]
                assert torch.equal(o, blocks[t]) or torch.equal(o, rt[t]), "get returned wrong bytes"
                checked += 1
    s2 = store._n.stats()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    got = 0
    with ClockSampler(local) as clk:
        ev0.record()
        for s in range(args.warmup, total_steps):
            sz, f = store.get_ptrs(keys[draws[s * gb:(s + 1) * gb]], outs, caps, True)
            got += int(sz[(f & 0x0F) != 0].sum())
        ev1.record()
        torch.cuda.synchronize()
    get_s = ev0.elapsed_time(ev1) / 1e3
    s3 = store._n.stats()

    def dd(a, b, f):
        return getattr(b, f) - getattr(a, f)

    ev_b, ev_ns = dd(s0, s1, "tier_bytes"), dd(s0, s1, "tier_ns")
    pr_b, pr_ns = dd(s2, s3, "tier_bytes"), dd(s2, s3, "tier_ns")
    # bytes that crossed the host link on demotion: packed (8 + size/2 per
    # block) with kv_compression, the whole block without
    link_b = ev_b // size * (8 + size // 2) if args.kv_compression else ev_b
    line = {
        "metric": "tier moves (config 3: HBM <-> pinned DRAM spill)", "value": round(got / get_s / GB, 3),
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(get_s / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded bf16 N(0,1) blocks generated on the GPU)",
        "config": {"workload": f"config3: {nb} x {size} B Qwen2.5-72B blocks ({nb * size / 1e9:.1f} GB), HBM pool "
                               f"{args.spill_hbm_gb} GB, pinned DRAM {args.spill_dram_gb} GB, 10% prefix, "
                               f"batch_get {gb} Zipf({args.zipf_alpha}) keys per step, promotion on DRAM hit"
                               + (", kv_compression (INT8 DRAM tier)" if args.kv_compression else "")},
        "value_is": "batch_get GB/s in the timed steps (DRAM hits promoted inline)",
        "put_phase": {"seconds": round(put_s, 2), "gb_put": round(nb * size / 1e9, 1),
                      "gpu_evictions": dd(s0, s1, "gpu_evictions"), "evicted_gb": round(ev_b / 1e9, 2),
                      "evict_kernel_gbs": round(ev_b / ev_ns, 2) if ev_ns else None,
                      "evict_link_gb": round(link_b / 1e9, 2),
                      "compression_savings_gb": round(dd(s0, s1, "compression_savings") / 1e9, 2),
                      "prefix_blocks_in_dram": pf_dram, "nonprefix_blocks_in_hbm": np_hbm},
        "get_phase": {"local_gpu_hits": dd(s2, s3, "local_gpu_hits"), "local_dram_hits": dd(s2, s3, "local_dram_hits"),
                      "promotions": dd(s2, s3, "promotions_to_local"), "tier_moved_gb": round(pr_b / 1e9, 2),
                      "tier_kernel_gbs": round(pr_b / pr_ns, 2) if pr_ns else None},
        "roofline": {"kernel": ("kv_minmax + kv_pack into HBM staging, then the D2H copy engine" if args.kv_compression
                                else "D2H copy engine (cudaMemcpyAsync of 5 MiB blocks)"), "bound": "host link",
                     "achieved": round(link_b / ev_ns, 2) if ev_ns else None,
                     "peak": round(peaks["d2h"], 2), "unit": "GB/s",
                     "frac": round((link_b / ev_ns) / peaks["d2h"], 4) if ev_ns else None,
                     "achieved_is": "host-link bytes of the demotions / their device time (CUDA events)",
                     "peak_source": "measured pinned D2H copy in this run", "h2d_peak": round(peaks["h2d"], 2)},
        "gpu_launches": dd(s2, s3, "kernel_launches"), "clocks": clk.summary(),
    }
    if n_keep:
        line["check"] = f"{checked} warm-up reads of kept blocks equal the original or its INT8 round trip"
    print(json.dumps(line), flush=True)
    store.close()


def config_dict(args):
    return {"workload": f"config2: {args.blocks} x {args.block_bytes} B Qwen2.5-7B KV blocks (fp16), 25% "
                        f"byte-identical copies of 64 prefix blocks; step = clear + batch_put all (batch "
                        f"{args.batch}) + batch_get all unique in uniform random order",
            "blocks": args.blocks, "block_bytes": args.block_bytes, "batch": args.batch,
            "layout": {"shuffled": "distinct blocks at shuffled places of one buffer (as in the CPU reference arm)",
                       "stream": "distinct blocks in the order of their first occurrence in the put stream"}[
                           getattr(args, "layout", "shuffled")],
            "put": "pipelined batch_put (cb_put_batch_async): each batch's SHA-256 launched at submission, up to "
                   f"{args.pipeline_blocks or 'the library default of 65536'} "
                   "blocks hashing at once, batches placed in submission order",
            "hash_sms": args.hash_sms or "library default (all SMs on one GPU; all but 8 on a DHT member)",
            "get": "stream-ordered batch_get (cb_get_batch_async)",
            "l2": "inputs (the distinct blocks, ~45 GB) resident in HBM, >> 126 MB L2 (no flush needed)",
            "copy_engine": {0: "tma", 1: "tma", 2: "lsu"}[args.copy_engine]}


def batch_sweep(args, store, ptrs, sizes, prefix, out_buf, size):
    """batch_put / batch_get GB/s at batch 64 / 256 / 1024 on an 8192-block
    slice of the same stream: the pipelined put and stream-ordered get (the
    bench's path) and, beside them, the synchronous calls."""
    res = {}
    n = min(8192, len(ptrs))
    for b in (64, 256, 1024):
        r = {}
        for mode, pipelined in (("", True), ("sync_", False)):
            store.clear()
            ps, gs, pb, gb = run_pass(store, ptrs[:n], sizes[:n], prefix[:n], b, out_buf, size, 7,
                                      pipelined=pipelined)
            r[mode + "put_gbs"] = round(pb / ps / GB, 3)
            r[mode + "get_gbs"] = round(gb / gs / GB, 3)
        res[str(b)] = r
    store.clear()
    return res


def e2e_run(args, rank, world, device, store):
    """Public API with pinned host buffers: H2D of every block and D2H of
    every result inside the timed region."""
    import torch
    size = args.block_bytes
    n = min(args.e2e_blocks, args.blocks)
    from cascade_cpp import workloads as W
    src, is_prefix = W.dedup_mix(n, 64, 0.25, 99 + rank)
    uniq = np.unique(src)
    # The put stream as a caller holds it: one pinned [n, block] array of KV
    # pages in stream order (copies of prefix blocks materialised).
    g = torch.Generator(device=device).manual_seed(5 + rank)
    dev_u = torch.randn(len(uniq) * size // 2, generator=g, device=device, dtype=torch.float16).view(torch.uint8)
    pos = torch.from_numpy(np.searchsorted(uniq, src)).to(device)
    host_u = torch.empty(n * size, dtype=torch.uint8, pin_memory=True)
    host_u.view(n, size).copy_(dev_u.view(len(uniq), size).index_select(0, pos))
    del dev_u
    torch.cuda.empty_cache()
    ptrs = (np.uint64(host_u.data_ptr()) + np.arange(n, dtype=np.uint64) * np.uint64(size)).astype(np.uint64)
    sizes = np.full(n, size, np.uint64)
    prefix = is_prefix.astype(np.uint8)
    out = torch.empty(args.batch * size, dtype=torch.uint8, pin_memory=True)
    store.clear()
    keys_ref = np.empty((n, 16), np.uint8)
    run_pass(store, ptrs, sizes, prefix, args.batch, out, size, 1, device_memory=False, keys_all=keys_ref)
    keys_step = np.empty_like(keys_ref)
    times, pb, gb = [], 0, 0
    for s in range(max(args.steps, 2)):
        store.clear()
        gk = plan_gets(keys_ref, 2 + s)
        gets = (gk, n_get_calls(gk, args.batch))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ps, gs, pb, gb = run_pass(store, ptrs, sizes, prefix, args.batch, out, size, 2 + s, device_memory=False,
                                  keys_all=keys_step, gets=gets)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    el = reduce_max(float(np.median(times)), world)
    tot = reduce_sum(pb + gb, world)
    store.clear()
    return {"value": round(tot / el / GB, 3), "unit": "GB/s", "h2d_bytes_per_step": int(pb + 16 * len(uniq)),
            "d2h_bytes_per_step": int(gb + 32 * n), "blocks": n,
            "note": f"pinned host buffers through batch_put/batch_get (put_ptrs/get_ptrs) on a {n}-block "
                    "slice of the stream (same block size and duplicate mix)"}


if __name__ == "__main__":
    main()
