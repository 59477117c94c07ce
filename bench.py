"""Decode hot-path benchmark (configuration 2 of the reference's headline).

One step = one decode step of the sparse-attention hot path for every request
of the rank: for each of the 32 layers, Quest page selection, the row
resolver, the host->pool miss gather and physical-row attention, for 16
requests per GPU (Llama-3-8B shape: 32 q / 8 KV heads, head_dim 128, bf16) at
32,768 tokens of context with 25% of the KV pages resident in the GPU pool and
the rest only in pinned host memory. Weak scaling: every rank decodes its own
16 requests (requests are independent; no collective on the data path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line on rank 0. `--impl reference` times the CPU restatement
of the reference's path (the oracle) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "nano-hisparse_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s at 32k ctx, 25% KV resident; miss-gather GB/s vs host-link peak"
# configuration 2
REQUESTS, LAYERS, CONTEXT = 16, 32, 32768
REQUESTS_DEFAULT = REQUESTS
Q_HEADS, KV_HEADS, HEAD_DIM, PAGE = 32, 8, 128, 16
TOP_PAGES = 2048 // PAGE          # Quest budget of 2048 tokens incl. sink and tail
HOT_ROWS = 2 * 2048               # reference default: 2 x max_union_rows
RESIDENT_FRACTION = 0.25
DTYPE = torch.bfloat16
MICRO = 2  # request groups pipelined on separate streams
TRANSFER = "shared"  # the micro-batches' gathers share one transfer stream
SETTLE_STEPS = 12  # untimed steps that fill the hot buffers before the warm-up steps
# PCIe read bytes per byte the gather stores into the pool: ncu's
# pcie__read_bytes.sum / l1tex__t_bytes_pipe_lsu_mem_global_op_st.sum on four
# gather launches of configuration 2 at one layer, 1.09375 on each
# (profiles/gather_kernel_config2_one_layer.md); the roofline traffic of a
# launch is this ratio times its bytes
PCIE_READ_PER_GATHERED_BYTE = 1.09375
HOST_STORE = {}  # size of the pinned host store actually allocated (set by build_workload)


def workload_config():
    reduced = REQUESTS != 16 or LAYERS != 32
    return {
        **({"reduced_for_profiling": True} if reduced else {}),
        "workload": "config 2: Llama-3-8B-shaped sparse decode hot path (Quest select, row "
                    "resolve, host->pool miss gather, row attention) for every layer",
        "requests_per_gpu": REQUESTS, "layers": LAYERS, "context": CONTEXT,
        "q_heads": Q_HEADS, "kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "page_size": PAGE,
        "quest_budget_tokens": TOP_PAGES * PAGE, "hot_rows": HOT_ROWS,
        "resident_fraction": RESIDENT_FRACTION, "kv_dtype": "bf16", "accumulate": "fp32",
        "queries": "N(0,1) per request, layer and step (seed 1)",
        "kv": "N(0,1) bf16, page min/max metadata from K (seed 1)",
        "l2": "inputs larger than L2 (about 12 GiB of metadata and KV rows read per step)",
        "parallelism": "requests sharded over ranks, no collective on the hot path",
        "microbatches": MICRO, "transfer_streams": TRANSFER,
        "settle_steps": SETTLE_STEPS,
        **({"host_store": HOST_STORE} if HOST_STORE else {}),
    }


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json)"
    return 6650.0, "fallback (6.65 TB/s)"


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock/throttle samples every 50 ms, kept for the timed window."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, None
        self.t0 = self.t1 = None

    def start(self):
        import tempfile

        # raw samples: HS_BENCH_LOG_DIR when set (to keep them), else a temp dir
        out = Path(os.environ.get("HS_BENCH_LOG_DIR", tempfile.gettempdir()))
        out.mkdir(parents=True, exist_ok=True)
        self.path = out / f"clocks_rank{self.index}.csv"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def wait_ready(self, timeout=10.0):
        """Block until the first sample is on disk (nvidia-smi takes a moment
        to start on a many-GPU box), so the timed window is covered."""
        deadline = time.time() + timeout
        while self.proc is not None and time.time() < deadline:
            if self.path.exists() and self.path.stat().st_size > 0:
                return
            time.sleep(0.05)

    def window(self, t0, t1):
        self.t0, self.t1 = t0, t1

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        if self.t1 is not None:  # a few samples past the window's end
            time.sleep(max(0.0, self.t1 + 0.15 - time.time()))
        self.proc.terminate()
        self.proc.wait(timeout=10)
        import datetime

        rows = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            when = None
            for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
                try:
                    when = datetime.datetime.strptime(parts[0], fmt).timestamp()
                    break
                except ValueError:
                    pass
            try:
                rows.append((when, float(parts[2]), float(parts[3]),
                             {n for n, f in zip(names, parts[6:10]) if f.lower().startswith("active")}))
            except ValueError:
                continue
        inside = [r for r in rows if self.t0 is not None and r[0] is not None
                  and self.t0 - 0.05 <= r[0] <= self.t1 + 0.05]
        chosen, where = (inside, "timed region") if len(inside) >= 2 else (rows, "whole run")
        reasons = set().union(*[r[3] for r in chosen]) if chosen else set()
        return {"sm_mhz": float(np.median([r[1] for r in chosen])) if chosen else None,
                "sm_max_mhz": max(r[2] for r in chosen) if chosen else None,
                "reasons": sorted(reasons), "samples": len(chosen), "window": where}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def available_host_bytes():
    """Host RAM this process may still use: MemAvailable, capped by the
    cgroup's limit when the container has one."""
    avail = None
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                avail = int(line.split()[1]) * 1024
    except OSError:
        pass
    for limit_file, usage_file in (("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory.current"),
                                   ("/sys/fs/cgroup/memory/memory.limit_in_bytes",
                                    "/sys/fs/cgroup/memory/memory.usage_in_bytes")):
        try:
            limit = Path(limit_file).read_text().strip()
            usage = int(Path(usage_file).read_text().strip())
        except (OSError, ValueError):
            continue
        if limit.isdigit() and int(limit) < (1 << 60):
            room = int(limit) - usage
            avail = room if avail is None else min(avail, room)
        break
    return avail


def host_store_pages(wanted_pages, page_bytes, log):
    """Distinct pinned host pages this rank allocates. The full store is
    REQUESTS x LAYERS x CONTEXT rows (64 GiB per rank for configuration 2);
    when all ranks of the node would not fit in half of the free host RAM, the
    (request, layer) units share a smaller store (unit pages wrap around it).
    The rows moved per step, and so the host-link bytes, are unchanged."""
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", os.environ.get("WORLD_SIZE", 1)))
    avail = available_host_bytes()
    if avail is None:
        return wanted_pages
    budget = avail // 2 // max(local_world, 1)
    pages = min(wanted_pages, budget // page_bytes)
    if pages < wanted_pages:
        log(f"host RAM: {avail / 2**30:.0f} GiB free for {local_world} rank(s); host store "
            f"shared by the units ({pages * page_bytes / 2**30:.1f} GiB per rank)")
    if pages < 4 * math.ceil(CONTEXT / PAGE):
        raise RuntimeError(f"not enough host RAM for the pinned host store "
                           f"({avail / 2**30:.1f} GiB free, {local_world} rank(s))")
    return pages


def build_workload(device, seed, log):
    from hisparse_b200 import CacheConfig, DecodeBatch, HotConfig, RowCache

    n = math.ceil(CONTEXT / PAGE)
    hot = HotConfig(TOP_PAGES * PAGE, HOT_ROWS)
    hot_blocks = hot.hot_blocks(PAGE)
    resident_pages = int(round(n * RESIDENT_FRACTION))
    units = REQUESTS * LAYERS
    page_bytes = 2 * PAGE * KV_HEADS * HEAD_DIM * 2
    host_pages = host_store_pages(units * n, page_bytes, log)
    HOST_STORE.update(gib_per_rank=round(host_pages * page_bytes / 2**30, 2),
                      shared_by_units=host_pages < units * n)
    config = CacheConfig(gpu_pages=units * (resident_pages + hot_blocks), host_pages=host_pages,
                         page_size=PAGE, kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                         device=str(device), dtype=DTYPE,
                         index_budget_bytes=1 << 40)
    t0 = time.time()
    host = torch.empty((config.host_pages, 2, PAGE, KV_HEADS, HEAD_DIM), dtype=DTYPE,
                       pin_memory=True)
    log(f"pinned host store {host.numel() * 2 / 2**30:.1f} GiB in {time.time() - t0:.1f}s")
    cache = RowCache(config, hot, host=host)
    gen = torch.Generator(device=device).manual_seed(seed)
    rng = np.random.default_rng(seed)
    mins = {r: torch.empty((LAYERS, n, KV_HEADS, HEAD_DIM), dtype=DTYPE, device=device)
            for r in range(REQUESTS)}
    maxs = {r: torch.empty_like(mins[r]) for r in range(REQUESTS)}
    block = 0
    t0 = time.time()
    for r in range(REQUESTS):
        for layer in range(LAYERS):
            base = ((r * LAYERS + layer) * n) % (host_pages - n + 1)
            kv = torch.randn((n, 2, PAGE, KV_HEADS, HEAD_DIM), generator=gen, device=device,
                             dtype=torch.float32).to(DTYPE)
            mins[r][layer] = kv[:, 0].amin(1)
            maxs[r][layer] = kv[:, 0].amax(1)
            host[base:base + n].copy_(kv, non_blocking=True)
            # 25% of the pages resident: the two tail pages plus a uniform sample
            chosen = rng.choice(n - 2, size=resident_pages - 2, replace=False)
            pages = np.sort(np.concatenate([chosen, [n - 2, n - 1]]))
            resident = np.full(n, -1, dtype=np.int64)
            resident[pages] = np.arange(block, block + resident_pages)
            idx = torch.from_numpy(pages).to(device)
            cache.pool[block:block + resident_pages] = kv.index_select(0, idx)
            block += resident_pages
            hot_list = list(range(block, block + hot_blocks))
            block += hot_blocks
            cache.add_layer(r, layer, CONTEXT, np.arange(base, base + n), resident, hot_list)
    torch.cuda.synchronize(device)
    log(f"generated KV, metadata and placement in {time.time() - t0:.1f}s")
    return cache, mins, maxs


def make_batches(cache, mins, maxs, micro, device):
    """`micro` decode batches over disjoint request groups, each with its own
    compute and transfer streams (micro-batch pipelining)."""
    from hisparse_b200 import DecodeBatch

    groups = [list(range(REQUESTS))[i::micro] for i in range(micro)]
    batches = []
    shared = torch.cuda.Stream(device=device)
    for g in groups:
        transfer = shared if TRANSFER == "shared" else torch.cuda.Stream(device=device)
        streams = (torch.cuda.Stream(device=device), transfer)
        with torch.cuda.stream(streams[0]):
            batches.append(DecodeBatch(cache, g, LAYERS, {r: mins[r] for r in g},
                                       {r: maxs[r] for r in g}, TOP_PAGES, Q_HEADS,
                                       streams=streams))
    torch.cuda.synchronize(device)
    return groups, batches


def bytes_per_unit(valid_rows, misses):
    """Algorithmic HBM bytes of one (request, layer): Quest metadata (min+max),
    K+V of every selected row, and the miss rows written into the pool."""
    row = 2 * KV_HEADS * HEAD_DIM * 2
    meta = 2 * math.ceil(CONTEXT / PAGE) * KV_HEADS * HEAD_DIM * 2
    return meta + valid_rows * row + misses * row


def hostlink_peak(device, sync=None):
    """Measured pinned host->device copy bandwidth (copy engine), GB/s: best of
    5 copies of 1 GiB; `sync` (a barrier over the ranks) runs before each copy
    so that concurrent measurements overlap."""
    nbytes = 1 << 30
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=device)
    best = float("inf")
    for _ in range(5):
        if sync is not None:
            sync()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize(device)
        best = min(best, a.elapsed_time(b))
    del src, dst
    return nbytes / best / 1e6


def hostlink_peaks(device, rank, world):
    """Host-link copy-engine bandwidth of this rank's GPU measured alone (the
    ranks take turns) and with every rank copying at once; with the sum of
    the concurrent rates over the ranks. One rank: the solo figure for all."""
    solo = hostlink_peak(device) if world == 1 else None
    if world == 1:
        return {"solo_gbs": solo, "concurrent_gbs": solo, "aggregate_concurrent_gbs": solo}
    import torch.distributed as dist

    def sync():
        torch.cuda.synchronize(device)
        dist.barrier()

    for r in range(world):
        sync()
        if r == rank:
            solo = hostlink_peak(device)
    sync()
    concurrent = hostlink_peak(device, sync)
    t = torch.tensor([concurrent], dtype=torch.float64, device=device)
    dist.all_reduce(t)
    return {"solo_gbs": solo, "concurrent_gbs": concurrent,
            "aggregate_concurrent_gbs": float(t.item())}


def run_gpu(args, rank, world, local_rank, log):
    import torch.distributed as dist

    from hisparse_b200 import _lib

    from hisparse_b200.sharding import bind_to_device_node

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    # pinned host store on the GPU's own NUMA node (first touch by these CPUs)
    local_cpus = bind_to_device_node(local_rank)
    HOST_STORE["numa_local_cpus"] = len(local_cpus) if local_cpus else None
    hbm_peak, hbm_source = measured_peaks()
    links = hostlink_peaks(device, rank, world)
    link_peak, link_concurrent = links["solo_gbs"], links["concurrent_gbs"]
    cache, mins, maxs = build_workload(device, 1 + rank, log)
    groups, batches = make_batches(cache, mins, maxs, args.microbatches, device)
    steps, warmup = args.steps, args.warmup
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    total = steps + warmup
    # fresh queries for every pass (timed graph steps, the eager per-stage pass,
    # the instrumented gather pass, the end-to-end steps): a repeated query would
    # find its rows already hot and gather less than a real step
    eager_base, roof_base, e2e_base = total, total + steps, 2 * total + steps
    settle_base = 3 * total + steps
    queries = torch.randn((3 * total + steps + SETTLE_STEPS, LAYERS, REQUESTS, Q_HEADS,
                           HEAD_DIM), generator=gen, device=device, dtype=torch.float32).to(DTYPE)
    counts = torch.zeros((total, LAYERS, REQUESTS, 3), dtype=torch.int64, device=device)
    compute = cache.compute

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    def max_over_ranks(value):
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from hisparse_b200.batched import DecodeGraph

    gq = [queries[:, :, g].contiguous() for g in groups]          # [sets, L, Bg, Hq, D]
    graph = DecodeGraph(batches, LAYERS)
    log("captured one decode step as a CUDA graph")

    def run_steps(first, last, g_=graph, base=0, out=counts):
        for s in range(first, last):
            for i in range(len(groups)):
                g_.queries[i].copy_(gq[i][base + s])
            g_.replay()
            for i, g in enumerate(groups):
                out[s, :, g] = g_.counts[i]

    # decode steady state: the hot buffers fill up (4096 rows a unit, ~440 misses
    # a step) before the W warm-up steps, as they are after the first dozen tokens
    settle = torch.zeros((SETTLE_STEPS, LAYERS, REQUESTS, 3), dtype=torch.int64, device=device)
    sampler = ClockSampler(local_rank)
    sampler.start()
    run_steps(0, SETTLE_STEPS, graph, settle_base, settle)
    run_steps(0, warmup)
    sampler.wait_ready()
    barrier()
    # ---- timed region: K steps, device-resident inputs ------------------------------
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    start.record(compute)
    run_steps(warmup, total)
    end.record(compute)
    barrier()
    sampler.window(wall0, time.time())
    clocks = sampler.stop()
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    timed_counts = counts[warmup:].cpu().numpy()  # [steps, L, B, 3]
    row_bytes = 2 * KV_HEADS * HEAD_DIM * 2

    # ---- gather roofline: the same step captured with CUDA events around every
    # gather launch (on the transfer stream it runs on), replayed W + K times on
    # fresh queries; the events hold the last step's 64 launch durations. (The
    # event nodes cost about 3% of a step, so the headline region above runs the
    # uninstrumented graph.)
    graph_t = DecodeGraph(batches, LAYERS, timing=("gather",))
    roof_counts = torch.zeros_like(counts)
    run_steps(0, warmup, graph_t, roof_base, roof_counts)
    barrier()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    r0.record(compute)
    run_steps(warmup, total, graph_t, roof_base, roof_counts)
    r1.record(compute)
    barrier()
    roof_step_ms = r0.elapsed_time(r1) / steps
    last = roof_counts[total - 1].cpu().numpy()
    nb = len(groups)
    live = []
    for idx, (_, a, b) in enumerate(graph_t.timing):
        layer, i = divmod(idx, nb)
        live.append((int(last[layer, groups[i], 2].sum()) * row_bytes, a, b))
    live_ms = [a.elapsed_time(b) for _, a, b in live]
    live_bytes = sum(x for x, _, _ in live)
    live_gbs = live_bytes / (sum(live_ms) * 1e-3) / 1e9
    spans = [(graph_t.timing[0][1].elapsed_time(a), graph_t.timing[0][1].elapsed_time(b))
             for _, a, b in live]
    for bt in batches:  # graph_t's warm-up leaves events the other graph must not wait on
        for st in bt.layers:
            st.ready = st.last_use = None

    # ---- per-stage device time: the same number of steps run eagerly, one stage
    # at a time (each micro-batch layer waits for the previous one, and its
    # ready-row attention for its gather), with CUDA events on each launch's
    # stream; a spin kernel ahead of every layer keeps the streams busy while the
    # host enqueues, so no host gap lands inside a measured span
    timing = []
    eager_counts = [torch.zeros((steps, LAYERS, len(g), 3), dtype=torch.int64, device=device)
                    for g in groups]
    ref = torch.cuda.Event(enable_timing=True)
    ref.record(compute)
    prev = ref
    for s in range(warmup, total):
        for layer in range(LAYERS):
            for i, bt in enumerate(batches):
                with torch.cuda.stream(bt.compute):
                    bt.compute.wait_event(prev)
                    torch.cuda._sleep(1_000_000)
                    bt.layer(layer, gq[i][eager_base + s - warmup, layer], graph.outputs[i][layer],
                             eager_counts[i][s - warmup, layer], timing, serial=True)
                    prev = torch.cuda.Event()
                    prev.record(bt.compute)
    for bt in batches:
        done = torch.cuda.Event()
        done.record(bt.compute)
        compute.wait_event(done)
    ref_end = torch.cuda.Event(enable_timing=True)
    ref_end.record(compute)
    barrier()
    for bt in batches:  # the eager pass leaves events the graph must not wait on
        for st in bt.layers:
            st.ready = st.last_use = None
    intervals = {}
    for name, a, b in timing:
        intervals.setdefault(name, []).append((ref.elapsed_time(a), ref.elapsed_time(b)))
    kernel_ms = {k: float(sum(e - s_ for s_, e in v)) for k, v in intervals.items()}
    launches = {k: len(v) for k, v in intervals.items()}

    def union_ms(spans):
        spans, total_ms, cur_s, cur_e = sorted(spans), 0.0, None, None
        for s_, e in spans:
            if cur_e is None or s_ > cur_e:
                if cur_e is not None:
                    total_ms += cur_e - cur_s
                cur_s, cur_e = s_, e
            else:
                cur_e = max(cur_e, e)
        return total_ms + ((cur_e - cur_s) if cur_e is not None else 0.0)

    gather_busy_ms = union_ms(intervals["gather"])
    misses = int(timed_counts[..., 2].sum())
    gather_bytes = misses * row_bytes
    # the eager pass runs its own queries: its miss bytes come from its own
    # resolver counts
    eager = np.concatenate([c.cpu().numpy() for c in eager_counts], axis=2)
    eager_gather_bytes = int(eager[..., 2].sum()) * row_bytes
    # micro-batches' gathers overlap on the one host link: the link's rate is
    # the bytes over the time any gather is running
    gather_gbs = eager_gather_bytes / (gather_busy_ms * 1e-3) / 1e9
    hbm_bytes = sum(bytes_per_unit(int(timed_counts[s, l, b].sum()), int(timed_counts[s, l, b, 2]))
                    for s in range(steps) for l in range(LAYERS) for b in range(REQUESTS))
    attend_ms = kernel_ms["attend_ready"] + kernel_ms["attend_gathered"]
    attend_bytes = int(eager.sum()) * row_bytes
    attend_gbs = attend_bytes / (attend_ms * 1e-3) / 1e9
    meta_bytes = steps * LAYERS * REQUESTS * 2 * math.ceil(CONTEXT / PAGE) * KV_HEADS * \
        HEAD_DIM * 2
    quest_gbs = meta_bytes / (kernel_ms["quest"] * 1e-3) / 1e9
    # the step's roofline takes the host link as it is when every rank copies
    t_roof = max(hbm_bytes / (hbm_peak * 1e9), gather_bytes / (link_concurrent * 1e9))
    step_frac = t_roof / (elapsed_ms * 1e-3)

    # ---- end to end: queries copied in from pinned host memory and outputs read
    # back every step, through the same captured step ------------------------------
    host_q = [g[e2e_base:].cpu().pin_memory() for g in gq]
    host_out = [torch.empty((total, *o.shape), dtype=DTYPE, pin_memory=True)
                for o in graph.outputs]
    e2e_counts = torch.zeros((total, LAYERS, REQUESTS, 3), dtype=torch.int64, device=device)

    def run_e2e(first, last):
        for s in range(first, last):
            for i in range(len(groups)):
                graph.queries[i].copy_(host_q[i][s], non_blocking=True)
            graph.replay()
            for i, g in enumerate(groups):
                host_out[i][s].copy_(graph.outputs[i], non_blocking=True)
                e2e_counts[s, :, g] = graph.counts[i]

    run_e2e(0, warmup)
    barrier()
    e2e_start = torch.cuda.Event(enable_timing=True)
    e2e_end = torch.cuda.Event(enable_timing=True)
    e2e_start.record(compute)
    run_e2e(warmup, total)
    e2e_end.record(compute)
    barrier()
    e2e_ms = max_over_ranks(e2e_start.elapsed_time(e2e_end))
    e2e_misses = int(e2e_counts[warmup:, ..., 2].sum().item())
    flags = _lib.device_flags(device)
    if flags:
        raise RuntimeError(f"device flags raised during the bench: {flags}")
    prof_ms = ref.elapsed_time(ref_end)

    tokens = REQUESTS * steps * world
    value = tokens / (elapsed_ms * 1e-3)
    io_bytes = LAYERS * REQUESTS * Q_HEADS * HEAD_DIM * 2
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(elapsed_ms / steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config(),
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": io_bytes,
                "miss_rows_per_unit": round(e2e_misses / (steps * LAYERS * REQUESTS), 1)},
        # per layer and micro-batch: quest, resolve, gather, two attention phases
        # and the merge (replayed from one CUDA graph per step)
        "gpu_launches": int(6 * LAYERS * steps * len(batches)),
        "roofline": {
            "kernel": "gather_kernel (host->pool miss gather)", "bound": "hostlink",
            "achieved": round(live_gbs, 2),
            "peak": round(link_peak, 2), "unit": "GB/s", "frac": round(live_gbs / link_peak, 4),
            "peak_source": "measured in bench.py: pinned host->device cudaMemcpyAsync, 1 GiB, "
                           "this GPU alone (hostlink: the same with every rank copying)",
            "traffic": round(PCIE_READ_PER_GATHERED_BYTE * live_bytes / len(live)),
            "traffic_definition": "PCIe read bytes per launch (ncu pcie__read_bytes.sum, scaled "
                                  "from a one-layer capture by the bytes gathered)",
            "achieved_definition": "miss rows x 4 KiB per launch / launch duration, CUDA events "
                                   "around each gather on its transfer stream, captured in an "
                                   "instrumented copy of the step graph replayed W+K steps "
                                   "after the headline region; the last step's launches",
            "instrumented_ms_per_step": round(roof_step_ms, 3),
            "bytes_per_launch": round(live_bytes / len(live)),
            "ms_per_launch": round(sum(live_ms) / len(live), 4),
            "launches_timed": len(live),
            "hostlink_busy_frac": round(union_ms(spans) / (max(e for _, e in spans) -
                                                           min(s_ for s_, _ in spans)), 4),
            "eager_pass_gbs": round(gather_gbs, 2),
        },
        "roofline_hbm": {
            "attend_kernels": {"achieved": round(attend_gbs, 1), "peak": hbm_peak,
                               "frac": round(attend_gbs / hbm_peak, 4), "unit": "GB/s",
                               "peak_source": hbm_source,
                               "note": "both attention phases, each timed alone",
                               "ms_per_launch": round(attend_ms / launches["attend_ready"], 4)},
            "quest_kernels": {"achieved": round(quest_gbs, 1), "peak": hbm_peak,
                              "frac": round(quest_gbs / hbm_peak, 4), "unit": "GB/s",
                              "peak_source": hbm_source,
                              "ms_per_launch": round(kernel_ms["quest"] / launches["quest"], 4)},
            "resolve_ms_per_launch": round(kernel_ms["resolve"] / launches["resolve"], 4),
        },
        "hostlink": {k: round(v, 2) for k, v in links.items()},
        "step_roofline": {
            "definition": "t_roof = max(HBM bytes / HBM peak, miss bytes / host-link peak "
                          "with every rank copying)",
            "hbm_bytes_per_step": int(hbm_bytes / steps),
            "hostlink_bytes_per_step": int(gather_bytes / steps), "t_roof_ms": round(
                t_roof * 1e3 / steps, 3), "frac": round(step_frac, 4)},
        "resolver": {"resident_hits": int(timed_counts[..., 0].sum()),
                     "hot_hits": int(timed_counts[..., 1].sum()), "misses": misses,
                     "miss_rows_per_unit": round(misses / (steps * LAYERS * REQUESTS), 1)},
        "kernel_ms_per_step": {k: round(v / steps, 3) for k, v in kernel_ms.items()},
        "kernel_ms_note": "per step, summed over micro-batches and layers; every stage timed "
                          "alone in an eager pass (in the captured step they overlap)",
        "clocks": clocks,
    }
    return result


# ---------------------------------------------------------------------------
# configuration 5: one 1M-token request, KV heads split over the ranks
# ---------------------------------------------------------------------------
C5 = {"layers": 28, "q_heads": 28, "kv_heads": 4, "head_dim": 128, "page_size": 64,
      "context": 1 << 20, "top_pages": 128, "resident_fraction": 0.10, "hot_rows": 16384}


def run_config5(args, rank, world, local_rank, log):
    """Decode of one 1,048,576-token request of a Qwen2.5-7B-shaped model (28
    layers, 28 query / 4 KV heads, page 64, 10 % resident) with its KV heads
    split over `world` ranks: per layer, each rank's partial Quest scores
    are all-gathered (NCCL) and every rank takes the same top-128 pages, then
    resolves, gathers and attends over its own head slice. Strong scaling:
    the request is the same at every N."""
    import torch.distributed as dist

    from hisparse_b200 import CacheConfig, DecodeBatch, HotConfig, RowCache
    from hisparse_b200.sharding import bind_to_device_node

    c = C5
    if c["kv_heads"] % world:
        raise SystemExit(f"configuration 5 splits {c['kv_heads']} KV heads: use 1, 2 or 4 GPUs")
    hkv, hq = c["kv_heads"] // world, c["q_heads"] // world
    L, P, D = c["layers"], c["page_size"], c["head_dim"]
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    bind_to_device_node(local_rank)
    hbm_peak, _ = measured_peaks()
    links = hostlink_peaks(device, rank, world)
    link_peak = links["concurrent_gbs"]  # every rank gathers at once
    n = c["context"] // P
    hot = HotConfig(c["top_pages"] * P, c["hot_rows"])
    hot_blocks = hot.hot_blocks(P)
    resident_pages = int(round(n * c["resident_fraction"]))
    page_bytes = 2 * P * hkv * D * 2
    host_pages = host_store_pages(L * n, page_bytes, log)
    config = CacheConfig(gpu_pages=L * (resident_pages + hot_blocks), host_pages=host_pages,
                         page_size=P, kv_heads=hkv, head_dim=D, device=str(device), dtype=DTYPE,
                         index_budget_bytes=1 << 40)
    host = torch.empty((host_pages, 2, P, hkv, D), dtype=DTYPE, pin_memory=True)
    cache = RowCache(config, hot, host=host)
    gen = torch.Generator(device=device).manual_seed(1 + rank)  # this rank's head slice
    rng = np.random.default_rng(5)  # placement: the same on every rank (replicated tables)
    mins = torch.empty((L, n, hkv, D), dtype=DTYPE, device=device)
    maxs = torch.empty_like(mins)
    block = 0
    for layer in range(L):
        base = (layer * n) % (host_pages - n + 1)
        for lo in range(0, n, 4096):
            kv = torch.randn((min(4096, n - lo), 2, P, hkv, D), generator=gen, device=device,
                             dtype=torch.float32).to(DTYPE)
            mins[layer, lo:lo + len(kv)] = kv[:, 0].amin(1)
            maxs[layer, lo:lo + len(kv)] = kv[:, 0].amax(1)
            host[base + lo:base + lo + len(kv)].copy_(kv, non_blocking=True)
        torch.cuda.synchronize(device)  # the host rows are read back below
        chosen = rng.choice(n - 2, size=resident_pages - 2, replace=False)
        pages = np.sort(np.concatenate([chosen, [n - 2, n - 1]]))
        resident = np.full(n, -1, dtype=np.int64)
        resident[pages] = np.arange(block, block + resident_pages)
        cache.pool[block:block + resident_pages] = host[torch.from_numpy(base + pages)].to(device)
        block += resident_pages
        hot_list = list(range(block, block + hot_blocks))
        block += hot_blocks
        cache.add_layer(0, layer, c["context"], np.arange(base, base + n), resident, hot_list)
    torch.cuda.synchronize(device)
    group = dist.group.WORLD if world > 1 else None
    streams = (torch.cuda.Stream(device=device), torch.cuda.Stream(device=device))
    batch = DecodeBatch(cache, [0], L, {0: mins}, {0: maxs}, c["top_pages"], hq, group=group,
                        streams=streams)
    steps, warmup, settle = args.steps, args.warmup, 2
    total = settle + warmup + steps
    qgen = torch.Generator(device=device).manual_seed(1000 + rank)
    queries = torch.randn((total, L, 1, hq, D), generator=qgen, device=device,
                          dtype=torch.float32).to(DTYPE)
    counts = torch.zeros((total, L, 1, 3), dtype=torch.int64, device=device)
    out = torch.empty((1, hq, D), dtype=DTYPE, device=device)

    def run(first, last):
        with torch.cuda.stream(batch.compute):
            for s_ in range(first, last):
                for layer in range(L):
                    batch.layer(layer, queries[s_, layer], out, counts[s_, layer])

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    run(0, settle + warmup)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(batch.compute)
    run(settle + warmup, total)
    end.record(batch.compute)
    barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    timed = counts[settle + warmup:].cpu().numpy()
    # the same kind of steps replayed from captured graphs: one graph per step
    # at N = 1; with a group, two per layer with the all-gather issued between
    # them (no collective is captured)
    from hisparse_b200.batched import DecodeGraph

    graph = DecodeGraph([batch], L)
    gq = torch.randn((warmup + steps, L, 1, hq, D), generator=qgen, device=device,
                     dtype=torch.float32).to(DTYPE)
    for s_ in range(warmup):
        graph.queries[0].copy_(gq[s_])
        graph.replay()
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for s_ in range(warmup, warmup + steps):
        graph.queries[0].copy_(gq[s_])
        graph.replay()
    g1.record()
    barrier()
    graph_ms = g0.elapsed_time(g1)
    if world > 1:
        t = torch.tensor([graph_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        graph_ms = float(t.item())
    segmented = graph.segmented
    for st in batch.layers:
        st.ready = st.last_use = None
    del graph
    # the headline is the graph replay (the eager loop is bound by the host's
    # launch rate once the step is short); the eager loop is reported beside it
    eager_ms, ms = ms, graph_ms
    # per-stage device time: one more step, each stage alone (CUDA events on its stream)
    timing = []
    extra = torch.randn((L, 1, hq, D), generator=qgen, device=device,
                        dtype=torch.float32).to(DTYPE)
    with torch.cuda.stream(batch.compute):
        for layer in range(L):
            torch.cuda._sleep(1_000_000)
            batch.layer(layer, extra[layer], out, None, timing, serial=True)
    barrier()
    stage_ms = {}
    for name, a_, b_ in timing:
        stage_ms[name] = stage_ms.get(name, 0.0) + a_.elapsed_time(b_)
    row_bytes = 2 * hkv * D * 2
    misses = int(timed[..., 2].sum())
    hostlink_bytes = misses * row_bytes / steps
    selected = int(timed.sum()) / steps
    hbm_bytes = L * 2 * n * hkv * D * 2 + selected * row_bytes + hostlink_bytes
    t_roof = max(hbm_bytes / (hbm_peak * 1e9), hostlink_bytes / (link_peak * 1e9))
    flags = __import__("hisparse_b200")._lib.device_flags(device)
    if flags:
        raise RuntimeError(f"device flags raised: {flags}")
    return {
        "metric": "decode tok/s, one 1M-token request, KV heads split over the GPUs",
        "value": round(steps / (ms * 1e-3), 2), "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms / steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config 5: Qwen2.5-7B-shaped decode of one 1M-token request, "
                               "KV heads sharded, per-layer all-gather of partial Quest scores",
                   **c, "kv_heads_per_rank": hkv, "q_heads_per_rank": hq,
                   "host_store_gib_per_rank": round(host_pages * page_bytes / 2**30, 2)},
        "exchange_bytes_per_layer": 4 * n * world,
        "stage_ms_per_step": {k: round(v, 3) for k, v in stage_ms.items()},
        "timed": ("CUDA graphs, two per layer, the NCCL all-gather issued between them"
                  if segmented else "CUDA graph replay of each step"),
        "eager_tok_s": round(steps / (eager_ms * 1e-3), 2),
        "stage_note": "one extra step, every stage timed alone; quest includes the all-gather",
        "per_rank": {"miss_rows_per_layer": round(misses / (steps * L), 1),
                     "hostlink_bytes_per_step": int(hostlink_bytes),
                     "hbm_bytes_per_step": int(hbm_bytes),
                     "gather_gbs_avg": round(hostlink_bytes / (ms / steps * 1e-3) / 1e9, 2),
                     "hostlink_peak_gbs": round(link_peak, 2),
                     "hostlink": {k: round(v, 2) for k, v in links.items()},
                     "t_roof_ms": round(t_roof * 1e3, 3),
                     "step_roofline_frac": round(t_roof / (ms / steps * 1e-3), 4)},
    }


# ---------------------------------------------------------------------------
# configuration 4: 256 requests of lognormal lengths sharded over the ranks
# ---------------------------------------------------------------------------
C4 = {"requests": 256, "median_context": 16384, "min_context": 4096, "max_context": 131072,
      "sigma": 0.8, "decode_steps": 512, "seed": 4}


def config4_lengths():
    """The 256 requests' context lengths: lognormal (median 16k, sigma 0.8),
    clipped to [4k, 128k], seeded; the same on every rank."""
    rng = np.random.default_rng(C4["seed"])
    raw = rng.lognormal(math.log(C4["median_context"]), C4["sigma"], C4["requests"])
    return np.clip(raw, C4["min_context"], C4["max_context"]).astype(np.int64)


def config4_pool_gib(lengths):
    """Device pool one rank needs for its requests (25 % resident + hot blocks)."""
    hot_blocks = math.ceil(HOT_ROWS / PAGE)
    pages = sum(int(round(math.ceil(int(n) / PAGE) * RESIDENT_FRACTION)) + hot_blocks
                for n in lengths)
    return pages * LAYERS * 2 * PAGE * KV_HEADS * HEAD_DIM * 2 / 2**30


def run_config4(args, rank, world, local_rank, log):
    """Configuration-2 model shape serving 256 requests of lognormal lengths:
    rank r decodes requests r, r + N, ... (no collective on the hot path), each
    with its own tables, 25 % of its pages resident; two micro-batches per rank
    as in configuration 2. A step decodes one token of every request of every
    rank; the timed steps are K of the configuration's 512 (the per-step work
    does not depend on the step's index beyond the hot-buffer warm-up)."""
    from hisparse_b200 import CacheConfig, DecodeBatch, HotConfig, RowCache, _lib
    from hisparse_b200.batched import DecodeGraph
    from hisparse_b200.sharding import bind_to_device_node
    import torch.distributed as dist

    lengths_all = config4_lengths()
    mine = lengths_all[rank::world]
    reduced = args.requests != REQUESTS_DEFAULT
    if reduced:  # a rank's first requests only: for functional checks and captures
        mine = mine[:args.requests]
    ids = list(range(len(mine)))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    bind_to_device_node(local_rank)
    need = config4_pool_gib(mine)
    free = torch.cuda.mem_get_info(device)[0] / 2**30
    base = {"metric": "decode tok/s, 256 requests of lognormal lengths (median 16k)",
            "unit": "tok/s", "n_gpus": world, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 4: 256 requests sharded over the ranks, lognormal "
                                   "lengths, configuration-2 model shape",
                       **({"reduced_for_profiling": True} if reduced else {}), **C4,
                       "requests_per_rank": len(mine), "pool_gib_per_rank": round(need, 1)}}
    fits = need + 12 < free
    if world > 1:  # every rank decides the same way
        t = torch.tensor([1.0 if fits else 0.0], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        fits = bool(t.item())
    if not fits:
        return {**base, "value": None,
                "unavailable": f"the pool of {len(mine)} requests per GPU needs {need:.0f} GiB "
                               f"(25 % resident) with {free:.0f} GiB free: use 4 or more GPUs"}
    hbm_peak, _ = measured_peaks()
    links = hostlink_peaks(device, rank, world)
    hot = HotConfig(TOP_PAGES * PAGE, HOT_ROWS)
    hot_blocks = hot.hot_blocks(PAGE)
    pages_of = [math.ceil(int(n) / PAGE) for n in mine]
    units_pages = sum(pages_of) * LAYERS
    page_bytes = 2 * PAGE * KV_HEADS * HEAD_DIM * 2
    host_pages = host_store_pages(units_pages, page_bytes, log)
    res_of = [int(round(n * RESIDENT_FRACTION)) for n in pages_of]
    config = CacheConfig(gpu_pages=LAYERS * sum(r_ + hot_blocks for r_ in res_of),
                         host_pages=host_pages, page_size=PAGE, kv_heads=KV_HEADS,
                         head_dim=HEAD_DIM, device=str(device), dtype=DTYPE,
                         index_budget_bytes=1 << 40)
    host = torch.empty((host_pages, 2, PAGE, KV_HEADS, HEAD_DIM), dtype=DTYPE, pin_memory=True)
    cache = RowCache(config, hot, host=host)
    gen = torch.Generator(device=device).manual_seed(40 + rank)
    rng = np.random.default_rng(40 + rank)
    mins = {r: [] for r in ids}
    maxs = {r: [] for r in ids}
    block, offset = 0, 0
    t0 = time.time()
    for r in ids:
        n, k = pages_of[r], res_of[r]
        for layer in range(LAYERS):
            hb = offset % (host_pages - n + 1)
            offset += n
            kv = torch.randn((n, 2, PAGE, KV_HEADS, HEAD_DIM), generator=gen, device=device,
                             dtype=torch.float32).to(DTYPE)
            mins[r].append(kv[:, 0].amin(1))
            maxs[r].append(kv[:, 0].amax(1))
            host[hb:hb + n].copy_(kv, non_blocking=True)
            chosen = rng.choice(n - 2, size=k - 2, replace=False)
            pages = np.sort(np.concatenate([chosen, [n - 2, n - 1]]))
            resident = np.full(n, -1, dtype=np.int64)
            resident[pages] = np.arange(block, block + k)
            cache.pool[block:block + k] = kv.index_select(0, torch.from_numpy(pages).to(device))
            block += k
            hot_list = list(range(block, block + hot_blocks))
            block += hot_blocks
            cache.add_layer(r, layer, int(mine[r]), np.arange(hb, hb + n), resident, hot_list)
        mins[r] = torch.stack(mins[r])
        maxs[r] = torch.stack(maxs[r])
        torch.cuda.synchronize(device)
    log(f"config4: {len(mine)} requests per rank built in {time.time() - t0:.1f}s")
    groups = [ids[i::2] for i in range(2)]
    shared = torch.cuda.Stream(device=device)
    batches = []
    for g in groups:
        streams = (torch.cuda.Stream(device=device), shared)
        with torch.cuda.stream(streams[0]):
            batches.append(DecodeBatch(cache, g, LAYERS, {r: mins[r] for r in g},
                                       {r: maxs[r] for r in g}, TOP_PAGES, Q_HEADS,
                                       streams=streams))
    torch.cuda.synchronize(device)
    graph = DecodeGraph(batches, LAYERS)
    steps, warmup = args.steps, args.warmup
    total = SETTLE_STEPS + warmup + steps
    qgen = torch.Generator(device=device).manual_seed(400 + rank)
    queries = [torch.randn((total, LAYERS, len(g), Q_HEADS, HEAD_DIM), generator=qgen,
                           device=device, dtype=torch.float32).to(DTYPE) for g in groups]
    counts = torch.zeros((total, LAYERS, len(ids), 3), dtype=torch.int64, device=device)

    def run(first, last):
        for s_ in range(first, last):
            for i in range(len(groups)):
                graph.queries[i].copy_(queries[i][s_])
            graph.replay()
            for i, g in enumerate(groups):
                counts[s_, :, g] = graph.counts[i]

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    run(0, SETTLE_STEPS + warmup)
    barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    sampler.wait_ready()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    a.record(cache.compute)
    run(SETTLE_STEPS + warmup, total)
    b_.record(cache.compute)
    barrier()
    sampler.window(wall0, time.time())
    clocks = sampler.stop()
    ms = a.elapsed_time(b_)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flags = _lib.device_flags(device)
    if flags:
        raise RuntimeError(f"device flags raised: {flags}")
    timed = counts[SETTLE_STEPS + warmup:].cpu().numpy()
    row_bytes = 2 * KV_HEADS * HEAD_DIM * 2
    misses = int(timed[..., 2].sum())
    meta = sum(2 * n * KV_HEADS * HEAD_DIM * 2 for n in pages_of) * LAYERS * steps
    hbm = meta + (int(timed.sum()) + misses) * row_bytes
    hostb = misses * row_bytes
    t_roof = max(hbm / (hbm_peak * 1e9), hostb / (links["concurrent_gbs"] * 1e9))
    sums = torch.tensor([len(ids) * steps, misses, hbm, hostb], dtype=torch.float64,
                        device=device)
    if world > 1:
        dist.all_reduce(sums)
    tokens = float(sums[0].item())
    return {**base, "value": round(tokens / (ms * 1e-3), 2), "steps": steps, "warmup": warmup,
            "ms_per_step": round(ms / steps, 3), "clocks": clocks,
            "hostlink": {k_: round(v, 2) for k_, v in links.items()},
            "per_rank": {"requests": len(ids), "context_tokens": int(sum(int(n) for n in mine)),
                         "miss_rows_per_unit": round(misses / (steps * LAYERS * len(ids)), 1),
                         "hbm_bytes_per_step": int(hbm / steps),
                         "hostlink_bytes_per_step": int(hostb / steps),
                         "step_roofline_frac": round(t_roof / (ms * 1e-3), 4)}}


# ---------------------------------------------------------------------------
# configuration 3: isolated decode attention, resident-fraction sweep
# ---------------------------------------------------------------------------
C3 = {"requests": 64, "q_heads": 32, "kv_heads": 8, "head_dim": 128, "context": 131072,
      "page_sizes": (16, 64), "rows": 4096, "resident_fractions": (0.10, 0.25, 0.50, 0.90),
      "hot_rows": 8192, "trace_steps": 64, "settle_steps": 16, "overlap": 0.70, "seed": 2}


def lru_trace(rng, pages, chosen, steps, overlap):
    """Selected pages of `steps` decode steps of one query: step 0 draws
    `chosen` pages uniformly; every later step keeps `overlap` of the previous
    step's pages (a uniform subset) and draws the rest uniformly from the
    pages not kept."""
    keep = int(round(chosen * overlap))
    cur = np.sort(rng.choice(pages, size=chosen, replace=False))
    out = [cur]
    for _ in range(1, steps):
        kept = rng.choice(cur, size=keep, replace=False)
        mask = np.ones(pages, dtype=bool)
        mask[kept] = False
        fresh = rng.choice(np.flatnonzero(mask), size=chosen - keep, replace=False)
        cur = np.sort(np.concatenate([kept, fresh]))
        out.append(cur)
    return out


def run_config3(args, rank, world, local_rank, log):
    """Decode attention of 64 queries over 4,096 selected rows each at 131,072
    tokens of context (32 q / 8 KV heads, bf16), page sizes 16 and 64, with 10,
    25, 50 and 90 % of each request's pages resident in the pool and the rest
    only in pinned host memory. Each query's selection follows a 64-step trace
    whose steps keep 70 % of the previous step's pages; the hot buffer (8,192
    rows per request) is filled by the first 16 steps, the other 48 are timed.
    A step resolves, gathers and attends every query (one DecodeBatch layer
    over the trace's positions); Quest scoring of the same requests' metadata
    is timed beside it."""
    from hisparse_b200 import CacheConfig, DecodeBatch, HotConfig, RowCache, _lib
    from hisparse_b200.sharding import bind_to_device_node

    c = dict(C3)
    if args.requests != REQUESTS_DEFAULT:  # fewer queries: for ncu captures only
        c["requests"] = args.requests
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    bind_to_device_node(local_rank)
    hbm_peak, hbm_source = measured_peaks()
    link_peak = hostlink_peak(device)
    B, HQ, HKV, D, T = c["requests"], c["q_heads"], c["kv_heads"], c["head_dim"], c["context"]
    row_bytes = 2 * HKV * D * 2
    steps_total, settle = c["trace_steps"], c["settle_steps"]
    timed_steps = steps_total - settle
    lines = []
    for P in c["page_sizes"]:
        n = T // P
        chosen = c["rows"] // P
        hot = HotConfig(c["rows"], c["hot_rows"])
        hot_blocks = hot.hot_blocks(P)
        page_bytes = 2 * P * HKV * D * 2
        host_pages = host_store_pages(B * n, page_bytes, log)
        top_res = int(round(n * max(c["resident_fractions"])))
        config = CacheConfig(gpu_pages=B * (top_res + hot_blocks), host_pages=host_pages,
                             page_size=P, kv_heads=HKV, head_dim=D, device=str(device),
                             dtype=DTYPE, index_budget_bytes=1 << 40)
        t0 = time.time()
        host = torch.empty((host_pages, 2, P, HKV, D), dtype=DTYPE, pin_memory=True)
        cache = RowCache(config, hot, host=host)
        gen = torch.Generator(device=device).manual_seed(c["seed"])
        rng = np.random.default_rng(c["seed"])
        mins, maxs, order, bases = {}, {}, {}, {}
        block = 0
        for r in range(B):
            base = (r * n) % (host_pages - n + 1)
            bases[r] = base
            kv = torch.randn((n, 2, P, HKV, D), generator=gen, device=device,
                             dtype=torch.float32).to(DTYPE)
            mins[r] = kv[:, 0].amin(1)[None].contiguous()
            maxs[r] = kv[:, 0].amax(1)[None].contiguous()
            host[base:base + n].copy_(kv, non_blocking=True)
            # residency: the first f*n pages of one permutation are resident at
            # fraction f (nested sets); the pool holds the largest set
            perm = rng.permutation(n)
            order[r] = perm
            idx = torch.from_numpy(np.sort(perm[:top_res])).to(device)
            res_blocks = block + torch.arange(top_res, device=device)
            cache.pool[res_blocks] = kv.index_select(0, idx)
            block += top_res
            hot_list = list(range(block, block + hot_blocks))
            block += hot_blocks
            cache.add_layer(r, 0, T, np.arange(base, base + n), np.full(n, -1), hot_list)
            torch.cuda.synchronize(device)
        log(f"config3 P{P}: KV, metadata and pool placement in {time.time() - t0:.1f}s")
        # pool block of page p at the largest fraction (its rank in the sorted prefix)
        block_of = {}
        for r in range(B):
            top = np.sort(order[r][:top_res])
            base_block = r * (top_res + hot_blocks)
            blk = np.full(n, -1, dtype=np.int64)
            blk[top] = base_block + np.arange(top_res)
            block_of[r] = blk
        traces = [lru_trace(rng, n, chosen, steps_total, c["overlap"]) for _ in range(B)]
        offs = np.arange(P, dtype=np.int32)
        positions = torch.from_numpy(np.stack([
            np.stack([(tr[s][:, None] * P + offs).reshape(-1).astype(np.int32)
                      for tr in traces]) for s in range(steps_total)])).to(device)
        qgen = torch.Generator(device=device).manual_seed(c["seed"] + 1)
        queries = torch.randn((steps_total, B, HQ, D), generator=qgen, device=device,
                              dtype=torch.float32).to(DTYPE)
        streams = (torch.cuda.Stream(device=device), torch.cuda.Stream(device=device))
        with torch.cuda.stream(streams[0]):
            batch = DecodeBatch(cache, list(range(B)), 1, mins, maxs, chosen, HQ,
                                streams=streams)
        torch.cuda.synchronize(device)
        # Quest scoring + top-k of the same 64 requests, timed alone
        lib = _lib.load()
        st0 = batch.layers[0]
        qws = batch.quest_ws
        q_events = []
        with torch.cuda.stream(batch.compute):
            for s_ in range(8):
                a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                _lib.check(lib.hs_quest_select_batched(
                    B, queries[s_].data_ptr(), HQ * D, _lib.HS_BFLOAT16, st0.min_ptrs.data_ptr(),
                    st0.max_ptrs.data_ptr(), _lib.HS_BFLOAT16, st0.lengths.data_ptr(), HQ, HKV,
                    D, batch.max_pages, P, chosen, 1, batch.tokens.data_ptr(), batch.width,
                    batch.token_counts.data_ptr(), _lib.ptr(qws), batch.quest_ws_bytes,
                    batch.status.data_ptr(), batch.compute.cuda_stream))
                b_.record()
                q_events.append((a, b_))
        torch.cuda.synchronize(device)
        quest_ms = float(np.median([a.elapsed_time(b_) for a, b_ in q_events[2:]]))
        quest_bytes = B * 2 * n * HKV * D * 2
        out = torch.empty((B, HQ, D), dtype=DTYPE, device=device)
        counts = torch.zeros((steps_total, B, 3), dtype=torch.int64, device=device)
        for frac in c["resident_fractions"]:
            k = int(round(n * frac))
            for r in range(B):
                res = np.full(n, -1, dtype=np.int64)
                pages = order[r][:k]
                res[pages] = block_of[r][pages]
                t_ = cache.tables[r, 0]
                t_.resident.copy_(torch.from_numpy(res.astype(np.int32)))
                t_.tags.fill_(-1)
                t_.lru.copy_(torch.arange(c["hot_rows"], dtype=torch.int64))
            for st in batch.layers:
                st.ready = st.last_use = None
            torch.cuda.synchronize(device)
            events = []
            with torch.cuda.stream(batch.compute):
                for s_ in range(steps_total):
                    if s_ >= settle:
                        a = torch.cuda.Event(enable_timing=True)
                        a.record()
                    batch.layer(0, queries[s_], out, counts[s_], positions=positions[s_])
                    if s_ >= settle:
                        b_ = torch.cuda.Event(enable_timing=True)
                        b_.record()
                        events.append((a, b_))
            torch.cuda.synchronize(device)
            span_ms = events[0][0].elapsed_time(events[-1][1])
            # per-stage device time: one more trace step, each stage alone
            timing = []
            with torch.cuda.stream(batch.compute):
                torch.cuda._sleep(1_000_000)
                batch.layer(0, queries[steps_total - 1], out, None, timing, serial=True,
                            positions=positions[steps_total - 1])
            torch.cuda.synchronize(device)
            stage = {}
            for name, a, b_ in timing:
                stage[name] = stage.get(name, 0.0) + a.elapsed_time(b_)
            cnt = counts[settle:].sum(dim=(0, 1)).cpu().numpy()  # resident, hot, miss
            per_step = cnt / timed_steps
            sel_rows = float(per_step.sum())
            misses = float(per_step[2])
            hbm = (sel_rows + misses) * row_bytes  # KV rows read, miss rows written
            hostb = misses * row_bytes
            ms = span_ms / timed_steps
            t_roof = max(hbm / (hbm_peak * 1e9), hostb / (link_peak * 1e9))
            attend_ms = stage.get("attend_ready", 0.0) + stage.get("attend_gathered", 0.0)
            gather_ms = stage.get("gather", 0.0)
            lines.append({
                "page_size": P, "resident_fraction": frac,
                "queries_per_s": round(B / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
                "rows_per_query": {"resident": round(per_step[0] / B, 1),
                                   "hot": round(per_step[1] / B, 1),
                                   "miss": round(per_step[2] / B, 1)},
                "hbm_bytes_per_step": int(hbm), "hostlink_bytes_per_step": int(hostb),
                "step_roofline": {"t_roof_ms": round(t_roof * 1e3, 4),
                                  "frac": round(t_roof / (ms * 1e-3), 4),
                                  "bound": "hbm" if hbm / hbm_peak > hostb / link_peak
                                  else "hostlink"},
                "stage_ms": {k_: round(v, 4) for k_, v in stage.items()},
                "attend_gbs": round(sel_rows * row_bytes / (attend_ms * 1e-3) / 1e9, 1)
                if attend_ms > 0 else None,
                "gather_gbs": round(hostb / (gather_ms * 1e-3) / 1e9, 2) if gather_ms > 0
                else None,
            })
            log(f"config3 P{P} resident {frac:.2f}: {ms:.3f} ms/step, "
                f"roofline {t_roof / (ms * 1e-3):.3f}")
        lines_quest = {"page_size": P, "ms_per_launch": round(quest_ms, 4),
                       "bytes_per_launch": quest_bytes,
                       "achieved_gbs": round(quest_bytes / (quest_ms * 1e-3) / 1e9, 1),
                       "frac_of_hbm": round(quest_bytes / (quest_ms * 1e-3) / 1e9 / hbm_peak, 4)}
        lines.append({"page_size": P, "quest": lines_quest})
        flags = _lib.device_flags(device)
        if flags:
            raise RuntimeError(f"device flags raised: {flags}")
        del batch, cache, host, mins, maxs, positions, queries
        torch.cuda.empty_cache()
    sweep = [x for x in lines if "quest" not in x]
    quest = [x["quest"] for x in lines if "quest" in x]
    # headline: the HBM-bound corner (page 64, 90 % resident)
    head = [x for x in sweep if x["page_size"] == 64 and x["resident_fraction"] == 0.9][0]
    return {
        "metric": "decode-attention queries/s (64 queries x 4096 rows, 131072 ctx)",
        "value": head["queries_per_s"], "unit": "queries/s", "n_gpus": world,
        "steps": timed_steps, "warmup": settle, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "config 3: isolated decode attention (resolve, miss gather, "
                               "two-phase row attention, merge) over a 64-step LRU trace, "
                               "resident fraction and page size swept",
                   **({"reduced_for_profiling": True} if c["requests"] != C3["requests"]
                      else {}),
                   **{k: v for k, v in c.items()}},
        "headline_point": {"page_size": 64, "resident_fraction": 0.9},
        "hbm_peak": {"gbs": hbm_peak, "source": hbm_source},
        "hostlink_peak_gbs": round(link_peak, 2),
        "sweep": sweep, "quest": quest,
    }


# ---------------------------------------------------------------------------
# CPU arm (oracle restatement of the reference's path)
# ---------------------------------------------------------------------------
def cpu_sample(seed=1, budget_s=10.0, threads=None, log=print):
    """Times oracle.decode_layer_batched — the whole per-(request, layer) hot
    path, OpenMP over the 16 requests — on the host cores for one layer at a
    time, and extrapolates to tok/s over 32 layers."""
    import oracle

    threads = threads or os.cpu_count() or 1
    n = math.ceil(CONTEXT / PAGE)
    hot_blocks = math.ceil(HOT_ROWS / PAGE)
    resident_pages = int(round(n * RESIDENT_FRACTION))
    rng = np.random.default_rng(seed)
    t0 = time.time()
    host = torch.empty((REQUESTS * n, 2, PAGE, KV_HEADS, HEAD_DIM), dtype=DTYPE)

    def fill(r):  # one request's pages per task; torch releases the GIL
        gen = torch.Generator().manual_seed(seed * 1000 + r)
        host[r * n:(r + 1) * n] = torch.randn(host[r * n:(r + 1) * n].shape, generator=gen)

    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=threads) as pool_exec:
        list(pool_exec.map(fill, range(REQUESTS)))
    pool = torch.zeros((REQUESTS * (resident_pages + hot_blocks), 2, PAGE, KV_HEADS, HEAD_DIM),
                       dtype=DTYPE)
    queries, mins, maxs, sources, residents, hots, tags, lrus = ([] for _ in range(8))
    block = 0
    for r in range(REQUESTS):
        base = r * n
        keys = host[base:base + n, 0].float()
        mins.append(keys.amin(1).to(DTYPE))
        maxs.append(keys.amax(1).to(DTYPE))
        chosen = rng.choice(n - 2, size=resident_pages - 2, replace=False)
        pages = np.sort(np.concatenate([chosen, [n - 2, n - 1]]))
        resident = np.full(n, -1, dtype=np.int64)
        resident[pages] = np.arange(block, block + resident_pages)
        pool[block:block + resident_pages] = host[base + pages]
        block += resident_pages
        hots.append(np.arange(block, block + hot_blocks, dtype=np.int64))
        block += hot_blocks
        sources.append(np.arange(base, base + n, dtype=np.int64))
        residents.append(resident)
        tags.append(np.full(HOT_ROWS, -1, dtype=np.int64))
        lrus.append(np.arange(HOT_ROWS, dtype=np.int64))
    log(f"cpu sample data in {time.time() - t0:.1f}s")
    host_np = host.view(torch.int16).numpy()
    pool_np = pool.view(torch.int16).numpy()
    times = []
    t_start = time.time()
    it = 0
    while it < 2 or (time.time() - t_start < budget_s and it < 64):
        qgen = torch.Generator().manual_seed(seed * 7919 + it)
        qs = [torch.randn((Q_HEADS, HEAD_DIM), generator=qgen).to(DTYPE) for _ in range(REQUESTS)]
        a = time.perf_counter()
        oracle.decode_layer_batched(qs, mins, maxs, [CONTEXT] * REQUESTS, PAGE, TOP_PAGES, n,
                                    sources, residents, hots, tags, lrus, host_np, pool_np,
                                    threads=threads)
        times.append(time.perf_counter() - a)
        it += 1
    per_layer = float(np.mean(times[1:])) if len(times) > 1 else times[0]
    value = REQUESTS / (per_layer * LAYERS)
    return {
        "value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
        "sample": f"{len(times)} layer passes of {REQUESTS} requests (first untimed warm-up), "
                  f"{per_layer * 1e3:.1f} ms per layer, extrapolated x{LAYERS} layers; oracle "
                  "restatement in C (OpenMP over requests; fp64 attention)",
        "note": "a C port of the reference's per-layer path, batched over the requests, not "
                "the reference's own torch code: the reference is Python and does not travel "
                "to the GPU box, and its torch CPU path (one request at a time) is slower still",
    }


def main():
    global REQUESTS, LAYERS, MICRO, TRANSFER
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="hisparse_b200", choices=["hisparse_b200", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-config5", action="store_true",
                        help="at 2 or 4 GPUs, skip the configuration-5 sub-line")
    parser.add_argument("--microbatches", type=int, default=2,
                        help="independent request groups pipelined on separate streams")
    # Smaller request/layer counts are for ncu captures only; the bench line of
    # configuration 2 uses the defaults.
    parser.add_argument("--transfer", choices=["shared", "separate"], default=TRANSFER,
                        help="one transfer stream for all micro-batches (gathers take the "
                             "host link in turn) or one each")
    parser.add_argument("--workload", choices=["config2", "config3", "config4", "config5"],
                        default="config2",
                        help="config2 (the bench line), config3 (isolated decode attention, "
                             "resident-fraction sweep), config4 (256 requests sharded over the "
                             "GPUs) or config5 (one 1M-token request, KV heads split over 1, 2 "
                             "or 4 GPUs)")
    parser.add_argument("--requests", type=int, default=REQUESTS)
    parser.add_argument("--layers", type=int, default=LAYERS)
    args = parser.parse_args()
    REQUESTS, LAYERS, MICRO = args.requests, args.layers, args.microbatches
    TRANSFER = args.transfer
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    def log(msg):
        if rank == 0:
            print(f"[bench] {msg}", file=sys.stderr, flush=True)

    if args.impl == "reference":
        if rank != 0:
            return
        base = cpu_sample(log=log)
        line = {"metric": METRIC, "value": base["value"], "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": workload_config(), "impl": "reference", "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime

        import torch.distributed as dist

        # stdout carries exactly one JSON line: NCCL's own messages go to stderr
        os.environ["NCCL_DEBUG"] = "WARN"
        os.environ["NCCL_DEBUG_FILE"] = "/dev/stderr"

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        all_cpus = os.sched_getaffinity(0)
        if args.workload in ("config3", "config4", "config5"):
            run = {"config3": run_config3, "config4": run_config4,
                   "config5": run_config5}[args.workload]
            result = run(args, rank, world, local_rank, log)
            if rank == 0:
                print(json.dumps(result), flush=True)
            return
        result = run_gpu(args, rank, world, local_rank, log)
        if world in (2, 4) and not args.no_config5:
            # configuration 5 (one 1M-token request, its KV heads split over these
            # ranks) measured after the configuration-2 line, with that workload's
            # device and pinned host memory released first
            import gc
            import types

            gc.collect()
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            torch._C._host_emptyCache()
            c5_args = types.SimpleNamespace(**vars(args))
            c5_args.steps, c5_args.warmup = min(args.steps, 10), max(args.warmup, 3)
            sub = run_config5(c5_args, rank, world, local_rank, log)
            result["config5"] = {k: sub[k] for k in ("metric", "value", "unit", "n_gpus", "steps",
                                                    "warmup", "ms_per_step", "scaling", "config",
                                                    "stage_ms_per_step", "timed", "eager_tok_s",
                                                    "per_rank")}
        os.sched_setaffinity(0, all_cpus)  # the CPU baseline uses every host core
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                result["cpu_baseline"] = cpu_sample(log=log)
            print(json.dumps(result), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
