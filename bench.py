"""Benchmark of the B200 functional executor on BASELINE.json's headline configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--no-suite]

Workload (the metric's "GB/s vs B200 roofline"): one step = the reference's
vector-unit row programs over bf16 [4096, 4096] -- the bundle's softmax kernel
(vector_softmax_4096x4096_bf16/00_*) and the Qwen3 RMSNorm kernel (qwen3_8b_layer_prefill_4096x4096_bf16/00_*,
weight N(1, 0.02), eps 1e-6) -- each executed from its lowered kernel object (tests/golden/objects/) through
the C ABI.  Inputs N(0, 1) from seed 0, resident in HBM; L2 (126 MB) is flushed by a 512 MiB write (then a
256 MiB read, so the flush's own dirty lines are written back before the timed region) before
every timed step; each step is timed with CUDA events on the launching stream, max over ranks.
Multi-GPU: every rank runs its own copy of the workload (independent programs, no collective): weak
scaling, value = all ranks' bytes / the slowest rank's time.

Algorithmic bytes per step: softmax 2 * 2 * 4096^2 = 67,108,864; RMSNorm 67,108,864 + 8,192 (weight).
`e2e` repeats the step through the same API with the inputs copied from pinned host memory and both
outputs read back inside the timed region.  `cpu_baseline` times the CPU oracle (torch, all host threads)
on the same programs.  --impl reference runs only that CPU restatement of the reference's programs (the
reference's own functional simulator, Spike + the Coprocessor model, is not installable here)."""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "pytorchsim-triton-backend_b200"))
sys.path.insert(0, ROOT)

OBJECTS = os.path.join(ROOT, "tests", "golden", "objects")
METRIC = "lowered-kernel GB/s (softmax + RMSNorm bf16 4096x4096) vs B200 HBM roofline"
SOFTMAX_BYTES = 2 * 2 * 4096 * 4096
RMSNORM_BYTES = 2 * 2 * 4096 * 4096 + 2 * 4096
STEP_BYTES = SOFTMAX_BYTES + RMSNORM_BYTES
FALLBACK_HBM_GBS = 6650.0


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", 1590.0)), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, 1590.0, "fallback"


def load_object(name):
    from pytorchsim_triton_compiler.contract import kernel_object as ko
    d = os.path.join(OBJECTS, name)
    m = ko.read(d)
    return m, ko.read_desc(d, m)


def profile_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary (profiles/traffic.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as fh:
            t = json.load(fh)
        return t.get(kernel, {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


class L2Flush:
    """Empties L2 before a timed step: a 512 MiB write evicts every line of the workload, and a 256 MiB read
    then replaces the write's dirty lines with clean ones, so the timed kernel does not pay for writing
    the flush buffer back to HBM."""

    def __init__(self, dev):
        import torch
        self.w = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.r.sum()


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.path = index, None, None

    def start(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.err = self.path + ".err"
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv",
                                          "-i", str(self.index), "-lms", "200"], stdout=open(self.path, "w"),
                                         stderr=open(self.err, "w"))
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"error": "nvidia-smi not runnable"}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        lines = [ln.strip() for ln in open(self.path) if ln.strip()]
        err = open(self.err).read().strip()
        os.unlink(self.path)
        os.unlink(self.err)
        if len(lines) < 2:
            return {"error": (err or "no samples")[:200]}
        head = [h.strip() for h in lines[0].split(",")]

        def col(name):
            return next((i for i, h in enumerate(head) if h.startswith(name)), None)

        def num(x):
            try:
                return float(x.strip().split()[0])
            except (ValueError, IndexError):
                return None

        ism, imax = col("clocks.current.sm"), col("clocks.max.sm")
        rows = [[f.strip() for f in ln.split(",")] for ln in lines[1:] if not ln.startswith("index")]
        sm = [num(r[ism]) for r in rows if ism is not None and len(r) == len(head)]
        mx = [num(r[imax]) for r in rows if imax is not None and len(r) == len(head)]
        sm, mx = [x for x in sm if x is not None], [x for x in mx if x is not None]
        reasons = set()
        for name in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"):
            i = next((k for k, h in enumerate(head) if h.endswith("." + name)), None)
            if i is not None and any(len(r) == len(head) and r[i].lower() == "active" for r in rows):
                reasons.add(name)
        top = max(mx) if mx else None
        loaded = [x for x in sm if top and x > 0.5 * top] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": top,
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "b200":
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def reduce_max(v, world, device=None):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_per_step(times, world, device=None):
    """Per-step device times (ms) of this rank -> the element-wise maximum over ranks (a step of a
    partitioned launch ends when its slowest rank ends)."""
    if world == 1:
        return list(times)
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(times), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def my_range(units, world, rank):
    """This rank's unit range of a launch of `units` (the reference's split edges total * w // n,
    runtime/spike.py:257-258)."""
    return units * rank // world, units * (rank + 1) // world


# ---------------------------------------------------------------------------------------------------
# CPU oracle timing (cpu_baseline and the reference arm)
# ---------------------------------------------------------------------------------------------------

def cpu_step_inputs(rows):
    import torch
    g = torch.Generator().manual_seed(0)
    xs = torch.randn(rows * 4096, generator=g).to(torch.bfloat16)
    xr = torch.randn(rows * 4096, generator=g).to(torch.bfloat16)
    w = (torch.randn(4096, generator=g) * 0.02 + 1.0).to(torch.bfloat16)
    return xs, xr, w


def cpu_rate(seconds=10.0, rows=4096):
    """GB/s of the CPU oracle on the workload, timed for about `seconds` of repeated full steps."""
    import torch
    from oracle import programs as O
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    xs, xr, w = cpu_step_inputs(rows)
    O.softmax_rows(xs, rows, 4096)
    O.rmsnorm_rows(xr, w, rows, 4096, 1e-6)
    n, t0 = 0, time.perf_counter()
    while True:
        O.softmax_rows(xs, rows, 4096)
        O.rmsnorm_rows(xr, w, rows, 4096, 1e-6)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds or n >= 200:
            break
    bytes_per = (STEP_BYTES * rows) / 4096
    return {"value": round(n * bytes_per / dt / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n} full steps ({rows}x4096 softmax + RMSNorm) in {dt:.1f} s, torch CPU "
                                      f"restatement of the reference programs (oracle/programs.py)"}, dt / n


def interpreter_baseline():
    """The reference's own Triton kernels timed under the Triton interpreter (one core), as
    tests/golden/interpreter_baseline.py recorded them in the build container (the reference tree is not on
    the GPU box), or None."""
    try:
        with open(os.path.join(ROOT, "tests", "golden", "interpreter_baseline.json")) as fh:
            return json.load(fh)
    except (OSError, ValueError):
        return None


def run_reference(args, world, rank):
    if rank != 0:
        return
    base, sec_per_step = cpu_rate(seconds=min(30.0, 4.0 * max(1, args.steps)))
    line = {"metric": METRIC, "value": base["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(sec_per_step * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "softmax+rmsnorm bf16 [4096,4096] (BASELINE.json configs[1])", "rows": 4096,
                       "cols": 4096, "l2": "n/a (CPU)"},
            "impl": "reference", "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's functional simulator (Spike + Coprocessor model) is not installable here; "
                    "this arm times the CPU restatement of the same programs on all host threads"}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------------------------------

def tp_layer_timing(dev, world, rank, steps, warmup):
    """BASELINE.json config 5 across the ranks: the Qwen3-8B-shaped layer (T = 2048) split column- and
    row-wise over `world` GPUs, each rank's two segments replayed from CUDA graphs with an NCCL all-reduce
    after each row-parallel GEMM (o_proj, down).  Whole-layer TFLOP/s from the slowest rank's time.  Beside
    it: the whole layer on one GPU (every rank runs it on its own GPU at once; the slowest counts), the
    efficiency t1 / (n t_n), and where the TP step's time goes (the two graph segments and one all-reduce of
    the 16 MiB partial sums, each timed alone, slowest rank)."""
    import torch
    import torch.distributed as dist
    from oracle import programs as O
    from pytorchsim_triton_compiler.runtime import qwen3 as Q
    T = 2048
    stream = torch.cuda.current_stream(dev)
    _, tflops, _ = peaks()
    one = layer_timing(dev, stream, 5, 2, L2Flush(dev), tflops)
    t1 = reduce_max(one["ms"], world, dev)
    p = Q.random_params(0)
    x = torch.randn(T * Q.HIDDEN, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    cos, sin = O.rope_tables(T)
    g1, g2 = Q.build_layer(dev, T, Q.shard(p, rank, world), cos, sin, x, tp=world, rank=rank)
    g1.capture()
    g2.capture()
    x1, y = g1.buffers["x1"], g1.buffers["y"]

    def layer():
        g1.run()
        dist.all_reduce(x1)
        g2.run()
        dist.all_reduce(y)

    for _ in range(warmup):
        layer()
    torch.cuda.synchronize()
    dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev:
        a.record()
        layer()
        b.record()
    torch.cuda.synchronize()
    ms = reduce_max(statistics.median([a.elapsed_time(b) for a, b in ev]), world, dev)

    def alone(fn, n=8):
        e = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        dist.barrier()
        torch.cuda.synchronize()
        for a, b in e:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return reduce_max(statistics.median([a.elapsed_time(b) for a, b in e[2:]]), world, dev)

    seg1, seg2 = alone(g1.run), alone(g2.run)
    ar = alone(lambda: dist.all_reduce(x1))
    del g1, g2
    serial_ms = ms
    # The same layer with the o projection and the MLP in row blocks whose all-reduces overlap the next
    # block's compute (runtime/qwen3.py TpLayer); the fastest blocking is the reported figure.
    overlapped = {}
    for chunks in (2, 4):
        lay = Q.TpLayer(dev, T, Q.shard(p, rank, world), cos, sin, x, world, rank, chunks=chunks)
        lay.capture()
        for _ in range(warmup):
            lay.run(dist.all_reduce)
        overlapped[chunks] = alone(lambda: lay.run(dist.all_reduce), n=steps + 2)
        del lay
    best = min(overlapped, key=overlapped.get)
    # The layer with both all-reduces done by the executor's own kernels over NVLink peer memory (rank-order sum of
    # the rows each rank owns, stored into every rank's buffer; runtime/qwen3.py TpLayerPeer): "pull" loads every
    # rank's partial in one all-reduce kernel; "fused" pushes each GEMM's output rows to their owners from the
    # GEMM's epilogue and sums the staging in a second kernel.  Beside each: its collective (the 16 MiB all-reduce,
    # or the reduce-gather half) and its two segments timed alone.
    s_ = torch.cuda.current_stream(dev).cuda_stream
    peer = {}
    for fused in (False, True):
        lay = Q.TpLayerPeer(dev, T, Q.shard(p, rank, world), cos, sin, x, world, rank, fused=fused)
        lay.capture()
        for _ in range(warmup):
            lay.run()
        key = "fused" if fused else "pull"
        peer[key] = {"ms": alone(lay.run, n=steps + 2),
                     "collective_alone_ms": alone(lambda: lay.allreduce("x1p", "x1", "sig1", s_), n=10),
                     "segment_1_ms": alone(lay.g1.run), "segment_2_ms": alone(lay.g2.run)}
        lay.close()
        del lay
    peer_ms = min(v["ms"] for v in peer.values())
    ms = min(ms, overlapped[best], peer_ms)
    tf = Q.layer_flops(T) / ms / 1e9
    return {"n_gpus": world, "ms": round(ms, 4), "TFLOP/s": round(tf, 1), "frac_bf16": round(tf / (world * tflops), 3),
            "scaling": "strong", "one_gpu_ms": round(t1, 4), "speedup": round(t1 / ms, 3),
            "efficiency": round(t1 / (world * ms), 3),
            "nccl_serial_ms": round(serial_ms, 4),
            "nccl_overlapped_ms": {f"{c}_row_blocks": round(v, 4) for c, v in overlapped.items()},
            "peer": {k: {kk: round(vv, 4) for kk, vv in v.items()} for k, v in peer.items()},
            "parts_ms": {"segment_1": round(seg1, 4), "segment_2": round(seg2, 4),
                         "nccl_all_reduce_16MiB": round(ar, 4), "all_reduces_per_layer": 2},
            "collective": "after o_proj and after down, an all-reduce of the 2048 x 4096 bf16 partial sums: NCCL "
                          "(serial, or in row blocks overlapped with compute) or the executor's own kernels over "
                          "NVLink peer memory (pull: ptsim_tp_allreduce; fused: the GEMM pushes its rows to their "
                          "owners, ptsim_launch_rows_to_owners, then ptsim_tp_reduce_gather); ms is the fastest"}


def strong_headline(dev, world, rank, steps, warmup, d_s, d_r, ps, pr, flush, stream):
    """The headline step partitioned over the ranks (strong scaling): rank r runs its unit range of the
    softmax and the RMSNorm launch (row blocks, the reference's split edges) over its own device-resident
    copy of the inputs; no collective on the data path.  GB/s of the whole step from the per-step maximum
    over ranks of each rank's device time."""
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    s_lo, s_hi = my_range(D.from_bytes(d_s).units, world, rank)
    r_lo, r_hi = my_range(D.from_bytes(d_r).units, world, rank)
    sp = stream.cuda_stream
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps + warmup)]
    barrier(world)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(1e7))
    for k in range(steps + warmup):
        flush()
        ev[k][0].record(stream)
        native.launch(d_s, ps, s_lo, s_hi, stream=sp)
        native.launch(d_r, pr, r_lo, r_hi, stream=sp)
        ev[k][1].record(stream)
    native.sync(sp)
    per = max_per_step([a.elapsed_time(b) for a, b in ev[warmup:]], world, dev)
    ms = sum(per) / len(per)
    return {"n_gpus": world, "scaling": "strong", "ms_per_step": round(ms, 4),
            "GB/s": round(STEP_BYTES / ms / 1e6, 1),
            "rows_per_rank": "4096 / n_gpus (unit ranges total * w // n of each launch)",
            "timing": "per step, the maximum over ranks of each rank's CUDA-event time; L2 flushed before each step"}


def split_suite(dev, world, rank, iters=5, warm=2):
    """BASELINE.json configs partitioned over the ranks, each rank running its unit range of the lowered
    kernel object over device-resident inputs (no collective): vector add by elements, GEMM 4096^3 by
    output rows (M), causal attention B4 H32 S4096 by (batch, query head).  Whole-job throughput from the
    maximum over ranks of each launch's device time (median over `iters`, L2 flushed before each)."""
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    hbm, tflops, _ = peaks()
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)
    out = {}
    for name, bound, work in (("vector_add_1m", "hbm", 3 * 4 * 1_048_576),
                              ("gemm_4096x4096x4096", "tensor", 2 * 4096 ** 3),
                              ("attention_32x8x4096_b4", "tensor", 549_755_813_888)):
        m, blob = load_object(name)
        d = D.from_bytes(blob)
        g = torch.Generator(device=dev).manual_seed(0)
        ts = []
        for a in m["args"]:
            dt = getattr(torch, a["dtype"])
            n = math.prod(a["shape"])
            std = 1.0 / math.sqrt(d.p.gemm.K) if d.kind == D.GEMM and a["name"] in ("arg_A", "arg_B") else 1.0
            ts.append((torch.randn(n, generator=g, device=dev) * std).to(dt) if a["role"] in ("in", "inout")
                      else torch.zeros(n, dtype=dt, device=dev))
        lo, hi = my_range(d.units, world, rank)
        wsn = native.workspace_size(blob, dev.index or 0)
        ws = torch.empty(max(1, wsn), dtype=torch.uint8, device=dev)
        ptrs = [t.data_ptr() for t in ts]
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters + warm)]
        barrier(world)
        torch.cuda.synchronize()
        torch.cuda._sleep(int(1e7))
        for k in range(iters + warm):
            flush()
            ev[k][0].record(stream)
            native.launch(blob, ptrs, lo, hi, ws.data_ptr(), wsn, stream.cuda_stream)
            ev[k][1].record(stream)
        native.sync(stream.cuda_stream)
        per = max_per_step([a.elapsed_time(b) for a, b in ev[warm:]], world, dev)
        ms = statistics.median(per)
        entry = {"ms": round(ms, 4), "units_per_rank": f"{d.units} / {world}"}
        if bound == "hbm":
            gbs = work / ms / 1e6
            entry.update({"GB/s": round(gbs, 1), "frac_hbm": round(gbs / (world * hbm), 3)})
        else:
            tf = work / ms / 1e9
            entry.update({"TFLOP/s": round(tf, 1), "frac_bf16": round(tf / (world * tflops), 3)})
        out[name] = entry
        del ts, ws
    out["note"] = ("strong scaling: one launch's units split over the ranks (spike.py's total * w // n edges); "
                   "frac is of n_gpus x the measured per-GPU peak")
    return out


def sweep_timing(dev, world, rank, iters=5, warm=2):
    """BASELINE.json configs[2]'s M sweep (M in {128, 512, 2048, 4096, 8192}, N = K = 4096) spread over the ranks
    by longest processing time (runtime/sweep.py, the reference's validation/gemm/simulate_shapes.py shard): each
    rank runs only its own points on its own GPU, no collective.  Per iteration a rank's time is the sum of its
    points' device times (L2 flushed before each launch); the job's time is the maximum over ranks.  Beside it:
    the whole sweep on one GPU (every rank runs all points at once; the slowest counts), and the bound no split
    of these points can beat (the costliest point alone, 8192 x 4096 x 4096)."""
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    from pytorchsim_triton_compiler.runtime import sweep as SW
    _, tflops, _ = peaks()
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)
    names = [f"gemm_{m}x4096x4096" for m in (128, 512, 2048, 4096, 8192)]
    objs = {n: load_object(n) for n in names}
    pts = [SW.Point(n, objs[n][1]) for n in names]
    bufs = {}
    for n in names:
        m, blob = objs[n]
        d = D.from_bytes(blob)
        g = torch.Generator(device=dev).manual_seed(0)
        ts = [(torch.randn(math.prod(a["shape"]), generator=g, device=dev) / math.sqrt(d.p.gemm.K)).to(torch.bfloat16)
              if a["role"] in ("in", "inout") else torch.zeros(math.prod(a["shape"]), dtype=torch.bfloat16, device=dev)
              for a in m["args"]]
        wsn = native.workspace_size(blob, dev.index or 0)
        bufs[n] = (blob, d.units, ts, torch.empty(max(1, wsn), dtype=torch.uint8, device=dev), wsn)

    def run(points):
        """Per iteration, this rank's summed device time (ms) over `points`, and each point's median."""
        each = {p.name: [] for p in points}
        total = []
        barrier(world)
        torch.cuda.synchronize()
        for k in range(iters + warm):
            ev = []
            for p in points:
                blob, units, ts, ws, wsn = bufs[p.name]
                flush()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                native.launch(blob, [t.data_ptr() for t in ts], 0, units, ws.data_ptr(), wsn, stream.cuda_stream)
                b.record(stream)
                ev.append((p.name, a, b))
            native.sync(stream.cuda_stream)
            if k >= warm:
                ms = [(n, a.elapsed_time(b)) for n, a, b in ev]
                total.append(sum(t for _, t in ms))
                for n, t in ms:
                    each[n].append(t)
        return total, {n: statistics.median(v) for n, v in each.items() if v}

    mine = SW.shard(pts, rank, world)
    t_n, _ = run(mine)   # every rank runs it (a rank without points too: run() meets the barrier)
    tn = statistics.median(max_per_step(t_n, world, dev))
    t_1, per_point = run(pts)
    t1 = statistics.median(max_per_step(t_1, world, dev))
    flops = 2 * sum(p.cost for p in pts)
    return {"points": [p.name for p in SW.longest_first(pts)], "shards": [[p.name for p in SW.shard(pts, r, world)] for r in range(world)],
            "ms": round(tn, 4), "TFLOP/s": round(flops / tn / 1e9, 1), "frac_bf16": round(flops / tn / 1e9 / (world * tflops), 3),
            "one_gpu_ms": round(t1, 4), "speedup": round(t1 / tn, 3),
            "costliest_point_ms": round(per_point.get(names[-1], 0.0), 4),
            "note": "no split of these five points finishes before the costliest one (8192 x 4096 x 4096); "
                    "speedup is bounded by one_gpu_ms / costliest_point_ms"}


def run_b200(args, world, rank, local):
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import cuda as RC
    from pytorchsim_triton_compiler.runtime import native

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    native.init(local)
    m_s, d_s = load_object("softmax_4096x4096")
    m_r, d_r = load_object("rmsnorm_4096x4096")
    xs_h, xr_h, w_h = cpu_step_inputs(4096)
    xs, xr, w = xs_h.to(dev), xr_h.to(dev), w_h.to(dev)
    ys = torch.empty_like(xs)
    yr = torch.empty_like(xr)
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        native.launch(d_s, [xs.data_ptr(), ys.data_ptr()], 0, D.from_bytes(d_s).units, stream=sp)
        if ev is not None:
            ev[1].record(stream)
        native.launch(d_r, [xr.data_ptr(), w.data_ptr(), yr.data_ptr()], 0, D.from_bytes(d_r).units, stream=sp)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(args.warmup):
        flush()
        step()
    native.sync(sp)
    # Correctness of what is timed: compare one row block against the oracle.
    from oracle import programs as O
    chk = slice(0, 64 * 4096)
    want_s = O.softmax_rows(xs_h[chk], 64, 4096)
    want_r = O.rmsnorm_rows(xr_h[chk], w_h, 64, 4096, 1e-6)
    from oracle import tolerance as T
    try:
        T.check(ys[chk], want_s, T.POINTWISE, name="softmax rows 0-63")
        T.check(yr[chk], want_r, T.POINTWISE, name="RMSNorm rows 0-63")
    except AssertionError as why:
        raise SystemExit(f"bench: the timed kernels disagree with the oracle: {why}")

    clocks = Clocks(local)
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    # The GPU spins while the host enqueues every timed step, so the events measure kernels, not the
    # host's launch latency.  A step is timed from an event before the softmax launch to one after the
    # RMSNorm launch: the RMSNorm kernel, a programmatic dependent, is scheduled while the softmax grid
    # drains (an event between the two would serialise them).
    torch.cuda._sleep(int(1e7))
    for k in range(args.steps):
        flush()                     # L2 flush, outside the timed events
        events[k][0].record(stream)
        step()
        events[k][1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    native.sync(sp)
    total_ms = sum(e[0].elapsed_time(e[1]) for e in events)
    total_ms = reduce_max(total_ms, world, dev)
    ms_per_step = total_ms / args.steps
    value = world * STEP_BYTES * args.steps / (total_ms / 1e3) / 1e9

    # Per-kernel device times for the roofline, from the same number of extra steps with an event between
    # the two launches (each launch then runs alone).
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    torch.cuda.synchronize()
    torch.cuda._sleep(int(1e7))
    for k in range(args.steps):
        flush()
        step(kev[k])
    torch.cuda.synchronize()
    native.sync(sp)
    t_soft = [e[0].elapsed_time(e[1]) for e in kev]
    t_rms = [e[1].elapsed_time(e[2]) for e in kev]

    # e2e: the same step through the runtime's host-memory launcher (runtime.cuda.HostPipeline, one C-ABI call
    # ptsim_launch_host per launch) with pinned host buffers: every step copies the inputs in and the outputs
    # back inside the timed region, 4 row ranges pipelined so PCIe carries both directions while the kernels
    # run (8, 16 and 32 ranges measured slower: 77.4, 66.8 and 59.3 GB/s against 80.7).
    xs_p, xr_p, w_p = xs_h.pin_memory(), xr_h.pin_memory(), w_h.pin_memory()
    ys_p, yr_p = torch.empty_like(xs_p).pin_memory(), torch.empty_like(xr_p).pin_memory()
    e2e_steps = max(3, args.steps)
    pipe = RC.HostPipeline(local, chunks=4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d = xs_p.numel() * 2 + xr_p.numel() * 2 + w_p.numel() * 2
    d2h = ys_p.numel() * 2 + yr_p.numel() * 2
    e2e_ms = 0.0
    for k in range(e2e_steps + 1):
        flush()
        pipe.s_in.wait_stream(stream)
        e0.record(pipe.s_in)
        pipe.submit(d_s, [xs_p, ys_p])
        pipe.submit(d_r, [xr_p, w_p, yr_p])
        e1.record(pipe.s_out)
        pipe.wait()
        if k > 0:
            e2e_ms += e0.elapsed_time(e1)
    try:
        T.check(ys_p[chk], want_s, T.POINTWISE, name="end-to-end softmax rows 0-63")
        T.check(yr_p[chk], want_r, T.POINTWISE, name="end-to-end RMSNorm rows 0-63")
    except AssertionError as why:
        raise SystemExit(f"bench: the end-to-end outputs disagree with the oracle: {why}")
    e2e_ms = reduce_max(e2e_ms, world, dev)
    e2e_val = world * STEP_BYTES * e2e_steps / (e2e_ms / 1e3) / 1e9

    # The ceiling of e2e: the same host<->device bytes as plain pinned copies, the inputs going in on one
    # stream while outputs come back on another (what the pipeline overlaps), with no kernel between.
    c_in, c_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    hin = [torch.empty_like(t).pin_memory() for t in (xs_h, xr_h, w_h)]
    din = [torch.empty_like(t, device=dev) for t in hin]
    hout = [torch.empty_like(t).pin_memory() for t in (xs_h, xr_h)]
    cp = []
    for k in range(4):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        c_in.wait_stream(stream)
        c_out.wait_stream(stream)
        with torch.cuda.stream(c_in):
            for h, d_ in zip(hin, din):
                d_.copy_(h, non_blocking=True)
        with torch.cuda.stream(c_out):
            hout[0].copy_(ys, non_blocking=True)
            hout[1].copy_(yr, non_blocking=True)
        stream.wait_stream(c_in)
        stream.wait_stream(c_out)
        b.record(stream)
        torch.cuda.synchronize()
        if k > 0:
            cp.append(a.elapsed_time(b))
    copy_ms = reduce_max(statistics.median(cp), world, dev)
    e2e_ceiling = world * STEP_BYTES / (copy_ms / 1e3) / 1e9
    del hin, din, hout

    # Context for the roofline: a plain device copy of the same 32 MiB under the same flush.
    cp_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(8)]
    for a, b in cp_ev:
        flush()
        a.record(stream)
        ys.copy_(xs)
        b.record(stream)
    torch.cuda.synchronize()
    cp_ms = statistics.median([a.elapsed_time(b) for a, b in cp_ev[2:]])

    hbm, _, peak_src = peaks()
    soft_ms, rms_ms = sum(t_soft) / len(t_soft), sum(t_rms) / len(t_rms)
    dom, dom_ms, dom_bytes = ("row_softmax", soft_ms, SOFTMAX_BYTES) if sum(t_soft) >= sum(t_rms) else \
        ("row_rmsnorm", rms_ms, RMSNORM_BYTES)
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    traffic = profile_traffic(dom)
    # The same launch time over the DRAM bytes ncu counted for the kernel (reads + writes during the launch):
    # the output stays in L2 as dirty lines and is written back after the kernel, so this is about half the
    # algorithmic figure.
    dram_frac = round(traffic / (dom_ms / 1e3) / 1e9 / hbm, 4) if traffic else None
    line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "softmax+rmsnorm bf16 [4096,4096] (BASELINE.json configs[1])",
                       "rows": 4096, "cols": 4096, "programs": ["vector_softmax_4096x4096_bf16/00",
                                                                 "qwen3_8b_layer_prefill_4096x4096_bf16/00"],
                       "l2": "flushed before every timed step (512 MiB write, then a 256 MiB read so no dirty flush lines are written back inside the timed region)", "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic, "frac_dram_bytes": dram_frac,
                         "copy_same_bytes_gbs": round(SOFTMAX_BYTES / cp_ms / 1e6, 1),
                         "per_kernel": {"row_softmax": {"ms": round(soft_ms, 4), "GB/s": round(SOFTMAX_BYTES / soft_ms / 1e6, 1)},
                                        "row_rmsnorm": {"ms": round(rms_ms, 4), "GB/s": round(RMSNORM_BYTES / rms_ms / 1e6, 1)}}},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "runtime.cuda.HostPipeline -> C ABI ptsim_launch_host over pinned host buffers, 4 pipelined row ranges per launch",
                    "copy_ceiling": round(e2e_ceiling, 2), "frac_of_copy_ceiling": round(e2e_val / e2e_ceiling, 3),
                    "copy_ceiling_note": "the same bytes as plain pinned copies (inputs in and outputs out on two "
                                         "streams at once, no kernel), in this metric's units"},
            "gpu_launches": 2 * args.steps,
            "timing": "value and ms_per_step: one event pair around each step's two launches (the RMSNorm launch "
                      "is the softmax's programmatic dependent); roofline.per_kernel: the same steps again with an "
                      "event between the launches",
            "clocks": clk}
    if world > 1:
        line["strong"] = strong_headline(dev, world, rank, args.steps, args.warmup, d_s, d_r,
                                         [xs.data_ptr(), ys.data_ptr()], [xr.data_ptr(), w.data_ptr(), yr.data_ptr()],
                                         flush, stream)
    if world > 1 and args.suite:
        line["split_suite"] = split_suite(dev, world, rank)
        line["sweep"] = sweep_timing(dev, world, rank)
        line["tp_layer"] = tp_layer_timing(dev, world, rank, steps=10, warmup=3)
    if rank == 0 and world == 1 and args.cpu:
        base, _ = cpu_rate(seconds=10.0)
        interp = interpreter_baseline()
        if interp is not None:
            base["interpreter"] = interp
        line["cpu_baseline"] = base
        if args.suite:
            line["suite"] = suite(dev, stream)
    if rank == 0:
        print(json.dumps(line), flush=True)


def suite(dev, stream, iters=5, only=None, warm=1):
    """Device-timed throughput of the other BASELINE.json configurations' lowered kernels (not the
    headline): median of `iters` launches with an L2 flush before each."""
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    hbm, tflops, _ = peaks()
    flush = L2Flush(dev)
    out = {}

    def timed(name, bound, work, int_fill=None, given=None):
        if only is not None and name != only:
            return
        m, blob = load_object(name)
        d = D.from_bytes(blob)
        g = torch.Generator(device=dev).manual_seed(0)
        ts = []
        for a in m["args"]:
            dt = getattr(torch, a["dtype"])
            n = math.prod(a["shape"])
            if given is not None and a["name"] in given:
                ts.append(given[a["name"]].to(dt).to(dev))
            elif a["role"] in ("in", "inout") and dt.is_floating_point:
                std = 1.0
                if d.kind == D.GEMM and a["name"] in ("arg_A", "arg_B"):
                    std = 1.0 / math.sqrt(d.p.gemm.K)   # N(0, 1/sqrt(K))
                ts.append((torch.randn(n, generator=g, device=dev) * std).to(dt))
            elif a["role"] in ("in", "inout") and int_fill is not None:
                ts.append(int_fill(n).to(dt).to(dev))
            else:
                ts.append(torch.zeros(n, dtype=dt, device=dev))
        wsn = native.workspace_size(blob, dev.index or 0)
        ws = torch.empty(max(1, wsn), dtype=torch.uint8, device=dev)
        ptrs = [t.data_ptr() for t in ts]
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters + warm)]
        torch.cuda.synchronize()
        torch.cuda._sleep(int(1e7))       # the host enqueues every launch before the GPU reaches them
        for k in range(iters + warm):
            flush()
            ev[k][0].record(stream)
            native.launch(blob, ptrs, 0, d.units, ws.data_ptr(), wsn, stream.cuda_stream)
            ev[k][1].record(stream)
        native.sync(stream.cuda_stream)
        times = [a.elapsed_time(b) for a, b in ev[warm:]]
        ms = statistics.median(times)
        if bound == "hbm":
            gbs = work / ms / 1e6
            out[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3)}
        else:
            tf = work / ms / 1e9
            out[name] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1), "frac_bf16": round(tf / tflops, 3)}

    timed("vector_add_1m", "hbm", 3 * 4 * 1_048_576)
    if only is None or only == "vector_add_1m_amortized":
        out["vector_add_1m_amortized"] = amortized_vector_add(dev, stream, hbm)
    timed("vector_add1_4096x4096", "hbm", 2 * 2 * 4096 * 4096)
    for m in (128, 512, 2048, 4096, 8192):
        timed(f"gemm_{m}x4096x4096", "tensor", 2 * m * 4096 * 4096)
    timed("attention_32x8x4096_b4", "tensor", 549_755_813_888)
    # Decode side: the M = 1 matmul reads the matrix once (plus the vector and the output); decode
    # attention reads every key and value once (plus q and o), 2 x 8 heads x S x 128 x 2 bytes.
    gemv_bytes = 2 * (4096 * 4096 + 4096 + 4096)
    dec_bytes = {s: 2 * 2 * 8 * s * 128 + 2 * 2 * 4096 for s in (4096, 8192)}
    timed("gemm_1x4096x4096", "hbm", gemv_bytes)
    timed("attention_decode_32x8x4096", "hbm", dec_bytes[4096])
    timed("attention_decode_32x8x8192", "hbm", dec_bytes[8192])
    # MoE routing at T = 4096 (128 experts, top-8, hidden 2048): the dispatch copy writes 32768 rows of 4 KB
    # (each of the 4096 token rows read 8 times, mostly from L2); the top-k reads 4096 x 128 fp32 router
    # probabilities; the sort reorders 32768 expert ids.
    perm = lambda n: torch.randperm(n, generator=torch.Generator().manual_seed(1))          # sorted positions
    experts = lambda n: torch.randint(0, 128, (n,), generator=torch.Generator().manual_seed(2))  # expert ids
    timed("moe_dispatch_t4096_01_gather", "hbm", 2 * 32768 * 2048 + 2 * 4096 * 2048 + 8 * 32768, perm)
    timed("moe_router_t4096_01_topk", "hbm", 4 * 4096 * 128 + (4 + 8) * 32768)
    timed("moe_dispatch_t4096_00_sort", "hbm", 3 * 8 * 32768, experts)
    # combine: 32768 expert-output rows gathered (4 KB each) and weighted into 4096 token rows
    if only is None or only == "moe_combine_t4096_03_weighted":
        ids, cum, cnt, pos = moe_routing(4096, 8, 128, 7)
        timed("moe_combine_t4096_03_weighted", "hbm", 2 * 32768 * 2048 + 2 * 4096 * 2048 + 8 * 3 * 32768,
              given={"in_ptr0": ids, "in_ptr1": cum, "in_ptr2": cnt, "in_ptr3": pos})
    # combine's routing tables: counts and running counts of 128 experts over 32768 routed ids (writes the
    # [32768, 128] int64 running table), and each routed row's slot (the program sums the table row times a
    # one-hot of the row's expert: the one selected element, its id and the output per row are what it needs)
    if only is None or only in ("moe_combine_t4096_00_counts", "moe_combine_t4096_02_slot"):
        ids = moe_routing(4096, 8, 128, 7)[0]
        timed("moe_combine_t4096_00_counts", "hbm", 8 * 32768 * 128 + 8 * 32768 + 8 * 128, given={"in_ptr0": ids})
        run_ = torch.randint(0, 300, (32768 * 128,), generator=torch.Generator().manual_seed(3))
        timed("moe_combine_t4096_02_slot", "hbm", 3 * 8 * 32768, given={"in_ptr0": run_, "in_ptr1": ids})
    # The Qwen3-8B decode layer's fused matrix-vector products: the RMSNorm'd vector times the gate_up weights
    # (4096 x 24576, residual row added first), the SiLU'd vector times the down weights (12288 x 4096, two
    # residual rows added after); each streams its weights once.
    timed("qwen3_decode_06_rmsnorm_gate_up_mm", "hbm", 2 * 4096 * 24576 + 2 * 3 * 4096 + 4 + 2 * 24576)
    timed("qwen3_decode_07_silu_down_mm", "hbm", 2 * 12288 * 4096 + 2 * 24576 + 2 * 3 * 4096)
    for nm, K, N in (("moe_gmm_gate_up_t4096", 2048, 1536), ("moe_gmm_down_t4096", 768, 2048)):
        if only is None or only == nm:
            out[nm] = grouped_gemm_timing(dev, stream, iters, warm, flush, hbm, tflops, K, N)
    # The same objects as graph-replayed streams (launch latency amortised; inputs rotate past L2).
    for name, work, sets in (("gemm_1x4096x4096", gemv_bytes, 6), ("attention_decode_32x8x4096", dec_bytes[4096], 12),
                             ("attention_decode_32x8x8192", dec_bytes[8192], 6)):
        if only is None or only == name + "_amortized":
            out[name + "_amortized"] = amortized_object(dev, stream, hbm, name, work, sets)
    if only is None or only == "qwen3_layer":
        out["qwen3_layer_t2048"] = layer_timing(dev, stream, iters, warm, flush, tflops)
    if only is None or only == "qwen3_decode_layer_s4096":
        out["qwen3_decode_layer_s4096"] = decode_layer_timing(dev, stream, iters, warm, flush, hbm)
    return out


def moe_routing(tokens, topk, experts, seed):
    """A consistent synthetic MoE routing: each slot's expert id, the experts' counts and inclusive cumulative
    counts, and each slot's 1-based rank within its expert."""
    import torch
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, experts, (tokens * topk,), generator=g)
    cnt = torch.bincount(ids, minlength=experts)
    cum = torch.cumsum(cnt, 0)
    order = torch.argsort(ids, stable=True)
    rank = torch.empty_like(ids)
    rank[order] = torch.arange(tokens * topk) - (cum - cnt)[ids[order]]
    return ids, cum, cnt, rank + 1


def grouped_gemm_timing(dev, stream, iters, warm, flush, hbm, tflops, K, N, T=4096, G=128):
    """The MoE expert matmul at T tokens x top-8 over G experts (layer_op_gmm_*_4096x0 shapes), every expert
    receiving 8 T / G rows as the bundle's recorded routing does: median of `iters` launches, L2 flushed.
    The roofline is the slower of the weights' HBM read and the tensor work."""
    import torch
    from pytorchsim_triton_compiler.codegen import build as Bd
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    M = 8 * T
    blob = D.to_bytes(Bd.grouped_gemm(M, N, K, G, G))
    g = torch.Generator(device=dev).manual_seed(0)
    std = 1.0 / math.sqrt(K)
    a = (torch.randn(M * K, generator=g, device=dev) * std).to(torch.bfloat16)
    b = (torch.randn(G * K * N, generator=g, device=dev) * std).to(torch.bfloat16)
    rows = torch.full((G + 1,), M // G, dtype=torch.int32, device=dev)
    rows[G] = 0
    start = torch.arange(G + 1, dtype=torch.int32, device=dev) * (M // G)
    group = torch.arange(G, dtype=torch.int32, device=dev)
    c = torch.zeros(M * N, dtype=torch.bfloat16, device=dev)
    ptrs = [t.data_ptr() for t in (a, b, group, start, rows, c)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters + warm)]
    torch.cuda.synchronize()
    torch.cuda._sleep(int(1e7))
    for k in range(iters + warm):
        flush()
        ev[k][0].record(stream)
        native.launch(blob, ptrs, 0, 1, 0, 0, stream.cuda_stream)
        ev[k][1].record(stream)
    native.sync(stream.cuda_stream)
    ms = statistics.median([x.elapsed_time(y) for x, y in ev[warm:]])
    flops, nbytes = 2 * M * N * K, 2 * (G * K * N + M * K + M * N)
    ideal = max(flops / (tflops * 1e12), nbytes / (hbm * 1e9))
    return {"ms": round(ms, 4), "TFLOP/s": round(flops / ms / 1e9, 1), "GB/s": round(nbytes / ms / 1e6, 1),
            "bound": "hbm" if nbytes / (hbm * 1e9) > flops / (tflops * 1e12) else "tensor",
            "frac_roofline": round(ideal / (ms * 1e-3), 3)}


def amortized_vector_add(dev, stream, hbm, sets=16, launches=1024):
    """BASELINE.json configs[0] amortised: the lowered vector-add object (1,048,576 fp32 per launch,
    12.6 MB) replayed as `launches` back-to-back launches from one CUDA graph over `sets` rotating
    input/output sets (201 MB, more than L2), so the per-launch figure excludes the host and the timing
    events but keeps every launch's HBM traffic."""
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    m, blob = load_object("vector_add_1m")
    d = D.from_bytes(blob)
    n = 1_048_576
    g = torch.Generator(device=dev).manual_seed(0)
    bufs = [(torch.randn(n, generator=g, device=dev), torch.randn(n, generator=g, device=dev),
             torch.empty(n, device=dev)) for _ in range(sets)]
    s = torch.cuda.Stream(dev)
    s.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        native.launch(blob, [t.data_ptr() for t in bufs[0]], 0, d.units, stream=s.cuda_stream)
        native.sync(s.cuda_stream)
        with torch.cuda.graph(graph, stream=s):
            for i in range(launches):
                native.launch(blob, [t.data_ptr() for t in bufs[i % sets]], 0, d.units, stream=s.cuda_stream)
    stream.wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    native.sync(stream.cuda_stream)
    ms = statistics.median(ts) / launches
    ok = all(torch.equal(o, x + y) for x, y, o in bufs[:2])
    gbs = 3 * 4 * n / ms / 1e6
    del graph
    return {"ms_per_launch": round(ms, 5), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3),
            "launches": launches, "sets": sets, "bit_exact": ok}


def amortized_object(dev, stream, hbm, name, work, sets, launches=48):
    """A suite kernel object replayed as `launches` back-to-back launches from one CUDA graph over `sets`
    rotating input sets whose total exceeds L2, so the per-launch figure excludes the host and the timing
    events but keeps every launch's HBM traffic (`work` algorithmic bytes per launch)."""
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    m, blob = load_object(name)
    d = D.from_bytes(blob)
    g = torch.Generator(device=dev).manual_seed(0)
    bufs = []
    for _ in range(sets):
        ts = []
        for a in m["args"]:
            dt = getattr(torch, a["dtype"])
            n = math.prod(a["shape"])
            ts.append(torch.randn(n, generator=g, device=dev).to(dt) if a["role"] in ("in", "inout")
                      else torch.zeros(n, dtype=dt, device=dev))
        bufs.append(ts)
    wsn = native.workspace_size(blob, dev.index or 0)
    ws = torch.empty(max(1, wsn), dtype=torch.uint8, device=dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        native.launch(blob, [t.data_ptr() for t in bufs[0]], 0, d.units, ws.data_ptr(), wsn, s.cuda_stream)
        native.sync(s.cuda_stream)
        with torch.cuda.graph(graph, stream=s):
            for i in range(launches):
                native.launch(blob, [t.data_ptr() for t in bufs[i % sets]], 0, d.units, ws.data_ptr(), wsn,
                              s.cuda_stream)
    stream.wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    native.sync(stream.cuda_stream)
    ms = statistics.median(times) / launches
    gbs = work / ms / 1e6
    del graph
    return {"ms_per_launch": round(ms, 5), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3),
            "launches": launches, "sets": sets}


def decode_layer_timing(dev, stream, iters, warm, flush, hbm):
    """The Qwen3-8B decode layer at a 4096-token context (validation/pytorchsim/qwen3_8b_layer_decode_1x4096_bf16:
    sums of squares, the RMSNorm'd q projection, q-norm + RoPE, decode attention over the KV cache, the o
    projection, the residual sum's sum of squares, the RMSNorm'd gate_up projection, the SiLU'd down projection)
    as its 8 lowered kernel objects, one step replayed from a CUDA graph with L2 flushed before it.  Every
    argument is read or written once: their bytes are the step's algorithmic HBM traffic."""
    import torch
    from pytorchsim_triton_compiler.codegen import descriptors as D
    from pytorchsim_triton_compiler.runtime import native
    names = sorted(n for n in os.listdir(OBJECTS) if n.startswith("qwen3_decode_s4096_"))
    g = torch.Generator(device=dev).manual_seed(0)
    steps, keep, work = [], [], 0
    for name in names:
        m, blob = load_object(name)
        d = D.from_bytes(blob)
        ts = []
        for a in m["args"]:
            dt = getattr(torch, a["dtype"])
            n = math.prod(a["shape"])
            t = torch.randn(n, generator=g, device=dev)
            if n > 1 << 20:
                t = t / 64.0                       # weights and caches at a realistic scale
            ts.append((t.abs() if n == 1 else t).to(dt) if a["role"] in ("in", "inout") else torch.zeros(n, dtype=dt, device=dev))
            work += n * ts[-1].element_size()
        wsn = native.workspace_size(blob, dev.index or 0)
        ws = torch.empty(max(1, wsn), dtype=torch.uint8, device=dev)
        keep += ts + [ws]
        steps.append((blob, [t.data_ptr() for t in ts], d.units, ws.data_ptr(), wsn))
    s_ = torch.cuda.Stream(dev)
    s_.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s_):
        for blob, ptrs, units, wp, wn in steps:
            native.launch(blob, ptrs, 0, units, wp, wn, s_.cuda_stream)
        native.sync(s_.cuda_stream)
        with torch.cuda.graph(graph, stream=s_):
            for blob, ptrs, units, wp, wn in steps:
                native.launch(blob, ptrs, 0, units, wp, wn, s_.cuda_stream)
    stream.wait_stream(s_)
    graph.replay()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters + warm)]
    for k in range(iters + warm):
        flush()
        ev[k][0].record(stream)
        graph.replay()
        ev[k][1].record(stream)
    torch.cuda.synchronize()
    native.sync(stream.cuda_stream)
    ms = statistics.median(a.elapsed_time(b) for a, b in ev[warm:])
    del graph
    gbs = work / ms / 1e6
    return {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3), "programs": len(steps),
            "bytes": work}


def layer_timing(dev, stream, iters, warm, flush, tflops):
    """BASELINE.json config 4 on one GPU: the Qwen3-8B-shaped prefill layer (T = 2048) as the 14 launches
    of the reference's lowered kernel objects, replayed from a CUDA graph; TFLOP/s of GEMM + attention."""
    import torch
    from oracle import programs as O
    from pytorchsim_triton_compiler.contract import kernel_object as ko
    from pytorchsim_triton_compiler.runtime import qwen3 as Q
    T = 2048
    objs = {n.split("_")[2]: ko.read_desc(os.path.join(OBJECTS, n)) for n in os.listdir(OBJECTS)
            if n.startswith("qwen3_t2048_")}
    p = Q.random_params(0)
    x = torch.randn(T * Q.HIDDEN, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    cos, sin = O.rope_tables(T)
    g, _ = Q.build_layer(dev, T, p, cos, sin, x, objects=objs)
    g.capture()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters + warm)]
    torch.cuda.synchronize()
    torch.cuda._sleep(int(1e7))
    for k in range(iters + warm):
        flush()
        ev[k][0].record(stream)
        g.run()
        ev[k][1].record(stream)
    torch.cuda.synchronize()
    times = [a.elapsed_time(b) for a, b in ev[warm:]]
    ms = statistics.median(times)
    tf = Q.layer_flops(T) / ms / 1e9
    return {"ms": round(ms, 4), "TFLOP/s": round(tf, 1), "frac_bf16": round(tf / tflops, 3), "launches": g.launch_count(),
            "flops": Q.layer_flops(T)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-suite", dest="suite", action="store_false")
    ap.add_argument("--no-cpu", dest="cpu", action="store_false", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--kernel", default=None, help="time one suite kernel object only (for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.kernel:
        import torch
        dev = torch.device("cuda", 0)
        print(json.dumps(suite(dev, torch.cuda.current_stream(dev), iters=max(1, args.steps), only=args.kernel,
                               warm=args.warmup)))
        return
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_b200(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "b200":
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
