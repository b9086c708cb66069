"""The Qwen3-8B-shaped decoder layer (prefill) as the launch sequence of the validation bundle's workload
(validation/pytorchsim/qwen3_8b_layer_prefill_2048x2048_bf16/manifest.json, 14 launches):

    00 RMSNorm -> 01 q proj -> 02 q-norm + RoPE -> 03 k proj -> 04 k-norm + RoPE -> 03 v proj -> 05 v relayout
    -> 06 causal GQA attention -> 07 head->token relayout -> 08 o proj + residual -> 00 RMSNorm
    -> 09 gate_up proj -> 10 SiLU * mul -> 11 down proj + residual

wired over resident buffers (runtime/graph.py).  On one GPU the launches are the reference kernels' own
lowered objects (`objects`: launch name -> (kernel.json, desc blob)) or descriptors built for the shape.

Tensor parallel over `tp` GPUs (no counterpart in the reference, which runs one device): q/k/v and
gate_up are split by output columns (heads / intermediate), o and down by input rows; each rank's o and
down projections produce a partial sum and one NCCL all-reduce per row-parallel projection adds them
(two per layer), the residual added by rank 0's epilogue only.  RMSNorms and the RoPE tables are
replicated.  Shards: 32/tp query heads and 8/tp KV heads per rank (tp <= 8), 12288/tp intermediate."""
from ..codegen import build as B
from ..codegen import descriptors as D
from .graph import Graph

HIDDEN, HQ, HKV, DIM, INTER = 4096, 32, 8, 128, 12288


def weight_shapes(T):
    """Element counts of the layer's tensors (bf16 unless named fp32)."""
    return {"x": T * HIDDEN, "ln1": HIDDEN, "wq": HIDDEN * HQ * DIM, "wk": HIDDEN * HKV * DIM,
            "wv": HIDDEN * HKV * DIM, "qn": DIM, "kn": DIM, "wo": HQ * DIM * HIDDEN, "ln2": HIDDEN,
            "wgu": HIDDEN * 2 * INTER, "wd": INTER * HIDDEN}


def shard(p, rank, tp):
    """Rank `rank`'s shards of the full weights `p` (CPU tensors, [in, out] row-major as the bundle feeds
    them): column shards of wq/wk/wv/wgu (gate and up halves sharded alike), row shards of wo/wd."""
    import torch
    hq, hkv, it = HQ // tp, HKV // tp, INTER // tp

    def cols(w, rows, ncols, lo, hi):
        return w.view(rows, ncols)[:, lo:hi].contiguous().reshape(-1)

    def rows_(w, nrows, ncols, lo, hi):
        return w.view(nrows, ncols)[lo:hi].contiguous().reshape(-1)

    q0, k0, i0 = rank * hq * DIM, rank * hkv * DIM, rank * it
    gu = p["wgu"].view(HIDDEN, 2 * INTER)
    return {
        "ln1": p["ln1"], "ln2": p["ln2"], "qn": p["qn"], "kn": p["kn"],
        "wq": cols(p["wq"], HIDDEN, HQ * DIM, q0, q0 + hq * DIM),
        "wk": cols(p["wk"], HIDDEN, HKV * DIM, k0, k0 + hkv * DIM),
        "wv": cols(p["wv"], HIDDEN, HKV * DIM, k0, k0 + hkv * DIM),
        "wo": rows_(p["wo"], HQ * DIM, HIDDEN, q0, q0 + hq * DIM),
        "wgu": torch.cat([gu[:, i0:i0 + it], gu[:, INTER + i0:INTER + i0 + it]], dim=1).contiguous().reshape(-1),
        "wd": rows_(p["wd"], INTER, HIDDEN, i0, i0 + it),
    }


def build_layer(device, T, params, cos, sin, x, tp=1, rank=0, objects=None):
    """A Graph of one layer on `device` for `T` tokens (rank `rank` of `tp`).  `params` are this rank's
    (sharded when tp > 1) weights, `x` the input hidden states.  With tp > 1 the graph stops before each
    all-reduce: it returns the two segments and the caller all-reduces `x1` between them and `y` after."""
    hq, hkv, it = HQ // tp, HKV // tp, INTER // tp
    g = Graph(device)
    bf = "bfloat16"
    g.buffer("x", T * HIDDEN, bf, x)
    for n in ("ln1", "ln2", "qn", "kn", "wq", "wk", "wv", "wo", "wgu", "wd"):
        g.buffer(n, params[n].numel(), bf, params[n])
    g.buffer("cos", T * DIM, "float32", cos)
    g.buffer("sin", T * DIM, "float32", sin)
    for n, cnt in (("h", T * HIDDEN), ("q", T * hq * DIM), ("k", T * hkv * DIM), ("v", T * hkv * DIM),
                   ("qh", hq * T * DIM), ("kh", hkv * T * DIM), ("vh", hkv * T * DIM), ("o", hq * T * DIM),
                   ("ot", T * hq * DIM), ("x1", T * HIDDEN), ("h2", T * HIDDEN), ("gu", T * 2 * it),
                   ("a", T * it), ("y", T * HIDDEN)):
        g.buffer(n, cnt, bf)

    def obj(key, fallback):
        if objects and key in objects and tp == 1:
            return objects[key]
        return D.to_bytes(fallback())

    resid_o = rank == 0
    seg1 = [
        ("00_rmsnorm", obj("00", lambda: B.row_rmsnorm(T, HIDDEN, 1e-6)), ["x", "ln1", "h"]),
        ("01_q_mm", obj("01", lambda: B.gemm(T, hq * DIM, HIDDEN)), ["h", "wq", "q"]),
        ("02_qnorm_rope", obj("02", lambda: B.qknorm_rope(T, hq)), ["q", "qn", "cos", "sin", "qh"]),
        ("03_k_mm", obj("03", lambda: B.gemm(T, hkv * DIM, HIDDEN)), ["h", "wk", "k"]),
        ("04_knorm_rope", obj("04", lambda: B.qknorm_rope(T, hkv)), ["k", "kn", "cos", "sin", "kh"]),
        ("03_v_mm", obj("03", lambda: B.gemm(T, hkv * DIM, HIDDEN)), ["h", "wv", "v"]),
        ("05_v_relayout", obj("05", lambda: B.copy_map(T * hkv * DIM, T * hkv * DIM,
                                                       [(1, DIM, 1), (DIM, T, hkv * DIM), (T * DIM, hkv, DIM)])),
         ["v", "vh"]),
        ("06_attention", obj("06", lambda: B.attention(1, hq, hkv, T)), ["qh", "kh", "vh", "o"]),
        ("07_o_relayout", obj("07", lambda: B.copy_map(T * hq * DIM, T * hq * DIM,
                                                       [(1, DIM, 1), (DIM, hq, T * DIM), (hq * DIM, T, DIM)])),
         ["o", "ot"]),
    ]
    if resid_o:
        seg1.append(("08_o_mm_residual", obj("08", lambda: B.gemm(T, HIDDEN, hq * DIM, residual=True)),
                     ["x", "ot", "wo", "x1"]))
    else:
        seg1.append(("08_o_mm", D.to_bytes(B.gemm(T, HIDDEN, hq * DIM)), ["ot", "wo", "x1"]))
    seg2 = [
        ("00_rmsnorm_2", obj("00", lambda: B.row_rmsnorm(T, HIDDEN, 1e-6)), ["x1", "ln2", "h2"]),
        ("09_gate_up_mm", obj("09", lambda: B.gemm(T, 2 * it, HIDDEN)), ["h2", "wgu", "gu"]),
        ("10_silu_mul", obj("10", lambda: B.silu_mul(T, it)), ["gu", "a"]),
    ]
    if resid_o:
        seg2.append(("11_down_mm_residual", obj("11", lambda: B.gemm(T, HIDDEN, it, residual=True)),
                     ["x1", "a", "wd", "y"]))
    else:
        seg2.append(("11_down_mm", D.to_bytes(B.gemm(T, HIDDEN, it)), ["a", "wd", "y"]))
    if tp == 1:
        for name, blob, bufs in seg1 + seg2:
            g.add(name, blob, bufs)
        return g, None
    g1, g2 = g, Graph(device)
    g2.buffers = g.buffers
    for name, blob, bufs in seg1:
        g1.add(name, blob, bufs)
    for name, blob, bufs in seg2:
        g2.add(name, blob, bufs)
    return g1, g2


class TpLayer:
    """Rank `rank`'s share of the tensor-parallel layer with its two all-reduces overlapped with compute.

    The o projection and everything after it (RMSNorm, gate_up, SiLU * mul, down) treat token rows
    independently, so they run in `chunks` row blocks: the all-reduce of the o projection's block c goes
    out on a communication stream while block c + 1 is computed, the MLP of block c starts as soon as its
    reduced rows are in, and the all-reduce of the MLP's block c overlaps block c + 1.  Only the last
    block's all-reduce is exposed.  Each piece is a CUDA graph over the same resident buffers; the
    collective is the caller's (`all_reduce(tensor)`, e.g. torch.distributed.all_reduce over NCCL), issued
    on the communication stream.  Rows are cut into equal blocks (T % chunks == 0)."""

    def __init__(self, device, T, params, cos, sin, x, tp, rank, chunks=2):
        import torch
        if tp < 2 or T % chunks != 0:
            raise ValueError(f"TpLayer needs tp >= 2 and T divisible by chunks, got tp={tp}, T={T}, chunks={chunks}")
        self.torch = torch
        self.device = torch.device(device)
        self.chunks = chunks
        hq, it = HQ // tp, INTER // tp
        self.main, _ = build_layer(device, T, params, cos, sin, x, tp=tp, rank=rank)
        self.main.steps = [st for st in self.main.steps if not st[0].startswith("08_")]   # o proj goes by blocks
        bufs = self.main.buffers
        Tc = T // chunks
        self.o_parts, self.mlp_parts = [], []
        resid = rank == 0
        for c in range(chunks):
            def view(name, width):
                key = f"{name}@{c}"
                bufs[key] = bufs[name][c * Tc * width:(c + 1) * Tc * width]
                return key
            xc, otc, x1c = view("x", HIDDEN), view("ot", hq * DIM), view("x1", HIDDEN)
            h2c, guc, ac, yc = view("h2", HIDDEN), view("gu", 2 * it), view("a", it), view("y", HIDDEN)
            go = Graph(device)
            go.buffers = bufs
            if resid:
                go.add("08_o_mm_residual", D.to_bytes(B.gemm(Tc, HIDDEN, hq * DIM, residual=True)), [xc, otc, "wo", x1c])
            else:
                go.add("08_o_mm", D.to_bytes(B.gemm(Tc, HIDDEN, hq * DIM)), [otc, "wo", x1c])
            gm = Graph(device)
            gm.buffers = bufs
            gm.add("00_rmsnorm_2", D.to_bytes(B.row_rmsnorm(Tc, HIDDEN, 1e-6)), [x1c, "ln2", h2c])
            gm.add("09_gate_up_mm", D.to_bytes(B.gemm(Tc, 2 * it, HIDDEN)), [h2c, "wgu", guc])
            gm.add("10_silu_mul", D.to_bytes(B.silu_mul(Tc, it)), [guc, ac])
            if resid:
                gm.add("11_down_mm_residual", D.to_bytes(B.gemm(Tc, HIDDEN, it, residual=True)), [x1c, ac, "wd", yc])
            else:
                gm.add("11_down_mm", D.to_bytes(B.gemm(Tc, HIDDEN, it)), [ac, "wd", yc])
            self.o_parts.append((go, bufs[x1c]))
            self.mlp_parts.append((gm, bufs[yc]))
        self.buffers = bufs
        self.comm = torch.cuda.Stream(self.device)

    def graphs(self):
        return [self.main] + [g for g, _ in self.o_parts] + [g for g, _ in self.mlp_parts]

    def capture(self):
        for g in self.graphs():
            g.capture()

    def launch_count(self):
        return sum(g.launch_count() for g in self.graphs())

    def run(self, all_reduce):
        """Enqueue one layer on the current stream (compute) and the communication stream; returns with the
        current stream ordered after the last all-reduce."""
        torch = self.torch
        compute = torch.cuda.current_stream(self.device)
        comm = self.comm
        self.main.run()
        done_x1 = []
        for g, part in self.o_parts:
            g.run()
            ev = torch.cuda.Event()
            ev.record(compute)
            comm.wait_event(ev)
            with torch.cuda.stream(comm):
                all_reduce(part)
                e2 = torch.cuda.Event()
                e2.record(comm)
            done_x1.append(e2)
        for (g, part), ev_x1 in zip(self.mlp_parts, done_x1):
            compute.wait_event(ev_x1)
            g.run()
            ev = torch.cuda.Event()
            ev.record(compute)
            comm.wait_event(ev)
            with torch.cuda.stream(comm):
                all_reduce(part)
        compute.wait_stream(comm)


class TpLayerPeer:
    """Rank `rank`'s share of the tensor-parallel layer with its two all-reduces done by the executor's own kernels
    over NVLink peer memory instead of NCCL.  Every sum is over the ranks' bf16 partials in rank order in fp32 with
    one bf16 rounding, so both forms give the same bits on every rank and every run.

    fused=True: the o projection and the down projection push their output rows to the rank that owns them as
    they leave the tensor cores (ptsim_launch_rows_to_owners: rank q owns token rows [q T / tp, (q + 1) T / tp)
    and holds one staging slot per rank for them), so the reduce-scatter half of the all-reduce travels inside the
    GEMM; a second kernel (ptsim_tp_reduce_gather) sums each rank's staging from local memory and stores the rows
    into every rank's x1 (y).  fused=False: the GEMMs write a local partial and one kernel (ptsim_tp_allreduce)
    loads the owned rows of every rank's partial over NVLink, sums them and stores them everywhere.

    The collectives run on the compute stream, on grids sized to keep every owned row's loads in flight at once,
    and need no communication stream.  Buffers are set up once (runtime/peer.py PeerSet); the two graph segments
    are replayed from CUDA graphs.  Every rank of the process group builds it and calls run() the same number of
    times."""

    def __init__(self, device, T, params, cos, sin, x, tp, rank, group=None, fused=True):
        from . import native
        from .peer import PeerSet
        if tp < 2 or T % tp != 0:
            raise ValueError(f"TpLayerPeer needs tp >= 2 dividing T, got tp={tp}, T={T}")
        self.native = native
        self.T, self.tp, self.rank, self.fused = T, tp, rank, fused
        self.g1, self.g2 = build_layer(device, T, params, cos, sin, x, tp=tp, rank=rank)
        self.peers = PeerSet(device, tp, rank, group)
        bufs = self.g1.buffers
        # x1p / yp: the o and down projections' partials (fused: each rank's staging, tp slots of T / tp rows).
        for name in ("x1p", "x1", "yp", "y"):
            t, _ = self.peers.alloc(name, T * HIDDEN)
            bufs[name] = t
        self.peers.alloc("sig1", 64, "int32")
        self.peers.alloc("sig2", 64, "int32")
        R = T // tp
        slot = rank * R * HIDDEN * 2            # bytes: this rank's slot in every staging

        def redirect(g, step_prefix, old, new):
            for k, st in enumerate(g.steps):
                if not st[0].startswith(step_prefix):
                    continue
                if fused:   # the output argument stays `old` (not written); the rows go to the owners' staging
                    g.steps[k] = tuple(st[:5]) + (([p + slot for p in self.peers.ptrs[new]], R),)
                else:
                    g.steps[k] = (st[0], st[1], [new if b == old else b for b in st[2]]) + tuple(st[3:])
        redirect(self.g1, "08_", "x1", "x1p")     # the o projection (rank 0's with the residual)
        redirect(self.g2, "11_", "y", "yp")       # the down projection (rank 0's with the residual x1)
        self.buffers = bufs

    def capture(self):
        self.g1.capture()
        self.g2.capture()

    def launch_count(self):
        return self.g1.launch_count() + self.g2.launch_count() + 2

    def allreduce(self, part, out, sig, stream):
        p = self.peers.ptrs
        if self.fused:
            self.native.tp_reduce_gather(p[part][self.rank], p[out], p[sig], self.rank, self.T, HIDDEN, stream)
        else:
            self.native.tp_allreduce(p[part], p[out], p[sig], self.rank, self.T, HIDDEN, stream)

    def run(self):
        torch = self.peers.torch
        s = torch.cuda.current_stream(self.peers.device).cuda_stream
        self.g1.run()
        self.allreduce("x1p", "x1", "sig1", s)
        self.g2.run()
        self.allreduce("yp", "y", "sig2", s)

    def close(self):
        self.peers.close()


def layer_flops(T):
    """GEMM + causal attention flops of one layer (824,633,720,832 at T = 2048)."""
    gemm = 2 * T * HIDDEN * (HQ * DIM + 2 * HKV * DIM) + 2 * T * HQ * DIM * HIDDEN + 2 * T * HIDDEN * 2 * INTER \
        + 2 * T * INTER * HIDDEN
    attn = 4 * HQ * T * T * DIM // 2
    return gemm + attn


def random_params(seed=0):
    """Weights of the layer: linear weights N(0, 0.02), norm weights N(1, 0.02), bf16."""
    import torch
    g = torch.Generator().manual_seed(seed)
    out = {}
    for n, cnt in weight_shapes(1).items():
        if n == "x":
            continue
        std, mean = 0.02, (1.0 if n in ("ln1", "ln2", "qn", "kn") else 0.0)
        out[n] = (torch.randn(cnt, generator=g) * std + mean).to(torch.bfloat16)
    return out
