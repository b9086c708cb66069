"""Descriptor builders: launch descriptors of each executor class from plain shapes, for programs that
arrive without Triton source (a launch stated directly by a caller, as the reference's tests state
kernel.json manifests by hand in tests/runtime/spike_launch_cases.py:23-25).  The lowering
(targets/b200/lower.py) fills the same structures from a traced kernel."""
from . import descriptors as D


def _args(specs):
    return [{"name": n, "dtype": dt, "shape": [int(numel)]} for n, dt, numel in specs]


def elementwise_add(n, dtype="float32", block=1024):
    """o = x + y over n elements (tests/cases/smoke/add.py, scaled)."""
    d = D.new(D.ELEMENTWISE, _args([("x", dtype, n), ("y", dtype, n), ("o", dtype, n)]), [-(-n // block)],
              units=-(-n // block), unit_size=block)
    e = d.p.ew
    e.numel, e.nmap, e.store_map = n, 3, 2
    for i in range(3):
        m = e.map[i]
        m.arg, m.ndigit, m.offset = i, 1, 0
        m.div[0], m.mod[0], m.stride[0] = 1, max(1, n), 1
    prog = [("load", 0, 0, 0), ("load", 1, 1, 0), ("add", 2, 0, 1), ("store", 0, 2, 0)]
    e.ncode = len(prog)
    for i, (op, dst, a, b) in enumerate(prog):
        e.code[i].op, e.code[i].dst, e.code[i].a, e.code[i].b = D.OP[op], dst, a, b
    return d


def row_softmax(rows, cols, dtype="bfloat16", xblock=128):
    d = D.new(D.ROW_SOFTMAX, _args([("in_ptr0", dtype, rows * cols), ("out_ptr2", dtype, rows * cols)]),
              [-(-rows // xblock)], units=-(-rows // xblock), unit_size=xblock)
    r = d.p.row
    r.rows, r.cols, r.in_row_stride, r.out_row_stride = rows, cols, cols, cols
    r.in_arg, r.out_arg, r.weight_arg = 0, 1, -1
    return d


def row_rmsnorm(rows, cols, eps=1e-6, dtype="bfloat16", xblock=256):
    d = D.new(D.ROW_RMSNORM, _args([("in_ptr0", dtype, rows * cols), ("in_ptr1", dtype, cols),
                                    ("out_ptr1", dtype, rows * cols)]),
              [-(-rows // xblock)], units=-(-rows // xblock), unit_size=xblock)
    r = d.p.row
    r.rows, r.cols, r.in_row_stride, r.out_row_stride = rows, cols, cols, cols
    r.in_arg, r.weight_arg, r.out_arg, r.eps = 0, 1, 2, eps
    return d


def qknorm_rope(tokens, heads, dim=128, eps=1e-6, xblock=8192):
    rows = tokens * heads
    d = D.new(D.QKNORM_ROPE, _args([("in_ptr0", "bfloat16", rows * dim), ("in_ptr1", "bfloat16", dim),
                                    ("in_ptr2", "float32", tokens * dim), ("in_ptr3", "float32", tokens * dim),
                                    ("out_ptr2", "bfloat16", rows * dim)]),
              [-(-rows // xblock)], units=-(-rows // xblock), unit_size=xblock)
    q = d.p.qk
    q.tokens, q.heads, q.dim, q.eps = tokens, heads, dim, eps
    q.out_tok_stride, q.out_head_stride = dim, tokens * dim
    q.in_arg, q.weight_arg, q.cos_arg, q.sin_arg, q.out_arg = 0, 1, 2, 3, 4
    return d


def gemm(M, N, K, residual=False, b_kmajor=False, out_dtype="bfloat16"):
    """C[M,N] = A[M,K] . B (+ R[M,N]); B is [K,N] (the Inductor mm layout) or [N,K] when b_kmajor."""
    specs = ([("in_ptr0", "bfloat16", M * N)] if residual else []) + [
        ("arg_A", "bfloat16", M * K), ("arg_B", "bfloat16", K * N), ("out_ptr0", out_dtype, M * N)]
    d = D.new(D.GEMM, _args(specs), [1], units=M, unit_size=1)
    g = d.p.gemm
    off = 1 if residual else 0
    g.M, g.N, g.K = M, N, K
    g.lda, g.ldb, g.ldc, g.ldr = K, (K if b_kmajor else N), N, N
    g.a_arg, g.b_arg, g.c_arg, g.r_arg = off, off + 1, off + 2, (0 if residual else -1)
    g.b_kmajor = 1 if b_kmajor else 0
    return d


def attention(batch, hq, hkv, seq, dim=128, causal=True, scale=None, bq=1024, bkv=1024):
    import math
    scale = 1.0 / math.sqrt(dim) if scale is None else scale
    nq, nk = batch * hq * seq * dim, batch * hkv * seq * dim
    d = D.new(D.ATTN_PREFILL, _args([("q_ptr", "bfloat16", nq), ("k_ptr", "bfloat16", nk), ("v_ptr", "bfloat16", nk),
                                     ("o_ptr", "bfloat16", nq)]), [batch * hq], units=batch * hq, unit_size=1)
    a = d.p.attn
    a.batch, a.hq, a.hkv, a.seq, a.dim = batch, hq, hkv, seq, dim
    a.q_arg, a.k_arg, a.v_arg, a.o_arg = 0, 1, 2, 3
    a.causal, a.scale, a.ref_bq, a.ref_bkv = 1 if causal else 0, scale, min(bq, seq), min(bkv, seq)
    return d


def attention_decode(hkv, group, seq, dim=128, scale=None, bkv=None, gp=16):
    """The attention_decode_* program (validation/pytorchsim/attention_decode_32x8x4096_bf16/00__decode_kernel/
    _decode_kernel_triton.py): grid hkv, q/o [hkv, group, dim], k/v [hkv, seq, dim]."""
    nq, nk = hkv * group * dim, hkv * seq * dim
    d = D.new(D.ATTN_DECODE, _args([("q_ptr", "bfloat16", nq), ("k_ptr", "bfloat16", nk), ("v_ptr", "bfloat16", nk),
                                    ("o_ptr", "bfloat16", nq)]), (hkv, 1, 1), units=hkv, unit_size=1)
    a = d.p.attn
    a.batch, a.hq, a.hkv, a.seq, a.dim = 1, hkv * group, hkv, seq, dim
    a.q_arg, a.k_arg, a.v_arg, a.o_arg = 0, 1, 2, 3
    a.causal = 0
    import math
    a.scale = float(scale if scale is not None else 1.0 / math.sqrt(dim))
    a.ref_bq, a.ref_bkv = gp, int(bkv or seq)
    return d


def gemv(N, K, b_kmajor=False, residual=False, out_dtype="bfloat16"):
    """The gemm_1x* program (Inductor's M = 1 matmul, a multiply-reduce): out[n] = sum_k a[k] * B[k, n]."""
    return gemm(1, N, K, residual=residual, b_kmajor=b_kmajor, out_dtype=out_dtype)


class _Shapes:
    """The name and argument dtypes a fused-program generator reads of a kernel spec."""

    class _Arg:
        def __init__(self, dtype):
            self.dtype = dtype

    def __init__(self, name, dtypes):
        self.name, self.args = name, [self._Arg(dt) for dt in dtypes]


def _fused_gemv(name, specs, N, K, vec, epi=None, red=None):
    """An M = 1 matmul descriptor over argument `specs` whose vector is expression `vec` (front-end nodes over
    r) and, when given, whose stored value is `epi` with `red` standing for the sum: the programs are the
    ones the lowering emits for the same expressions (targets/b200/lower.py _vprog)."""
    from ..targets.b200 import lower as L
    shapes = _Shapes(name, [dt for _, dt, _ in specs])
    mat = next(i for i, (n, _, _) in enumerate(specs) if n == "mat")
    out = len(specs) - 1
    d = D.new(D.GEMM, _args(specs), (1, 1, 1), units=1, unit_size=1)
    g = d.p.gemm
    g.M, g.N, g.K = 1, N, K
    g.lda, g.ldb, g.ldc, g.ldr = K, N, N, N
    g.b_arg, g.c_arg, g.r_arg, g.b_kmajor = mat, out, -1, 0
    g.pro = L._vprog(shapes, vec, "r")
    g.a_arg = g.pro.load[0].arg
    if epi is not None:
        g.epi = L._vprog(shapes, epi, "x", acc=red)
    return d


def rmsnorm_gemv(N, K, eps=1e-6, residual=False):
    """The Qwen3 decode layer's RMSNorm'd matrix-vector product (qwen3_8b_layer_decode_*/01_*, 06_* with the
    residual row): out[n] = sum_k ((x[k] (+ res[k])) * rsqrt(ss / K + eps) * w[k]) * B[k, n], the vector in
    fp32; arguments x, (res,) ss (fp32 [1]), w, mat [K, N], out (bf16)."""
    from ..targets.b200 import frontend as F
    r = F.Index.var("r")
    specs = [("x", "bfloat16", K)] + ([("res", "bfloat16", K)] if residual else []) + \
        [("ss", "float32", 1), ("w", "bfloat16", K), ("mat", "bfloat16", K * N), ("out", "bfloat16", N)]
    i = {n: k for k, (n, _, _) in enumerate(specs)}
    x = F.Load(i["x"], r)
    if residual:
        x = F.Op("add", x, F.Load(i["res"], r))
    scale = F.Op("rsqrt", F.Op("add", F.Op("div", F.Load(i["ss"], F.Index()), F.Const(K)), F.Const(eps)))
    return _fused_gemv("rmsnorm_gemv", specs, N, K, F.Op("mul", F.Op("mul", x, scale), F.Load(i["w"], r)))


def silu_gemv(N, K):
    """The Qwen3 decode layer's down projection (qwen3_8b_layer_decode_*/07_*): out[n] = sum_k (silu(gu[k]) *
    gu[K + k]) * B[k, n] + (res1[n] + res2[n]); arguments gu [2K], mat [K, N], res1, res2, out (bf16)."""
    from ..targets.b200 import frontend as F
    r, x = F.Index.var("r"), F.Index.var("x")
    specs = [("gu", "bfloat16", 2 * K), ("mat", "bfloat16", K * N), ("res1", "bfloat16", N), ("res2", "bfloat16", N),
             ("out", "bfloat16", N)]
    gate = F.Load(0, r)
    silu = F.Op("div", gate, F.Op("add", F.Op("exp", F.Op("neg", gate)), F.Const(1.0)))
    vec = F.Op("mul", silu, F.Load(0, r + K))
    red = F.Reduce("add", F.Const(0.0))
    epi = F.Op("add", red, F.Op("add", F.Load(2, x), F.Load(3, x)))
    return _fused_gemv("silu_gemv", specs, N, K, vec, epi, red)


def sumsq(n, residual=False):
    """A sum of squares (qwen3_8b_layer_decode_*/00_*, 05_* with the residual row): out = sum (x (+ res))^2 in
    fp32; arguments x, (res,) out (fp32 [1])."""
    from ..targets.b200 import frontend as F
    from ..targets.b200 import lower as L
    r = F.Index.var("r")
    specs = [("x", "bfloat16", n)] + ([("res", "bfloat16", n)] if residual else []) + [("out", "float32", 1)]
    v = F.Load(0, r)
    if residual:
        v = F.Op("add", v, F.Load(1, r))
    d = D.new(D.REDUCE_ALL, _args(specs), [1], units=1, unit_size=1, workspace_bytes=D.REDUCE_WORKSPACE_BYTES)
    q = d.p.red
    q.pro = L._vprog(_Shapes("sumsq", [dt for _, dt, _ in specs]), F.Op("mul", v, v), "r")
    q.numel, q.in_arg, q.out_arg, q.op = n, 0, len(specs) - 1, D.RED_SUM
    return d


def topk(rows, cols, k, largest=True, cols_padded=None, dtype="float32"):
    """The MoE router's _topk_kernel (validation/pytorchsim/layer_op_router_post_*/01__topk_kernel): per row of
    `cols` values, the k largest (or smallest) with their column indices."""
    d = D.new(D.TOPK, _args([("x_ptr", dtype, rows * cols), ("v_ptr", dtype, rows * k), ("i_ptr", "int64", rows * k)]),
              (1, 1, 1), units=rows, unit_size=1)
    e = d.p.sel
    e.rows, e.cols, e.k = rows, cols, k
    e.cols_padded = cols_padded or 1 << max(0, (cols - 1).bit_length())
    e.in_arg, e.val_arg, e.idx_arg, e.descending = 0, 1, 2, 1 if largest else 0
    return d


def sort(rows, cols, descending=False, float_keys=False, dtype="int64"):
    """The MoE dispatch's _sort_kernel (validation/pytorchsim/layer_op_dispatch_*/00__sort_kernel): each row of
    `cols` keys sorted, ties in source order, with int64 source indices."""
    d = D.new(D.SORT, _args([("x_ptr", dtype, rows * cols), ("v_ptr", dtype, rows * cols), ("i_ptr", "int64", rows * cols)]),
              (rows, 1, 1), units=rows, unit_size=1)
    e = d.p.sel
    e.rows, e.cols, e.k, e.cols_padded = rows, cols, 0, 1 << max(0, (cols - 1).bit_length())
    e.in_arg, e.val_arg, e.idx_arg = 0, 1, 2
    e.descending, e.float_keys = 1 if descending else 0, 1 if float_keys else 0
    return d


def row_divsum(rows, cols, in_dtype="float32", out_dtype="bfloat16"):
    """The MoE router's weight normalisation (layer_op_router_post_*/02_*): out = x / sum(x) per row."""
    d = D.new(D.ROW_DIVSUM, _args([("in_ptr0", in_dtype, rows * cols), ("out_ptr1", out_dtype, rows * cols)]),
              (1, 1, 1), units=rows, unit_size=1)
    r = d.p.row
    r.rows, r.cols, r.in_row_stride, r.out_row_stride = rows, cols, cols, cols
    r.in_arg, r.out_arg, r.weight_arg = 0, 1, -1
    return d


def row_sum(rows, cols, dtype="float32"):
    """The MoE layer's per-token weight sums (layer_layer_prefill_*/22_*): out[r] = fp32 sum of row r."""
    d = D.new(D.ROW_SUM, _args([("in_ptr0", dtype, rows * cols), ("out_ptr0", "float32", rows)]),
              (1, 1, 1), units=rows, unit_size=1)
    r = d.p.row
    r.rows, r.cols, r.in_row_stride, r.out_row_stride = rows, cols, cols, 1
    r.in_arg, r.out_arg, r.weight_arg = 0, 1, -1
    return d


def gather_rows_floordiv(rows, cols, table_rows, div, dtype="bfloat16", idx_dtype="int64"):
    """The MoE dispatch's token copy (layer_op_dispatch_*/01_*): out row r = table row t, t = floor(idx[r] / div)
    (Python floor division), negative t wrapped by + table_rows; the int64 program as the lowering emits it."""
    d = D.new(D.GATHER_ROWS, _args([("in_ptr0", idx_dtype, rows), ("in_ptr1", dtype, table_rows * cols),
                                    ("out_ptr0", dtype, rows * cols)]), (1, 1, 1), units=rows, unit_size=1)
    g = d.p.gat
    g.rows, g.cols, g.table_rows = rows, cols, table_rows
    g.out_arg, g.table_arg, g.idx_arg = 2, 1, 0
    g.idx_map.arg, g.idx_map.ndigit, g.idx_map.offset = 0, 1, 0
    g.idx_map.div[0], g.idx_map.mod[0], g.idx_map.stride[0] = 1, 1 << 62, 1
    prog = [("load", 0, 0, 0, 0), ("const", 0, 0, 0, 0), ("lt", 0, 1, 0, 0), ("inv", 0, 0, 0, 0),
            ("where", 3, 0, 2, 0), ("const", 0, 0, 0, div), ("div", 4, 5, 0, 0), ("inv", 6, 0, 0, 0),
            ("where", 7, 6, 2, 0), ("lt", 8, 1, 0, 0), ("const", 0, 0, 0, table_rows), ("add", 8, 10, 0, 0),
            ("where", 11, 8, 9, 0)]
    for k, (op, a, b, c, imm) in enumerate(prog):
        ins = g.code[k]
        ins.op, ins.dst, ins.a, ins.b, ins.c, ins.imm = D.IOP[op], k, a, b, c, imm
    g.ncode = len(prog)
    return d


def grouped_gemm(M, N, K, groups, programs):
    """The MoE expert matmul (layer_op_gmm_*/05__grouped_mm_kernel): a [M, K], b [groups, K, N], int32 group /
    start / rows tables, c [M, N] (inout)."""
    d = D.new(D.GROUPED_GEMM, _args([("a_ptr", "bfloat16", M * K), ("b_ptr", "bfloat16", groups * K * N),
                                     ("group_ptr", "int32", programs), ("start_ptr", "int32", groups + 1),
                                     ("rows_ptr", "int32", groups + 1), ("c_ptr", "bfloat16", M * N)]),
              (programs, 1, 1), units=1, unit_size=1)
    q = d.p.ggemm
    q.M, q.N, q.K, q.groups, q.programs, q.ldb, q.ldg = M, N, K, groups, programs, N, K * N
    q.a_arg, q.b_arg, q.group_arg, q.start_arg, q.rows_arg, q.c_arg = 0, 1, 2, 3, 4, 5
    return d


def combine_gather_sum(tokens, hidden, topk, experts, fused=False):
    """The MoE combine's weighted gather (layer_op_combine_*/03_*): out[t, :] = sum over k of w[t, k] *
    expert_out[p(t, k), :], p = cum[e] - cnt[e] + pos[t, k] - 1 with e = idx[t, k] (both wrapped when
    negative); arguments idx, cum, cnt, pos (int64), expert_out, w (bf16), out (bf16).  fused: the MoE layer's
    form (layer_layer_*/23_*, 27_*): fp32 weights divided by the token's sum wsum[t], and out = (res + out) +
    the sum, out read first; arguments idx, cum, cnt, pos, expert_out, w (fp32), wsum (fp32), res, out."""
    rows = tokens * topk
    specs = [("in_ptr0", "int64", rows), ("in_ptr1", "int64", experts), ("in_ptr2", "int64", experts),
             ("in_ptr3", "int64", rows), ("in_ptr4", "bfloat16", rows * hidden)]
    if fused:
        specs += [("in_ptr5", "float32", rows), ("in_ptr6", "float32", tokens), ("in_ptr7", "bfloat16", tokens * hidden)]
    else:
        specs += [("in_ptr5", "bfloat16", rows)]
    specs += [("out_ptr1", "bfloat16", tokens * hidden)]
    d = D.new(D.GATHER_SUM, _args(specs), (1, 1, 1), units=tokens, unit_size=1)
    g = d.p.gsum
    g.rows, g.cols, g.terms, g.table_rows = tokens, hidden, topk, rows
    g.out_arg, g.table_arg, g.w_arg = len(specs) - 1, 4, 5
    if fused:
        g.wdiv, g.wdiv_arg, g.wdiv_offset, g.wdiv_stride = 1, 6, 0, 1
        g.nres, g.res_arg[0], g.res_arg[1] = 2, 7, len(specs) - 1

    def flat(m, arg):
        m.arg, m.ndigit, m.offset = arg, 1, 0
        m.div[0], m.mod[0], m.stride[0] = 1, 1 << 62, 1
    flat(g.w_map, 5)
    flat(g.maps[0], 0)
    flat(g.maps[1], 3)
    prog = [("load", 0, 0, 0, 0), ("const", 0, 0, 0, 0), ("lt", 0, 1, 0, 0), ("const", 0, 0, 0, experts),
            ("add", 0, 3, 0, 0), ("where", 4, 0, 2, 0), ("loadi", 5, 0, 1, 0), ("loadi", 5, 0, 2, 0),
            ("sub", 6, 7, 0, 0), ("load", 1, 0, 0, 0), ("const", 0, 0, 0, 1), ("sub", 9, 10, 0, 0),
            ("add", 8, 11, 0, 0), ("lt", 12, 1, 0, 0), ("const", 0, 0, 0, rows), ("add", 12, 14, 0, 0),
            ("where", 15, 12, 13, 0)]
    for k, (op, a, b, c, imm) in enumerate(prog):
        ins = g.code[k]
        ins.op, ins.dst, ins.a, ins.b, ins.c, ins.imm = D.IOP[op], k, a, b, c, imm
    g.ncode = len(prog)
    return d


_NOMOD = 1 << 62


def _int_table(args, rows, cols, maps, code, outs):
    """An INT_TABLE descriptor: maps [(offset, [(div, mod, stride), ...])], code [(op, a, b, c, imm)] (the
    destination of instruction k is register k), outs [(mode, arg, map, reg)]."""
    d = D.new(D.INT_TABLE, _args(args), (1, 1, 1), units=rows, unit_size=1)
    q = d.p.itab
    q.rows, q.cols, q.ncode, q.nout = rows, cols, len(code), len(outs)
    for i, (offset, digits) in enumerate(maps):
        m = q.maps[i]
        m.arg, m.offset, m.ndigit = -1, offset, len(digits)
        for k, (dv, md, sd) in enumerate(digits):
            m.div[k], m.mod[k], m.stride[k] = dv, md, sd
    for k, (op, a, b, c, imm) in enumerate(code):
        ins = q.code[k]
        ins.op, ins.dst, ins.a, ins.b, ins.c, ins.imm = D.IOP[op], k, a, b, c, imm
    for i, (mode, arg, mp, reg) in enumerate(outs):
        o = q.out[i]
        o.mode, o.arg, o.map, o.reg = D.ITAB_MODE[mode], arg, mp, reg
    return d


def expert_counts(n, experts):
    """The MoE combine's expert counts (layer_op_combine_*/00_*): ids [n] (int64) -> count [experts] and the
    inclusive running counts [n * experts] (expert x after routed row r at x + experts * r)."""
    return _int_table([("in_ptr0", "int64", n), ("out_ptr0", "int64", experts), ("out_ptr1", "int64", n * experts)],
                      experts, n, [(0, [(1, n, 1)]), (0, [(n, _NOMOD, 1)]), (0, [(1, n, experts), (n, _NOMOD, 1)])],
                      [("load", 0, 0, 0, 0), ("idx", 1, 0, 0, 0), ("eq", 0, 1, 0, 0)],
                      [("scan", 2, 2, 2), ("sum", 1, 1, 2)])


def cumsum_int(n, in_dtype="int64", out_dtype="int64"):
    """An integer running sum (layer_op_gmm_*/01_* in int32, layer_op_combine_*/01_* in int64)."""
    return _int_table([("in_ptr0", in_dtype, n), ("out_ptr0", out_dtype, n)], 1, n, [(0, [(1, n, 1)])],
                      [("load", 0, 0, 0, 0)], [("scan", 1, 0, 0)])


def slot_of(n, experts):
    """Each routed row's slot in its expert (layer_op_combine_*/02_*): out[x] = sum over r of
    running[r + experts * x] * (ids[x] == r); arguments running, ids, out (int64)."""
    e = experts
    return _int_table([("in_ptr0", "int64", n * e), ("in_ptr1", "int64", n), ("out_ptr0", "int64", n)], n, e,
                      [(0, [(1, e, 1), (e, _NOMOD, e)]), (0, [(e, _NOMOD, 1)]), (0, [(1, e, 1)])],
                      [("load", 0, 0, 0, 0), ("load", 1, 0, 1, 0), ("idx", 2, 0, 0, 0), ("eq", 1, 2, 0, 0),
                       ("mul", 0, 3, 0, 0)],
                      [("sum", 2, 1, 4)])


def group_tables(n):
    """The grouped matmul's group tables (layer_op_gmm_*/02_*) from the running offsets o [n] (int32):
    nonempty = cumsum(o[r] - o[r - 1] > 0), prev = o[r - 1] (0 at r = 0), count = o[r] - prev (int64)."""
    return _int_table([("in_ptr0", "int32", n), ("out_ptr0", "int64", n), ("out_ptr1", "int64", n),
                       ("out_ptr2", "int64", n)], 1, n, [(0, [(1, n, 1)]), (-1, [(1, n, 1)])],
                      [("load", 0, 0, 0, 0), ("idx", 0, 0, 0, 0), ("const", 0, 0, 0, 1), ("lt", 1, 2, 0, 0),
                       ("const", 0, 0, 0, 0), ("where", 4, 4, 3, 0), ("ge", 1, 2, 0, 0), ("loadm", 1, 6, 0, 0),
                       ("where", 7, 4, 6, 0), ("where", 5, 8, 3, 0), ("sub", 0, 9, 0, 0), ("gt", 10, 4, 0, 0)],
                      [("scan", 1, 0, 11), ("elem", 2, 0, 9), ("elem", 3, 0, 10)])


def count_le(n, rows, in_dtype="int64", out_dtype="int32"):
    """Groups at or below each expert (layer_op_gmm_*/03_*): out[x] = the number of r < n with v[r] <= x."""
    return _int_table([("in_ptr0", in_dtype, n), ("out_ptr1", out_dtype, rows)], rows, n,
                      [(0, [(1, n, 1)]), (0, [(n, _NOMOD, 1)])],
                      [("load", 0, 0, 0, 0), ("idx", 1, 0, 0, 0), ("le", 0, 1, 0, 0)],
                      [("sum", 1, 1, 2)])


def reduce_all(numel, op="sum", dtype="bfloat16"):
    d = D.new(D.REDUCE_ALL, _args([("in_ptr0", dtype, numel), ("out_ptr0", "float32", 1)]), [1], units=1, unit_size=1,
              workspace_bytes=D.REDUCE_WORKSPACE_BYTES)
    r = d.p.red
    r.numel, r.in_arg, r.out_arg, r.op = numel, 0, 1, (D.RED_MAX if op == "max" else D.RED_SUM)
    return d


def copy_map(in_numel, out_numel, digits, dtype="bfloat16", block=None):
    """out[i] = in[sum ((i // div) % mod) * stride] (a relayout DMA), digits = [(div, mod, stride), ...]."""
    block = block or out_numel
    d = D.new(D.ELEMENTWISE, _args([("in_ptr0", dtype, in_numel), ("out_ptr0", dtype, out_numel)]),
              [-(-out_numel // block)], units=-(-out_numel // block), unit_size=block)
    e = d.p.ew
    e.numel, e.nmap, e.store_map, e.pure_copy = out_numel, 2, 1, 1
    m = e.map[0]
    m.arg, m.ndigit, m.offset = 0, len(digits), 0
    for k, (dv, md, st) in enumerate(sorted(digits)):
        m.div[k], m.mod[k], m.stride[k] = dv, md, st
    s = e.map[1]
    s.arg, s.ndigit, s.offset = 1, 1, 0
    s.div[0], s.mod[0], s.stride[0] = 1, out_numel, 1
    prog = [("load", 0, 0, 0), ("store", 0, 0, 0)]
    e.ncode = 2
    for i, (op, dst, a, b) in enumerate(prog):
        e.code[i].op, e.code[i].dst, e.code[i].a, e.code[i].b = D.OP[op], dst, a, b
    return d


def silu_mul(tokens, inter, block=2097152):
    n = tokens * inter
    d = D.new(D.ELEMENTWISE, _args([("in_ptr0", "bfloat16", 2 * n), ("out_ptr0", "bfloat16", n)]),
              [-(-n // block)], units=-(-n // block), unit_size=block)
    e = d.p.ew
    e.numel, e.nmap, e.store_map = n, 3, 2
    # gate = in[x % inter + 2*inter * (x // inter)], up = the same + inter
    for i, off in enumerate((0, inter)):
        m = e.map[i]
        m.arg, m.ndigit, m.offset = 0, 2, off
        m.div[0], m.mod[0], m.stride[0] = 1, inter, 1
        m.div[1], m.mod[1], m.stride[1] = inter, tokens, 2 * inter
    s = e.map[2]
    s.arg, s.ndigit, s.offset = 1, 1, 0
    s.div[0], s.mod[0], s.stride[0] = 1, n, 1
    prog = [("load", 0, 0, 0, 0.0), ("neg", 1, 0, 0, 0.0), ("exp", 1, 1, 1, 0.0), ("const", 2, 0, 0, 1.0),
            ("add", 2, 1, 2, 0.0), ("div", 2, 0, 2, 0.0), ("load", 0, 1, 0, 0.0), ("mul", 0, 2, 0, 0.0),
            ("store", 0, 0, 0, 0.0)]
    e.ncode = len(prog)
    for i, (op, dst, a, b, imm) in enumerate(prog):
        e.code[i].op, e.code[i].dst, e.code[i].a, e.code[i].b, e.code[i].imm = D.OP[op], dst, a, b, imm
    return d
