"""Lowering of a traced tile program into a B200 launch descriptor (the bridge from the reference's L3
compiler to a CUDA L1): the program's class decides which executor kernel runs it, and the program's index
maps, constants and argument roles fill that kernel's descriptor.

Classes (each with the reference program it was written against):
  ELEMENTWISE   Inductor pointwise kernels and tests/cases smoke/add.py: loads at affine index maps of the
                flat launch index, fp32 vector ops, one store.  Compiled to the executor's vector program.
  ROW_SOFTMAX   vector_softmax_* (validation/pytorchsim/vector_softmax_4096x4096_bf16/00_*).
  ROW_RMSNORM   qwen3_8b_layer_prefill_*/00_* (mean of squares, rsqrt(mean + eps), times weight).
  QKNORM_ROPE   qwen3_8b_layer_prefill_*/02_*, 04_* (per-head RMSNorm, rotary embedding, head-major store).
  REDUCE_ALL    vector_sum_*, vector_max_* (a whole tensor to one fp32 value).
  GEMM          every kernel with one tl.dot: gemm_*, Qwen3 01/03/08/09/11 (with a residual epilogue).
  ATTN_PREFILL  _prefill_kernel (causal GQA flash attention).
A program none of these match is refused with a Reason; nothing runs anywhere else."""
import ast
import math
import re

from ...codegen import descriptors as D
from ...contract.stop import Reason, Refused
from . import frontend as F


class Lowered:
    """A lowered kernel: the descriptor, its class name and a JSON-able summary."""

    def __init__(self, desc, summary):
        self.desc = desc
        self.blob = D.to_bytes(desc)
        self.summary = summary

    @property
    def kind(self):
        return self.summary["kind"]


def _manifest_args(spec):
    return [{"name": a.name, "dtype": a.dtype, "shape": list(a.shape)} for a in spec.args]


def _lookup(spec, prog, *names, default=None):
    """A size the program states: a constant assigned in its body, a constexpr, or a scalar value."""
    for n in names:
        if prog is not None and n in prog.assigned:
            return prog.assigned[n]
        if n in spec.constexprs and isinstance(spec.constexprs[n], (int, float)):
            return spec.constexprs[n]
        sv = spec.extra.get("scalar_values", {})
        if n in sv and sv[n] is not None:
            return sv[n]
    return default


def _grid_programs(spec):
    g = (list(spec.grid) + [1, 1, 1])[:3]
    return g


# ---------------------------------------------------------------------------------------------------
# Structural helpers over the value DAG
# ---------------------------------------------------------------------------------------------------

def key(n):
    """A canonical, hashable form of value node `n` (structural equality)."""
    if isinstance(n, F.Const):
        return ("c", n.v)
    if isinstance(n, F.Load):
        return ("l", n.arg, tuple(sorted(n.index.terms.items())), n.index.const, n.mask is not None)
    if isinstance(n, F.Op):
        return ("o", n.name) + tuple(key(a) if isinstance(a, F.Node) else _cond_key(a) for a in n.args)
    if isinstance(n, F.Reduce):
        return ("r", n.op, key(n.value))
    if isinstance(n, F.IndexValue):
        return ("i", tuple(sorted(n.index.terms.items())), n.index.const)
    if isinstance(n, F.Dot):
        return ("d", key(n.a), key(n.b))
    return ("?", id(n))


def _cond_key(c):
    """A hashable form of a mask / condition operand (index comparisons by their index and bound)."""
    if not isinstance(c, F.Cond):
        return ("m",)
    idx = (tuple(sorted(c.index.terms.items())), c.index.const) if isinstance(c.index, F.Index) else None
    val = key(c.value) if isinstance(c.value, F.Node) else c.value
    return ("m", c.op, idx, val, tuple(_cond_key(p) for p in c.parts))


def walk(n, seen=None):
    """Every node reachable from `n` (pre-order, once each)."""
    seen = set() if seen is None else seen
    if id(n) in seen:
        return
    seen.add(id(n))
    yield n
    if isinstance(n, F.Op):
        for a in n.args:
            if isinstance(a, F.Node):
                yield from walk(a, seen)
    elif isinstance(n, (F.Reduce, F.Scan, F.ChunkLast)):
        yield from walk(n.value, seen)
    elif isinstance(n, F.Dot):
        yield from walk(n.a, seen)
        yield from walk(n.b, seen)


def strip_casts(n):
    """`n` without round-trips through fp32 (Inductor's repeated .to(tl.float32))."""
    return n


def _row_index(idx, what, rows=None):
    """(row stride) of an index r + stride * x, else Refused.  A one-row program (xnumel 1: Inductor then
    indexes by r alone) has row stride 0."""
    r = idx.coeff_of("r")
    x = idx.coeff_of("x")
    if rows == 1 and idx.const == 0 and r == {F.Digit("r"): 1} and not x and len(idx.terms) == 1:
        return 0
    if idx.const != 0 or r != {F.Digit("r"): 1} or len(x) != 1 or F.Digit("x") not in x or len(idx.terms) != 2:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{what} index {idx} is not r + stride * x")
    return x[F.Digit("x")]


# ---------------------------------------------------------------------------------------------------
# Classes
# ---------------------------------------------------------------------------------------------------

def lower(spec, fn=None):
    """The Lowered kernel of `spec` (a contract.kernel_spec.KernelSpec), or Refused."""
    if fn is None:
        fn = F.load_kernel(spec)
    src, name = F.kernel_source(fn)
    tree = ast.parse(src)
    ce = set(spec.constexprs)
    if {"E", "EP", "K", "KP", "XBLOCK", "LARGEST"} <= ce:
        return _lower_topk(spec)
    if {"L", "D", "LOG", "DESCENDING", "FLOAT"} <= ce:
        return _lower_sort(spec)
    if {"sbg", "sbk", "sbn", "K", "KP", "N", "BM", "BN", "BK"} <= ce:
        return _lower_grouped_gemm(spec)
    dots = [n for n in ast.walk(tree) if isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute) and n.func.attr == "dot"]
    if dots:
        if len(dots) >= 2 and {"HQ", "G", "S", "D", "SCALE"} <= set(spec.constexprs):
            return _lower_attention(spec, tree)
        if len(dots) >= 2 and {"HKV", "G", "GP", "S", "D", "BKV", "SCALE"} <= set(spec.constexprs):
            return _lower_decode(spec, tree)
        return _lower_gemm(spec, tree, src)
    prog = F.Evaluator(spec, F.Program(), F.kernel_globals(fn)).run(src, name)
    if prog.stores and all(spec.args[st.arg].dtype in _INT_TYPES for st in prog.stores) and any(
            isinstance(n, (F.Scan, F.Reduce, F.Carry, F.ChunkLast)) for st in prog.stores for n in walk(st.value)):
        return _lower_int_table(spec, prog)
    if len(prog.stores) != 1:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {len(prog.stores)} stores; the executor's "
                                                    f"vector programs have one")
    st = prog.stores[0]
    if isinstance(strip_casts(st.value), F.Load) and strip_casts(st.value).data is not None:
        return _lower_gather(spec, prog, st)
    sums = [n for n in walk(st.value) if isinstance(n, F.Reduce)]
    sv = sums[0] if len(sums) == 1 else None
    if sv is not None and sv.op == "add" and isinstance(strip_casts(sv.value), F.Op) \
            and strip_casts(sv.value).name == "mul" and any(isinstance(strip_casts(a), F.Load) and strip_casts(a).data is not None
                                                            for a in strip_casts(sv.value).args):
        return _lower_gather_sum(spec, prog, st, sv)
    reduces = [n for n in walk(st.value) if isinstance(n, F.Reduce)]
    if not reduces:
        if any(isinstance(n, F.Op) and n.name == "where" for n in walk(st.value)) and \
                len({n.arg for n in walk(st.value) if isinstance(n, F.Load)}) == 3:
            return _lower_rope(spec, prog, st)
        return _lower_elementwise(spec, prog, st)
    ops = {n.name for n in walk(st.value) if isinstance(n, F.Op)}
    loads = [n for n in walk(st.value) if isinstance(n, F.Load)]
    args = {l.arg for l in loads}
    if not st.index.terms:
        return _lower_reduce_all(spec, prog, st, reduces)
    if _gemv_parts(st, reduces) is not None:
        return _lower_gemv(spec, prog, st, reduces[0])
    if "where" in ops and "rsqrt" in ops:
        return _lower_qknorm_rope(spec, prog, st, loads)
    if "rsqrt" in ops and len(args) in (2, 3):
        return _lower_rmsnorm(spec, prog, st, loads)
    if "exp" in ops and {r.op for r in reduces} == {"max", "add"} and len(args) == 1:
        return _lower_softmax(spec, prog, st, reduces)
    if ops == {"div"} and len(reduces) == 1 and reduces[0].op == "add" and len(args) == 1:
        return _lower_divsum(spec, prog, st, reduces[0])
    if not ops and st.value is reduces[0] and reduces[0].op == "add" and len(args) == 1:
        return _lower_rowsum(spec, prog, st, reduces[0])
    raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a reduction program of ops {sorted(ops)}")


def _lower_elementwise(spec, prog, st):
    xnumel = _lookup(spec, prog, "xnumel", "n", "N", "numel")
    gx, gy, gz = _grid_programs(spec)
    if gy != 1 or gz != 1:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: a pointwise program over a {gx}x{gy}x{gz} grid")
    block = prog.block.get("x")
    if block is None:
        # No pid * BLOCK + arange index: one program covers the whole (possibly broadcast) store.
        block = max(1, spec.args[st.arg].numel if not st.index.terms else spec.args[st.arg].numel)
    numel = gx * block
    if xnumel is not None:
        numel = min(numel, int(xnumel))
    if st.mask is not None:
        raise Refused(Reason.MASKED_STORE_NOT_A_BOX, f"{spec.name}: a masked pointwise store")
    maps, code = [], []

    def map_of(arg, idx):
        if idx.vars() - {"x"}:
            raise Refused(Reason.INDEX_NOT_AFFINE, f"{spec.name}: index {idx} uses {sorted(idx.vars())}")
        m = D.Map()
        m.arg = arg
        m.offset = idx.const
        digits = list(idx.terms.items())
        if len(digits) > D.MAX_DIGITS:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: an index of {len(digits)} digits")
        digits.sort(key=lambda dc: dc[0].div)
        m.ndigit = len(digits)
        for k, (dg, c) in enumerate(digits):
            if c < 0:
                raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: a negative stride in {idx}")
            m.div[k] = dg.div
            m.mod[k] = dg.mod if dg.mod is not None else max(1, -(-numel // dg.div))
            m.stride[k] = c
        if len(maps) >= D.MAX_MAPS:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: more than {D.MAX_MAPS} transfers")
        maps.append(m)
        return len(maps) - 1

    # Register allocation over the DAG: each node's value is computed once; a register is freed after the
    # last use of the node it holds.
    uses = {}
    for n in walk(st.value):
        for a in (n.args if isinstance(n, F.Op) else ()):
            if isinstance(a, F.Node):
                uses[id(a)] = uses.get(id(a), 0) + 1
    reg_of, free = {}, list(range(D.MAX_REGS))[::-1]

    def emit(op, dst=0, a=0, b=0, imm=0.0):
        if len(code) >= D.MAX_CODE:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: a vector program over {D.MAX_CODE} ops")
        ins = D.Insn()
        ins.op, ins.dst, ins.a, ins.b, ins.imm = D.OP[op], dst, a, b, imm
        code.append(ins)

    def release(n):
        uses[id(n)] -= 1
        if uses[id(n)] == 0:
            free.append(reg_of.pop(id(n)))

    def take():
        if not free:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: more than {D.MAX_REGS} live values")
        return free.pop()

    def gen(n):
        if id(n) in reg_of:
            return reg_of[id(n)]
        if isinstance(n, F.Load):
            if n.mask is not None:
                raise Refused(Reason.MASKED_BOX_BEFORE_TENSOR, f"{spec.name}: a masked pointwise load")
            r = take()
            emit("load", r, map_of(n.arg, n.index))
        elif isinstance(n, F.Const):
            r = take()
            emit("const", r, imm=n.v)
        elif isinstance(n, F.Op):
            if n.name == "sigmoid":
                x = n.args[0]
                one = F.Const(1.0)
                return gen(_retarget(n, F.Op("div", one, F.Op("add", one, F.Op("exp", F.Op("neg", x)))), uses))
            if n.name not in D.OP or n.name in ("load", "const", "store"):
                raise Refused(Reason.MATH_UNLOWERED, f"{spec.name}: vector op {n.name}")
            srcs = [gen(a) for a in n.args]
            for a in n.args:
                release(a)
            r = take()
            emit(n.name, r, srcs[0], srcs[1] if len(srcs) > 1 else srcs[0])
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a {type(n).__name__} in a pointwise program")
        reg_of[id(n)] = r
        uses.setdefault(id(n), 0)
        return r

    uses[id(st.value)] = uses.get(id(st.value), 0) + 1
    out_reg = gen(st.value)
    store_map = map_of(st.arg, st.index)
    emit("store", 0, out_reg)
    d = D.new(D.ELEMENTWISE, _manifest_args(spec), spec.grid, units=gx, unit_size=block)
    e = d.p.ew
    e.numel = numel
    e.nmap, e.ncode, e.store_map = len(maps), len(code), store_map
    for i, m in enumerate(maps):
        e.map[i] = m
    for i, c in enumerate(code):
        e.code[i] = c
    # A pure copy: the stored value is one load, of the store's dtype.
    v = st.value
    if isinstance(v, F.Op) and v.name == "rbf16" and spec.args[st.arg].dtype == "bfloat16":
        v = v.args[0]
    if isinstance(v, F.Load) and spec.args[v.arg].dtype == spec.args[st.arg].dtype and len(maps) == 2:
        e.pure_copy = 1
        # Map 0 must be the load for the copy kernel.
        if maps[0].arg != v.arg:
            e.map[0], e.map[1] = maps[1], maps[0]
            e.store_map = 0 if store_map == 1 else 1
    summary = D.describe(d)
    return Lowered(d, summary)


def _retarget(old, new, uses):
    uses[id(new)] = uses.get(id(old), 1)
    for n in walk(new):
        for a in (n.args if isinstance(n, F.Op) else ()):
            if isinstance(a, F.Node):
                uses[id(a)] = uses.get(id(a), 0) + 1
    return new


def _row_sizes(spec, prog, what):
    rows = _lookup(spec, prog, "xnumel")
    cols = _lookup(spec, prog, "r0_numel", "rnumel")
    xblock = _lookup(spec, prog, "XBLOCK")
    if rows is None or cols is None or xblock is None:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: {what} without xnumel/r0_numel/XBLOCK")
    return int(rows), int(cols), int(xblock)


def _lower_softmax(spec, prog, st, reduces):
    rows, cols, xblock = _row_sizes(spec, prog, "softmax")
    v = st.value
    if not (isinstance(v, F.Op) and v.name == "div" and isinstance(v.args[1], F.Reduce) and v.args[1].op == "add"):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: not exp(x - max) / sum")
    num = v.args[0]
    if not (isinstance(num, F.Op) and num.name == "exp" and key(num) == key(v.args[1].value)):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the softmax numerator is not the summed exp")
    sub = num.args[0]
    if not (isinstance(sub, F.Op) and sub.name == "sub" and isinstance(sub.args[1], F.Reduce) and sub.args[1].op == "max"
            and isinstance(sub.args[0], F.Load) and key(sub.args[1].value) == key(sub.args[0])):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: not exp(x - rowmax(x))")
    ld = sub.args[0]
    d = D.new(D.ROW_SOFTMAX, _manifest_args(spec), spec.grid, units=_grid_programs(spec)[0], unit_size=xblock)
    r = d.p.row
    r.rows, r.cols = rows, cols
    r.in_row_stride = _row_index(ld.index, "softmax load", rows)
    r.out_row_stride = _row_index(st.index, "softmax store", rows)
    r.in_arg, r.out_arg, r.weight_arg = ld.arg, st.arg, -1
    return Lowered(d, D.describe(d))


def _lower_rmsnorm(spec, prog, st, loads):
    """(x * rsqrt(sum(x^2) / cols + eps)) * w per row (qwen3_8b_layer_prefill_*/00_*); x may be the fp32 sum of
    two rows, unrounded (the MoE layer's residual add, layer_layer_prefill_*/18_*), and a one-row program
    indexes its row by r alone (layer_op_rmsnorm_1x0_bf16)."""
    rows, cols, xblock = _row_sizes(spec, prog, "RMSNorm")
    rs = [n for n in walk(st.value) if isinstance(n, F.Op) and n.name == "rsqrt"]
    inner = rs[0].args[0]
    if not (isinstance(inner, F.Op) and inner.name == "add" and isinstance(inner.args[1], F.Const)):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: rsqrt of something other than mean + eps")
    eps = inner.args[1].v
    mean = inner.args[0]
    if not (isinstance(mean, F.Op) and mean.name == "div" and isinstance(mean.args[0], F.Reduce)
            and isinstance(mean.args[1], F.Const) and mean.args[1].v == float(cols)):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the mean is not sum / {cols}")
    sq = mean.args[0].value
    if not (isinstance(sq, F.Op) and sq.name == "mul" and key(sq.args[0]) == key(sq.args[1])):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the reduced value is not x * x")
    xv = sq.args[0]
    if isinstance(xv, F.Load):
        row, res = xv, None
    elif isinstance(xv, F.Op) and xv.name == "add" and all(isinstance(a, F.Load) for a in xv.args) \
            and xv.args[0].arg != xv.args[1].arg and key(F.Load(0, xv.args[0].index)) == key(F.Load(0, xv.args[1].index)):
        row, res = xv.args
    else:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: RMSNorm of something other than a row or a row sum")
    if row.mask is not None or (res is not None and res.mask is not None):
        raise Refused(Reason.MASKED_BOX_BEFORE_TENSOR, f"{spec.name}: a masked RMSNorm row")
    row_args = {row.arg} | ({res.arg} if res is not None else set())
    w_args = {l.arg for l in loads} - row_args
    if len(w_args) != 1:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: RMSNorm wants one row input and one weight")
    w_arg = w_args.pop()
    if any(l.arg == w_arg and l.index.vars() != {"r"} for l in loads):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the RMSNorm weight is not a row over r")
    d = D.new(D.ROW_RMSNORM, _manifest_args(spec), spec.grid, units=_grid_programs(spec)[0], unit_size=xblock)
    r = d.p.row
    r.rows, r.cols, r.eps = rows, cols, eps
    r.in_row_stride = _row_index(row.index, "RMSNorm load", rows)
    r.out_row_stride = _row_index(st.index, "RMSNorm store", rows)
    r.in_arg, r.out_arg, r.weight_arg = row.arg, st.arg, w_arg
    if res is not None:
        r.res_arg_p1 = res.arg + 1
    return Lowered(d, D.describe(d))


def _lower_qknorm_rope(spec, prog, st, loads):
    rows, cols, xblock = _row_sizes(spec, prog, "QK-norm+RoPE")
    if cols != 128:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: head_dim {cols}; the executor runs 128")
    dt = {a: spec.args[a].dtype for a in {l.arg for l in loads}}
    f32 = sorted(a for a, t in dt.items() if t == "float32")
    bf = sorted(a for a, t in dt.items() if t == "bfloat16")
    if len(f32) != 2 or len(bf) != 2:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: QK-norm+RoPE wants bf16 x, w and fp32 cos, sin")
    x_arg = next(l.arg for l in loads if l.arg in bf and "x" in l.index.vars())
    w_arg = next(a for a in bf if a != x_arg)
    # cos multiplies the normalised row, sin the rotated one (the branch holding the where).
    v = st.value
    if not (isinstance(v, F.Op) and v.name == "add" and all(isinstance(a, F.Op) and a.name == "mul" for a in v.args)):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: not n * cos + rot * sin")
    cos_arg = sin_arg = None
    for m in v.args:
        tab = [a for a in m.args if isinstance(a, F.Load) and a.arg in f32]
        if len(tab) != 1:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a rotary product without its table")
        other = [a for a in m.args if a is not tab[0]][0]
        if any(isinstance(n, F.Op) and n.name == "where" for n in walk(other)):
            sin_arg, sin_load = tab[0].arg, tab[0]
        else:
            cos_arg = tab[0].arg
    if cos_arg is None or sin_arg is None:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: cannot tell the cos table from the sin table")
    tdig = [dg for dg in sin_load.index.terms if dg.var == "x"]
    if not tdig:
        # One token (the decode layer, qwen3_8b_layer_decode_*/02_*): every row is a head and the tables are
        # the one position's, indexed by r alone; the store index is r + h * H.
        heads, tok = rows, 0
        head = st.index.terms.get(F.Digit("x"))
        if head is None or st.index.terms.get(F.Digit("r")) != 1 or len(st.index.terms) != 2 or st.index.const:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: the store index {st.index} is not r + h*H")
    else:
        if len(tdig) != 1 or tdig[0].mod is not None:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: the table index is not x // heads")
        heads = tdig[0].div
        tok = st.index.terms.get(F.Digit("x", heads, None))
        head = st.index.terms.get(F.Digit("x", 1, heads))
        if tok is None or head is None or st.index.terms.get(F.Digit("r")) != 1:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: the store index {st.index} is not r + t*T + h*H")
    rs = [n for n in walk(v) if isinstance(n, F.Op) and n.name == "rsqrt"]
    inner = rs[0].args[0]
    if not (isinstance(inner, F.Op) and inner.name == "add" and isinstance(inner.args[1], F.Const)):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: rsqrt of something other than mean + eps")
    d = D.new(D.QKNORM_ROPE, _manifest_args(spec), spec.grid, units=_grid_programs(spec)[0], unit_size=xblock)
    q = d.p.qk
    q.tokens, q.heads, q.dim = rows // heads, heads, cols
    q.out_tok_stride, q.out_head_stride = tok, head
    q.in_arg, q.weight_arg, q.cos_arg, q.sin_arg, q.out_arg = x_arg, w_arg, cos_arg, sin_arg, st.arg
    q.eps = inner.args[1].v
    return Lowered(d, D.describe(d))


def _lower_rope(spec, prog, st):
    """The rotary embedding alone (validation/pytorchsim/layer_op_rope_{q,k}_*/00_*_triton.py): over [T, H, 128]
    rows, out = x * cos[t] + rot * sin[t], rot = cat(-x[64:], x[:64]) per row, the fp32 tables per token
    (index d + 128 * t).  The QK-norm + RoPE kernel with its norm off."""
    v = st.value
    if not (isinstance(v, F.Op) and v.name == "add" and all(isinstance(a, F.Op) and a.name == "mul" for a in v.args)):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: not x * cos + rot * sin")
    flat = {F.Digit("x"): 1}
    d_of = F.Digit("x", 1, 128)
    row_of = F.Digit("x", 128, None)
    x = cos = sin = rot = None
    for m in v.args:
        tab = [a for a in m.args if isinstance(a, F.Load) and spec.args[a.arg].dtype == "float32"]
        if len(tab) != 1:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a rotary product without its table")
        other = next(a for a in m.args if a is not tab[0])
        if any(isinstance(n, F.Op) and n.name == "where" for n in walk(other)):
            sin, rot = tab[0], other
        else:
            cos, x = tab[0], other
    if x is None or rot is None or not isinstance(x, F.Load) or x.index.const != 0 or x.index.terms != flat \
            or x.mask is not None or spec.args[x.arg].dtype != "bfloat16":
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the rotated rows are not one bf16 load at x")
    numel = int(_lookup(spec, prog, "xnumel") or spec.args[st.arg].numel)
    tdig = [dg for dg in cos.index.terms if dg != d_of]
    one_token = not tdig and cos.index.terms == {d_of: 1}   # T = 1: the one position's tables, indexed by d
    if cos.index.const != 0 or cos.index.terms.get(d_of) != 1 or key(F.Load(0, cos.index)) != key(F.Load(0, sin.index)) \
            or not (one_token or (len(tdig) == 1 and tdig[0].mod is None and cos.index.terms[tdig[0]] == 128)):
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: table index {cos.index} is not d + 128 * t")
    hd = numel if one_token else tdig[0].div
    if hd % 128:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: tokens of {hd} values are not whole heads")
    # rot: where(d < 64, -x[row, d + 64], x[row, d - 64]) over the same rows
    rloads = [n for n in walk(rot) if isinstance(n, F.Load)]
    negs = [n for n in walk(rot) if isinstance(n, F.Op) and n.name == "neg"]
    ops = {n.name for n in walk(rot) if isinstance(n, F.Op)}
    conds = [a for n in walk(rot) if isinstance(n, F.Op) and n.name == "where" for a in n.args[:1]]
    half = {F.Digit("x", 128, None): 128, d_of: 1}
    if ops - {"where", "neg"} or len(negs) != 1 or not all(l.arg == x.arg and l.index.terms == half for l in rloads) \
            or {l.index.const for l in rloads} != {64, -64} or not (isinstance(negs[0].args[0], F.Load) and negs[0].args[0].index.const == 64) \
            or not all(isinstance(c, F.Cond) and c.op == "lt" and c.value == 64 and c.index.terms == {d_of: 1} for c in conds):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the rotated half is not cat(-x[64:], x[:64])")
    if st.index.const != 0 or st.index.terms != flat or st.mask is not None:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: rotary store index {st.index} is not x")
    heads, tokens = hd // 128, numel // hd
    d = D.new(D.QKNORM_ROPE, _manifest_args(spec), spec.grid, units=tokens * heads, unit_size=1)
    q = d.p.qk
    q.tokens, q.heads, q.dim = tokens, heads, 128
    q.out_tok_stride, q.out_head_stride = hd, 128
    q.in_arg, q.weight_arg, q.cos_arg, q.sin_arg, q.out_arg = x.arg, -1, cos.arg, sin.arg, st.arg
    q.no_norm = 1
    return Lowered(d, D.describe(d))


def _gemv_parts(st, reduces):
    """(vector, matrix) of a matrix-vector program: one sum over r of vector * matrix, the matrix a load over x
    and r, every load of the vector over r alone (or a fixed element), stored at x; else None."""
    if len(reduces) != 1 or reduces[0].op != "add" or st.index.const != 0 or st.index.terms != {F.Digit("x"): 1}:
        return None
    prod = reduces[0].value
    if not (isinstance(prod, F.Op) and prod.name == "mul" and len(prod.args) == 2):
        return None
    for mat, vec in ((prod.args[1], prod.args[0]), (prod.args[0], prod.args[1])):
        if not (isinstance(mat, F.Load) and mat.index.vars() == {"x", "r"} and mat.mask is None and mat.data is None):
            continue
        vloads = [n for n in walk(vec) if isinstance(n, F.Load)]
        if vloads and all(l.index.vars() <= {"r"} for l in vloads) and not any(
                isinstance(n, (F.Reduce, F.Dot)) for n in walk(vec)):
            return vec, mat
    return None


def _lower_gemv(spec, prog, st, red):
    """Inductor's M = 1 matmul (validation/pytorchsim/gemm_1x*/00_*_triton.py): out[x] = sum over r of
    fp32(a[r]) * fp32(B[x + N * r]), one reduction over r, cast on the store.  The reference refuses M = 1
    on its MXU (targets/tpu/lower_matmul.py:464-489) and runs it on the vector unit; lowered here to a
    GEMM descriptor with M = 1, which the executor runs on its matrix-vector path.

    Fused forms (validation/pytorchsim/qwen3_8b_layer_decode_*/01_*, 06_*, 07_*): the vector may be any fp32
    expression of loads over r (an RMSNorm x * rsqrt(ss / n + eps) * w, silu(gate) * up), kept unrounded as
    the program keeps it -- a prologue program; the store may add loads over x to the sum (residual rows) --
    an epilogue program with the sum in r7."""
    n, k, _ = _row_sizes(spec, prog, "matrix-vector product")
    vec, mat = _gemv_parts(st, [red])
    rk, xn = mat.index.coeff_of("r"), mat.index.coeff_of("x")
    if mat.index.const != 0 or set(rk) != {F.Digit("r")} or set(xn) != {F.Digit("x")}:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: matrix index {mat.index} is not x * s + r * t")
    sk, sn = rk[F.Digit("r")], xn[F.Digit("x")]
    if sn == 1:
        b_kmajor, ldb = 0, sk
    elif sk == 1:
        b_kmajor, ldb = 1, sn
    else:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: matrix with strides ({sk}, {sn})")
    if spec.args[mat.arg].dtype != "bfloat16":
        raise Refused(Reason.DTYPE_NOT_RUN, f"{spec.name}: matrix operand is {spec.args[mat.arg].dtype}")
    plain = isinstance(vec, F.Load) and vec.index.const == 0 and vec.index.terms == {F.Digit("r"): 1} \
        and vec.mask is None and spec.args[vec.arg].dtype == "bfloat16"
    d = D.new(D.GEMM, _manifest_args(spec), spec.grid, units=1, unit_size=1)
    g = d.p.gemm
    g.M, g.N, g.K = 1, n, k
    g.lda, g.ldb, g.ldc, g.ldr = k, ldb, n, n
    g.c_arg, g.r_arg = st.arg, -1
    g.b_arg = mat.arg
    g.b_kmajor = b_kmajor
    if plain:
        g.a_arg = vec.arg
    else:
        if b_kmajor:
            raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: a fused vector over an [N, K] matrix")
        g.pro = _vprog(spec, vec, "r")
        g.a_arg = g.pro.load[0].arg if g.pro.nload else mat.arg
    if st.value is not red:
        if sum(1 for x in walk(st.value) if x is red) != 1:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the stored value uses the sum twice")
        g.epi = _vprog(spec, st.value, "x", acc=red)
    return Lowered(d, D.describe(d))


def _vprog(spec, root, var, acc=None):
    """The fused vector program (ptsim_vprog) of fp32 expression `root` over the one index `var` ('r': a
    matrix-vector prologue or a reduction's operand; 'x': an epilogue, with `acc` -- the reduction -- in r7):
    loads at offset + var * stride (or a fixed element), the elementwise op set, registers r0..r6 allocated
    over the DAG (a value's register is freed after its last use)."""
    v = D.VProg()
    loads, code = [], []
    uses = {}
    for n in walk(root):
        for a in (n.args if isinstance(n, F.Op) else ()):
            if isinstance(a, F.Node):
                uses[id(a)] = uses.get(id(a), 0) + 1
    reg_of, free = {}, [6, 5, 4, 3, 2, 1, 0]

    def emit(op, dst, a=0, b=0, imm=0.0):
        if len(code) >= D.VPROG_CODE:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: a fused vector program over {D.VPROG_CODE} ops")
        ins = D.Insn()
        ins.op, ins.dst, ins.a, ins.b, ins.imm = D.OP[op], dst, a, b, imm
        code.append(ins)

    def take():
        if not free:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: a fused vector program over 7 live values")
        return free.pop()

    def release(n):
        if n is acc or not isinstance(n, F.Node):
            return
        uses[id(n)] -= 1
        if uses[id(n)] == 0 and id(n) in reg_of:
            free.append(reg_of.pop(id(n)))

    def slot(l):
        idx = l.index
        if l.mask is not None or l.data is not None or idx.vars() - {var}:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a fused load at {idx} (over {var} only)")
        stride = 0
        if idx.terms:
            if len(idx.terms) != 1 or F.Digit(var) not in idx.terms:
                raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: fused load index {idx} is not {var} * s + c")
            stride = idx.terms[F.Digit(var)]
        if spec.args[l.arg].dtype not in ("float32", "bfloat16", "float16"):
            raise Refused(Reason.DTYPE_NOT_RUN, f"{spec.name}: a fused load of {spec.args[l.arg].dtype}")
        key_ = (l.arg, idx.const, stride)
        if key_ not in loads:
            if len(loads) >= D.VPROG_LOADS:
                raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: more than {D.VPROG_LOADS} fused loads")
            loads.append(key_)
        return loads.index(key_)

    def gen(n):
        if n is acc:
            return 7
        if id(n) in reg_of:
            return reg_of[id(n)]
        if isinstance(n, F.Load):
            s_ = slot(n)
            r = take()
            emit("load", r, s_)
        elif isinstance(n, F.Const):
            r = take()
            emit("const", r, imm=n.v)
        elif isinstance(n, F.Op):
            if n.name == "sigmoid":
                one = F.Const(1.0)
                return gen(_retarget(n, F.Op("div", one, F.Op("add", one, F.Op("exp", F.Op("neg", n.args[0])))), uses))
            if n.name not in D.OP or n.name in ("load", "const", "store"):
                raise Refused(Reason.MATH_UNLOWERED, f"{spec.name}: fused vector op {n.name}")
            srcs = [gen(a) for a in n.args]
            for a in n.args:
                release(a)
            r = take()
            emit(n.name, r, srcs[0], srcs[1] if len(srcs) > 1 else srcs[0])
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a {type(n).__name__} in a fused vector program")
        reg_of[id(n)] = r
        uses.setdefault(id(n), 0)
        return r

    uses[id(root)] = uses.get(id(root), 0) + 1
    out = gen(root)
    if not code or code[-1].dst != out:
        emit("add", take() if out == 7 else out, out, gen(F.Const(0.0)) if out != 7 else out)
    v.ncode, v.nload = len(code), len(loads)
    for i, (arg, off, stride) in enumerate(loads):
        v.load[i].arg, v.load[i].offset, v.load[i].stride = arg, off, stride
    for i, c in enumerate(code):
        v.code[i] = c
    return v


def _lower_reduce_all(spec, prog, st, reduces):
    xnumel = _lookup(spec, prog, "xnumel", default=1)
    cols = _lookup(spec, prog, "r0_numel", "rnumel")
    if int(xnumel) != 1 or cols is None or len(reduces) != 1:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a whole-tensor reduction wants xnumel 1")
    red = reduces[0]
    v = red.value
    if red.op not in ("add", "max"):
        raise Refused(Reason.MATH_UNLOWERED, f"{spec.name}: reduction {red.op}")
    if st.value is not red:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a whole-tensor reduction with work after it")
    d = D.new(D.REDUCE_ALL, _manifest_args(spec), spec.grid, units=1, unit_size=1,
              workspace_bytes=D.REDUCE_WORKSPACE_BYTES)
    r = d.p.red
    if isinstance(v, F.Load) and v.index.vars() == {"r"} and v.index.const == 0 and v.index.terms == {F.Digit("r"): 1} \
            and v.mask is None:
        in_arg = v.arg
    else:
        # a fused operand (the decode layer's sums of squares: x * x, (x + residual)^2), validation/pytorchsim/
        # qwen3_8b_layer_decode_*/00_*, 05_*
        r.pro = _vprog(spec, v, "r")
        if not r.pro.nload:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a reduction of constants")
        in_arg = r.pro.load[0].arg
    r.numel, r.in_arg, r.out_arg = int(cols), in_arg, st.arg
    r.op = D.RED_MAX if red.op == "max" else D.RED_SUM
    return Lowered(d, D.describe(d))


# ---------------------------------------------------------------------------------------------------
# Matrix-unit programs
# ---------------------------------------------------------------------------------------------------

def _int_assigns(tree):
    out = {}
    for n in ast.walk(tree):
        if isinstance(n, (ast.Assign, ast.AnnAssign)):
            tgt = n.targets[0] if isinstance(n, ast.Assign) else n.target
            val = n.value
            if isinstance(tgt, ast.Name) and isinstance(val, ast.Constant) and isinstance(val.value, int) \
                    and not isinstance(val.value, bool):
                out[tgt.id] = val.value
    return out


def _pointer_params(spec):
    return [n for n, s in spec.signature.items() if isinstance(s, str) and s.startswith("*")]


def _lower_gemm(spec, tree, src):
    c = _int_assigns(tree)
    for n in ("M", "N", "K"):
        if n not in c:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a tl.dot program without constant {n}")
    M, N, K = c["M"], c["N"], c["K"]
    ptrs = _pointer_params(spec)
    alias = {}
    for n in ast.walk(tree):
        if isinstance(n, ast.Assign) and isinstance(n.targets[0], ast.Name) and isinstance(n.value, ast.Name) \
                and n.value.id in ptrs:
            alias[n.targets[0].id] = n.value.id

    def resolve(name):
        return alias.get(name, name)

    loaded, stored = [], []
    for n in ast.walk(tree):
        if isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute) and n.func.attr in ("load", "store") and n.args:
            base = n.args[0]
            while isinstance(base, ast.BinOp):
                base = base.left
            if isinstance(base, ast.Name) and resolve(base.id) in ptrs:
                (loaded if n.func.attr == "load" else stored).append(resolve(base.id))
    a_name = resolve("A") if "A" in alias else ("arg_A" if "arg_A" in ptrs else None)
    b_name = resolve("B") if "B" in alias else ("arg_B" if "arg_B" in ptrs else None)
    if a_name is None or b_name is None or len(set(stored)) != 1:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: cannot name the matmul operands")
    c_name = stored[0]
    resid = [p for p in set(loaded) if p not in (a_name, b_name)]
    if len(resid) > 1:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: an epilogue reading {resid}")
    idx = {n: i for i, n in enumerate(ptrs)}
    a, b, cc = idx[a_name], idx[b_name], idx[c_name]
    for t, nm in ((a, "A"), (b, "B")):
        if spec.args[t].dtype != "bfloat16":
            raise Refused(Reason.DTYPE_NOT_RUN, f"{spec.name}: matmul operand {nm} is {spec.args[t].dtype}; the "
                                                f"executor's tensor-core path takes bf16")
    if M == 1:
        raise Refused(Reason.MATRIX_UNIT_ONE_ROW, f"{spec.name}: M=1 (the reference refuses it on the MXU too)")
    sam, sak = c.get("stride_am", K), c.get("stride_ak", 1)
    sbk, sbn = c.get("stride_bk", N), c.get("stride_bn", 1)
    if sak != 1:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: A with K stride {sak}")
    if sbn == 1:
        b_kmajor, ldb = 0, sbk
    elif sbk == 1:
        b_kmajor, ldb = 1, sbn
    else:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: B with strides ({sbk}, {sbn})")
    # The output index is the last `n + ldc * m` the template forms (the earlier ones index the operands).
    found = re.findall(r"(?:idx_n|out_n)\s*\+\s*(\d+)\s*\*\s*(?:idx_m|out_m)", src)
    ldc = int(found[-1]) if found else N
    if ldc < N:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: output row stride {ldc} below N = {N}")
    d = D.new(D.GEMM, _manifest_args(spec), spec.grid, units=M, unit_size=1)
    g = d.p.gemm
    g.M, g.N, g.K = M, N, K
    g.lda, g.ldb, g.ldc, g.ldr = sam, ldb, ldc, ldc
    g.a_arg, g.b_arg, g.c_arg = a, b, cc
    g.r_arg = idx[resid[0]] if resid else -1
    g.b_kmajor = b_kmajor
    return Lowered(d, D.describe(d))


def _lower_attention(spec, tree):
    ce = spec.constexprs
    HQ, G, S, Dh = int(ce["HQ"]), int(ce["G"]), int(ce["S"]), int(ce["D"])
    ptrs = _pointer_params(spec)
    idx = {n: i for i, n in enumerate(ptrs)}
    need = ("q_ptr", "k_ptr", "v_ptr", "o_ptr")
    if not all(n in idx for n in need):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: attention wants q_ptr, k_ptr, v_ptr, o_ptr")
    q = spec.args[idx["q_ptr"]]
    batch = q.numel // (HQ * S * Dh)
    if batch * HQ * S * Dh != q.numel or HQ % G:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: q of {q.numel} elements is not B x {HQ} x {S} x {Dh}")
    gx = _grid_programs(spec)[0]
    if gx != batch * HQ:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: grid {gx} is not batch x heads = {batch * HQ}")
    d = D.new(D.ATTN_PREFILL, _manifest_args(spec), spec.grid, units=gx, unit_size=1)
    a = d.p.attn
    a.batch, a.hq, a.hkv, a.seq, a.dim = batch, HQ, HQ // G, S, Dh
    a.q_arg, a.k_arg, a.v_arg, a.o_arg = idx["q_ptr"], idx["k_ptr"], idx["v_ptr"], idx["o_ptr"]
    a.causal = 1 if ce.get("CAUSAL", True) else 0
    a.scale = float(ce["SCALE"])
    a.ref_bq, a.ref_bkv = int(ce.get("BQ", 0)), int(ce.get("BKV", 0))
    return Lowered(d, D.describe(d))


def _lower_decode(spec, tree):
    """The attention_decode_* program (validation/pytorchsim/attention_decode_32x8x4096_bf16/00__decode_kernel/
    _decode_kernel_triton.py:4-31): program p = one KV head, q/o rows [p*G*D, (p+1)*G*D) (G real rows of GP),
    k/v [p*S*D, (p+1)*S*D); online softmax over key blocks of BKV (unmasked loads: S is a multiple of BKV)."""
    ce = spec.constexprs
    HKV, G, GP, S, Dh, BKV = (int(ce[k]) for k in ("HKV", "G", "GP", "S", "D", "BKV"))
    ptrs = _pointer_params(spec)
    idx = {n: i for i, n in enumerate(ptrs)}
    need = ("q_ptr", "k_ptr", "v_ptr", "o_ptr")
    if not all(n in idx for n in need):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: decode attention wants q_ptr, k_ptr, v_ptr, o_ptr")
    if G < 1 or G > GP or BKV < 1 or S % BKV:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: G={G} GP={GP} S={S} BKV={BKV}")
    gx = _grid_programs(spec)[0]
    if gx != HKV:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: grid {gx} is not one program per KV head ({HKV})")
    q, k = spec.args[idx["q_ptr"]], spec.args[idx["k_ptr"]]
    if q.numel < HKV * G * Dh or k.numel < HKV * S * Dh or spec.args[idx["v_ptr"]].numel < HKV * S * Dh:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: tensors smaller than {HKV} heads x (G={G} | S={S}) x {Dh}")
    for n in need:
        if spec.args[idx[n]].dtype != "bfloat16":
            raise Refused(Reason.DTYPE_NOT_RUN, f"{spec.name}: {n} is {spec.args[idx[n]].dtype}")
    d = D.new(D.ATTN_DECODE, _manifest_args(spec), spec.grid, units=HKV, unit_size=1)
    a = d.p.attn
    a.batch, a.hq, a.hkv, a.seq, a.dim = 1, HKV * G, HKV, S, Dh
    a.q_arg, a.k_arg, a.v_arg, a.o_arg = idx["q_ptr"], idx["k_ptr"], idx["v_ptr"], idx["o_ptr"]
    a.causal = 0
    a.scale = float(ce["SCALE"])
    a.ref_bq, a.ref_bkv = GP, BKV
    return Lowered(d, D.describe(d))


def _selection_args(spec, what):
    ptrs = _pointer_params(spec)
    idx = {n: i for i, n in enumerate(ptrs)}
    if not all(n in idx for n in ("x_ptr", "v_ptr", "i_ptr")):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {what} wants x_ptr, v_ptr, i_ptr")
    return idx["x_ptr"], idx["v_ptr"], idx["i_ptr"]


def _lower_topk(spec):
    """The MoE router's _topk_kernel (validation/pytorchsim/layer_op_router_post_128x0_bf16/01__topk_kernel/
    _topk_kernel_triton.py:3-26): rows of E values (row stride E), K passes of (best value, first column
    holding it) over EP candidate columns, the chosen column overwritten with the spent value; v [rows, K],
    i [rows, K] int64."""
    ce = spec.constexprs
    E, EP, K = int(ce["E"]), int(ce["EP"]), int(ce["K"])
    x, v, i = _selection_args(spec, "top-k")
    rows = _lookup(spec, None, "rows")
    if rows is None:
        rows = spec.args[x].numel // max(1, E)
    rows = int(rows)
    if EP < E or K > EP or spec.args[x].numel < rows * E or spec.args[v].numel < rows * K or spec.args[i].numel < rows * K:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: rows={rows} E={E} EP={EP} K={K}")
    d = D.new(D.TOPK, _manifest_args(spec), spec.grid, units=rows, unit_size=1)
    e = d.p.sel
    e.rows, e.cols, e.k, e.cols_padded = rows, E, K, EP
    e.in_arg, e.val_arg, e.idx_arg = x, v, i
    e.descending = 1 if ce["LARGEST"] else 0
    return Lowered(d, D.describe(d))


def _lower_sort(spec):
    """The MoE dispatch's _sort_kernel (validation/pytorchsim/layer_op_dispatch_128x0_bf16/00__sort_kernel/
    _sort_kernel_triton.py:3-53): program `row` sorts its E keys at row * E (a bitonic network over L x D
    positions, ties broken by position), writes the sorted values (keys mapped back) and int64 positions."""
    ce = spec.constexprs
    x, v, i = _selection_args(spec, "sort")
    rows = _grid_programs(spec)[0]
    E = _lookup(spec, None, "E")
    if E is None:
        E = spec.args[x].numel // max(1, rows)
    E = int(E)
    if E > int(ce["L"]) * int(ce["D"]) or spec.args[x].numel < rows * E or spec.args[v].numel < rows * E \
            or spec.args[i].numel < rows * E:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: {rows} rows of E={E} over L*D={ce['L'] * ce['D']}")
    d = D.new(D.SORT, _manifest_args(spec), spec.grid, units=rows, unit_size=1)
    e = d.p.sel
    e.rows, e.cols, e.k, e.cols_padded = rows, E, 0, int(ce["L"]) * int(ce["D"])
    e.in_arg, e.val_arg, e.idx_arg = x, v, i
    e.descending = 1 if ce["DESCENDING"] else 0
    e.float_keys = 1 if ce["FLOAT"] else 0
    return Lowered(d, D.describe(d))


def _lower_divsum(spec, prog, st, red):
    """x / sum(x) per row (the MoE router's weight normalisation, validation/pytorchsim/
    layer_op_router_post_128x0_bf16/02_*_triton.py: tmp4 = sum over r of x; x / tmp4, cast on the store)."""
    rows, cols, xblock = _row_sizes(spec, prog, "row normalisation")
    v = st.value
    while isinstance(v, F.Op) and v.name in ("to_fp32", "to_bf16", "cast"):
        v = v.args[0]
    if not (isinstance(v, F.Op) and v.name == "div" and isinstance(v.args[0], F.Load) and isinstance(v.args[1], F.Reduce)
            and key(strip_casts(v.args[1].value)) == key(v.args[0])):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: not x / sum(x)")
    ld = v.args[0]
    d = D.new(D.ROW_DIVSUM, _manifest_args(spec), spec.grid, units=_grid_programs(spec)[0], unit_size=xblock)
    r = d.p.row
    r.rows, r.cols = rows, cols
    r.in_row_stride = _row_index(ld.index, "normalisation load", rows)
    r.out_row_stride = _row_index(st.index, "normalisation store", rows)
    r.in_arg, r.out_arg, r.weight_arg = ld.arg, st.arg, -1
    return Lowered(d, D.describe(d))


def _lower_rowsum(spec, prog, st, red):
    """sum over r of x per row (the MoE layer's top-k weight sums, validation/pytorchsim/layer_layer_prefill_*/
    22_*_triton.py: an fp32 sum of the 8 weights of each token)."""
    rows, cols, xblock = _row_sizes(spec, prog, "row sum")
    ld = red.value
    if not isinstance(ld, F.Load) or ld.data is not None or ld.mask is not None:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a row sum of something other than a load")
    d = D.new(D.ROW_SUM, _manifest_args(spec), spec.grid, units=_grid_programs(spec)[0], unit_size=xblock)
    r = d.p.row
    r.rows, r.cols = rows, cols
    r.in_row_stride = _row_index(ld.index, "row-sum load", rows)
    r.out_row_stride = 1
    if st.index.const != 0 or st.index.terms != {F.Digit("x"): 1}:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: row-sum store index {st.index} is not x")
    r.in_arg, r.out_arg, r.weight_arg = ld.arg, st.arg, -1
    return Lowered(d, D.describe(d))


_NO_MOD = 1 << 62
_CMP = {"cmp_lt": "lt", "cmp_le": "le", "cmp_gt": "gt", "cmp_ge": "ge", "cmp_eq": "eq", "cmp_ne": "ne"}
_IBIN = {"add": "add", "sub": "sub", "mul": "mul", "idiv": "div", "imod": "mod", "iand": "and", "ior": "or",
         "ixor": "xor", "ishr": "shr", "ishl": "shl"}


def _int_program(spec, tree, idx_load):
    """The int64 program (descriptor instructions) of an index expression over one loaded index value:
    Triton's integer semantics (// and % truncate toward zero, comparisons are 0 / 1), shared subtrees
    computed once.  Result in the last instruction's register."""
    code, memo = [], {}

    def emit(op, a=0, b=0, c=0, imm=0):
        if len(code) >= D.MAX_ICODE:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: an index program over {D.MAX_ICODE} instructions")
        ins = D.IInsn()
        ins.op, ins.dst, ins.a, ins.b, ins.c, ins.imm = D.IOP[op], len(code), a, b, c, int(imm)
        code.append(ins)
        return ins.dst

    def gen(n):
        if isinstance(n, F.Cond):
            if n.op != "data" or not isinstance(n.value, F.Node):
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: an index condition on the program index")
            n = n.value
        k = key(n)
        if k in memo:
            return memo[k]
        if isinstance(n, F.Const):
            if n.v != int(n.v):
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a fractional constant {n.v} in an index")
            r = emit("const", imm=int(n.v))
        elif isinstance(n, F.Load):
            if n.data is not None or n.arg != idx_load.arg or key(n) != key(idx_load):
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: an index program reading two indices")
            r = emit("load")
        elif isinstance(n, F.Op):
            if n.name in _IBIN:
                a, b = gen(n.args[0]), gen(n.args[1])
                r = emit(_IBIN[n.name], a, b)
            elif n.name in _CMP:
                a, b = gen(n.args[0]), gen(n.args[1])
                r = emit(_CMP[n.name], a, b)
            elif n.name == "invert":
                r = emit("inv", gen(n.args[0]))
            elif n.name == "neg":
                z = gen(F.Const(0))
                r = emit("sub", z, gen(n.args[0]))
            elif n.name == "where":
                cnd = gen(n.args[0])
                a, b = gen(n.args[1]), gen(n.args[2])
                r = emit("where", a, b, cnd)
            elif n.name in ("rbf16", "rf16"):
                r = gen(n.args[0])
            else:
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {n.name} in an index program")
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {type(n).__name__} in an index program")
        memo[k] = r
        return r

    res = gen(tree)
    if code[-1].dst != res:
        emit("add", res, gen(F.Const(0)))
    return code


def _lower_gather(spec, prog, st):
    """A row gather (index_select), e.g. the MoE dispatch's token copy (validation/pytorchsim/
    layer_op_dispatch_128x0_bf16/01_*_triton.py: out[x] = table[x % 2048 + 2048 * t], t computed from
    idx[x // 2048] -- Python floor division by top-k, negative results wrapped by the token count): the
    store is flat over x, the gathered load's affine part is x % C, its data part C * t(idx[...])."""
    ld = strip_casts(st.value)
    if st.mask is not None or ld.mask is not None:
        raise Refused(Reason.MASKED_STORE_NOT_A_BOX, f"{spec.name}: a masked gather")
    if st.index.const != 0 or st.index.terms != {F.Digit("x"): 1}:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: gather store index {st.index} is not x")
    aff = ld.index
    if aff.const != 0 or len(aff.terms) != 1:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: gathered load index {aff} is not x % C + data")
    (dg, coef), = aff.terms.items()
    if dg.var != "x" or dg.div != 1 or dg.mod is None or coef != 1:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: gathered load index {aff} is not x % C + data")
    C = int(dg.mod)
    data = ld.data
    t = None
    if isinstance(data, F.Op) and data.name == "mul":
        for a, b in ((data.args[0], data.args[1]), (data.args[1], data.args[0])):
            if isinstance(a, F.Const) and int(a.v) == C:
                t = b
    if t is None:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: the gathered offset is not {C} * row")
    leaves = [n for n in walk(t) if isinstance(n, F.Load)]
    if not leaves:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a gather whose row reads no index")
    il = leaves[0]
    m = D.Map()
    m.arg = il.arg
    m.offset = il.index.const
    digits = []
    for d, c in sorted(il.index.terms.items(), key=lambda kv: (kv[0].var, kv[0].div)):
        if d.var != "x" or d.div % C != 0:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: index load {il.index} is not a function of x // {C}")
        digits.append((d.div // C, _NO_MOD if d.mod is None else int(d.mod), int(c)))
    if len(digits) > D.MAX_DIGITS:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: index load {il.index} has too many digits")
    m.ndigit = len(digits)
    for i, (dv, md, sd) in enumerate(digits):
        m.div[i], m.mod[i], m.stride[i] = dv, md, sd
    code = _int_program(spec, t, il)
    out, table = spec.args[st.arg], spec.args[ld.arg]
    numel = _lookup(spec, prog, "xnumel") or out.numel
    d = D.new(D.GATHER_ROWS, _manifest_args(spec), spec.grid, units=int(numel) // C, unit_size=1)
    g = d.p.gat
    g.rows, g.cols, g.table_rows = int(numel) // C, C, table.numel // C
    g.out_arg, g.table_arg, g.idx_arg, g.ncode = st.arg, ld.arg, il.arg, len(code)
    g.idx_map = m
    for i, ins in enumerate(code):
        g.code[i] = ins
    return Lowered(d, D.describe(d))


def _lower_grouped_gemm(spec):
    """The MoE expert matmul (validation/pytorchsim/layer_op_gmm_gate_up_128x0_bf16/05__grouped_mm_kernel/
    _grouped_mm_kernel_triton.py:4-44): program p takes group g = group_ptr[p], rows [start_ptr[g],
    + rows_ptr[g]) of a (row stride K) times b[g] (at g * sbg, strides sbk, sbn), stored to c (row stride N)."""
    ce = spec.constexprs
    ptrs = _pointer_params(spec)
    idx = {n: i for i, n in enumerate(ptrs)}
    need = ("a_ptr", "b_ptr", "group_ptr", "start_ptr", "rows_ptr", "c_ptr")
    if not all(n in idx for n in need):
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: grouped matmul wants {', '.join(need)}")
    K, N, sbg, sbk, sbn = (int(ce[k]) for k in ("K", "N", "sbg", "sbk", "sbn"))
    if sbn != 1 or sbg != K * sbk:
        raise Refused(Reason.SHAPE_NOT_RUN, f"{spec.name}: B strides ({sbg}, {sbk}, {sbn}) are not contiguous [K, N] groups")
    a, b = spec.args[idx["a_ptr"]], spec.args[idx["b_ptr"]]
    M = a.numel // K
    groups = b.numel // sbg
    programs = _grid_programs(spec)[0]
    for n in need:
        want = "bfloat16" if n in ("a_ptr", "b_ptr", "c_ptr") else "int32"
        if spec.args[idx[n]].dtype != want:
            raise Refused(Reason.DTYPE_NOT_RUN, f"{spec.name}: {n} is {spec.args[idx[n]].dtype}")
    d = D.new(D.GROUPED_GEMM, _manifest_args(spec), spec.grid, units=1, unit_size=1)
    q = d.p.ggemm
    q.M, q.N, q.K, q.groups, q.programs, q.ldb, q.ldg = M, N, K, groups, programs, sbk, sbg
    q.a_arg, q.b_arg, q.c_arg = idx["a_ptr"], idx["b_ptr"], idx["c_ptr"]
    q.group_arg, q.start_arg, q.rows_arg = idx["group_ptr"], idx["start_ptr"], idx["rows_ptr"]
    return Lowered(d, D.describe(d))


def _term_map(spec, idx, C, terms, arg):
    """The descriptor map over the term index f = row * terms + k of an index affine in x // C (rows of C
    output columns) and r (the term k)."""
    m = D.Map()
    m.arg, m.offset = arg, idx.const
    digits = []
    for d, c in sorted(idx.terms.items(), key=lambda kv: (kv[0].var, kv[0].div)):
        if d.var == "x" and d.div % C == 0:
            digits.append(((d.div // C) * terms, _NO_MOD if d.mod is None else int(d.mod), int(c)))
        elif d.var == "r" and terms % d.div == 0:
            span = terms // d.div
            digits.append((d.div, span if d.mod is None else min(span, int(d.mod)), int(c)))
        else:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: index {idx} is not a function of (x // {C}, r)")
    if len(digits) > D.MAX_DIGITS:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: index {idx} has too many digits")
    m.ndigit = len(digits)
    for i, (dv, md, sd) in enumerate(digits):
        m.div[i], m.mod[i], m.stride[i] = dv, md, sd
    return m


def _term_program(spec, tree, C, terms):
    """(instructions, maps) of an int64 index program over the term (row, k): direct loads through up to
    PTSIM_GSUM_MAPS maps over f = row * terms + k, loads through a loaded position as LOADI."""
    code, memo, maps = [], {}, []

    def emit(op, a=0, b=0, c=0, imm=0):
        if len(code) >= D.MAX_ICODE:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: an index program over {D.MAX_ICODE} instructions")
        ins = D.IInsn()
        ins.op, ins.dst, ins.a, ins.b, ins.c, ins.imm = D.IOP[op], len(code), a, b, c, int(imm)
        code.append(ins)
        return ins.dst

    def gen(n):
        if isinstance(n, F.Cond):
            if n.op != "data" or not isinstance(n.value, F.Node):
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: an index condition on the program index")
            n = n.value
        k = key(n)
        if k in memo:
            return memo[k]
        if isinstance(n, F.Const):
            if n.v != int(n.v):
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a fractional constant {n.v} in an index")
            r = emit("const", imm=int(n.v))
        elif isinstance(n, F.Load) and n.data is None:
            mk = (n.arg, key(n))
            slot = next((i for i, (kk, _) in enumerate(maps) if kk == mk), None)
            if slot is None:
                if len(maps) >= D.GSUM_MAPS:
                    raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: more than {D.GSUM_MAPS} index reads")
                maps.append((mk, _term_map(spec, n.index, C, terms, n.arg)))
                slot = len(maps) - 1
            r = emit("load", slot)
        elif isinstance(n, F.Load):
            if n.index.terms:
                raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: an index read at {n.index} + data")
            pos = gen(n.data)
            if n.index.const:
                pos = emit("add", pos, gen(F.Const(n.index.const)))
            r = emit("loadi", pos, 0, n.arg)
        elif isinstance(n, F.Op):
            if n.name in _IBIN:
                a, b = gen(n.args[0]), gen(n.args[1])
                r = emit(_IBIN[n.name], a, b)
            elif n.name in _CMP:
                a, b = gen(n.args[0]), gen(n.args[1])
                r = emit(_CMP[n.name], a, b)
            elif n.name == "invert":
                r = emit("inv", gen(n.args[0]))
            elif n.name == "neg":
                r = emit("sub", gen(F.Const(0)), gen(n.args[0]))
            elif n.name == "where":
                cnd = gen(n.args[0])
                a, b = gen(n.args[1]), gen(n.args[2])
                r = emit("where", a, b, cnd)
            elif n.name in ("rbf16", "rf16"):
                r = gen(n.args[0])
            else:
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {n.name} in an index program")
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {type(n).__name__} in an index program")
        memo[k] = r
        return r

    res = gen(tree)
    if code[-1].dst != res:
        emit("add", res, gen(F.Const(0)))
    return code, [m for _, m in maps]


def _lower_gather_sum(spec, prog, st, red):
    """A weighted sum of gathered rows, e.g. the MoE combine (validation/pytorchsim/layer_op_combine_128x0_bf16/
    03_*_triton.py: out[x] = sum over r of float(in4[x % 2048 + 2048 * p]) * float(in5[r + 8 * (x // 2048)]), p
    the expert-ordered row of token x // 2048's r-th choice, read through in0 (expert id), in1 / in2 (that
    expert's running offsets) and in3 (the slot))."""
    if st.mask is not None:
        raise Refused(Reason.MASKED_STORE_NOT_A_BOX, f"{spec.name}: a masked weighted gather")
    if st.index.const != 0 or st.index.terms != {F.Digit("x"): 1}:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: weighted gather store index {st.index} is not x")

    def at_out(n):
        return isinstance(n, F.Load) and n.data is None and n.mask is None and n.index.const == 0 \
            and n.index.terms == {F.Digit("x"): 1}

    # The MoE layer's fused combine (layer_layer_*/23_*, 27_*) adds the residual stream: (a + b) + sum.
    residuals = []
    if st.value is not red:
        v = st.value
        if not (isinstance(v, F.Op) and v.name == "add" and v.args[1] is red):
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a weighted gather with work after the sum")
        rs = v.args[0]
        if at_out(rs):
            residuals = [rs.arg]
        elif isinstance(rs, F.Op) and rs.name == "add" and all(at_out(a) for a in rs.args):
            residuals = [rs.args[0].arg, rs.args[1].arg]
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: the added rows are not loads at the output index")
    prod = strip_casts(red.value)
    a0, a1 = (strip_casts(a) for a in prod.args)
    tab, w = (a0, a1) if isinstance(a0, F.Load) and a0.data is not None else (a1, a0)
    divisor = None
    if isinstance(w, F.Op) and w.name == "div" and all(isinstance(a, F.Load) for a in w.args):
        w, divisor = w.args   # weights renormalised by their sum (layer_layer_*/23_*, 27_*)
    if not (isinstance(w, F.Load) and w.data is None) or tab.mask is not None or w.mask is not None:
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: not a gathered row times a weight")
    aff = tab.index
    if aff.const != 0 or len(aff.terms) != 1:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: gathered load index {aff} is not x % C + data")
    (dg, coef), = aff.terms.items()
    if dg.var != "x" or dg.div != 1 or coef != 1:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: gathered load index {aff} is not x % C + data")
    # x % C over rows of C columns; a one-row program indexes by x alone (C = xnumel)
    C = int(dg.mod) if dg.mod is not None else int(_lookup(spec, prog, "xnumel") or spec.args[st.arg].numel)
    t = None
    if isinstance(tab.data, F.Op) and tab.data.name == "mul":
        for p, q in ((tab.data.args[0], tab.data.args[1]), (tab.data.args[1], tab.data.args[0])):
            if isinstance(p, F.Const) and int(p.v) == C:
                t = q
    if t is None:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: the gathered offset is not {C} * row")
    terms = _lookup(spec, prog, "r0_numel", "rnumel")
    rblock = prog.block.get("r") or _lookup(spec, prog, "R0_BLOCK")
    if terms is None or (rblock is not None and int(rblock) != int(terms)):
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: a weighted gather over a looped reduction")
    terms = int(terms)
    code, maps = _term_program(spec, t, C, terms)
    out, table = spec.args[st.arg], spec.args[tab.arg]
    numel = _lookup(spec, prog, "xnumel") or out.numel
    d = D.new(D.GATHER_SUM, _manifest_args(spec), spec.grid, units=int(numel) // C, unit_size=1)
    g = d.p.gsum
    g.rows, g.cols, g.terms, g.table_rows = int(numel) // C, C, terms, table.numel // C
    g.out_arg, g.table_arg, g.w_arg, g.ncode = st.arg, tab.arg, w.arg, len(code)
    g.w_map = _term_map(spec, w.index, C, terms, w.arg)
    for i, m in enumerate(maps):
        g.maps[i] = m
    if divisor is not None:
        # divided per output row: a fixed element, or one per row (x // C)
        di = divisor.index
        if divisor.data is not None or divisor.mask is not None or \
                (di.terms and (len(di.terms) != 1 or next(iter(di.terms)) != F.Digit("x", C, None))):
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: weight divisor index {di} is not a per-row element")
        g.wdiv, g.wdiv_arg, g.wdiv_offset = 1, divisor.arg, di.const
        g.wdiv_stride = next(iter(di.terms.values())) if di.terms else 0
    g.nres = len(residuals)
    for i, a in enumerate(residuals):
        g.res_arg[i] = a
    for i, ins in enumerate(code):
        g.code[i] = ins
    return Lowered(d, D.describe(d))


# ---------------------------------------------------------------------------------------------------
# Integer table programs
# ---------------------------------------------------------------------------------------------------

_INT_TYPES = ("int64", "int32", "int16", "int8", "uint8", "bool")


def _itab_program(spec, cols, exprs):
    """(instructions, maps, result register per expression) of int64 programs over the element f = x * cols + r:
    loads and index values through up to PTSIM_ITAB_MAPS maps (deduplicated by index, the argument in the
    instruction), masked loads as LOADM, loads through a loaded position as LOADI, index comparisons as
    IDX + compare, shared subtrees computed once."""
    code, memo, maps = [], {}, []

    def emit(op, a=0, b=0, c=0, imm=0):
        if len(code) >= D.MAX_ICODE:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: an integer program over {D.MAX_ICODE} instructions")
        ins = D.IInsn()
        ins.op, ins.dst, ins.a, ins.b, ins.c, ins.imm = D.IOP[op], len(code), a, b, c, int(imm)
        code.append(ins)
        return ins.dst

    def slot(idx):
        k = (tuple(sorted(idx.terms.items())), idx.const)
        for i, (kk, _) in enumerate(maps):
            if kk == k:
                return i
        if len(maps) >= D.ITAB_MAPS:
            raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: more than {D.ITAB_MAPS} distinct indices")
        maps.append((k, _term_map(spec, idx, 1, cols, -1)))
        return len(maps) - 1

    def int_arg(a):
        if spec.args[a].dtype not in _INT_TYPES:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a {spec.args[a].dtype} load in an integer program")
        return a

    def gen_cond(c):
        if c.op == "data" and isinstance(c.value, F.Node):
            return gen(c.value)
        if c.op == "bounds":
            return gen(F.Const(1))
        if c.op in ("lt", "le", "gt", "ge", "eq", "ne") and isinstance(c.index, F.Index) and isinstance(c.value, int):
            return gen(F.Op("cmp_" + c.op, F.IndexValue(c.index), F.Const(c.value)))
        if c.op == "and" and c.parts:
            r = gen_cond(c.parts[0])
            for p in c.parts[1:]:
                r = emit("and", r, gen_cond(p))
            return r
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a condition {c.op} in an integer program")

    def gen(n):
        if isinstance(n, F.Cond):
            return gen_cond(n)
        k = (key(n), _cond_key(n.mask)) if isinstance(n, F.Load) else key(n)
        if k in memo:
            return memo[k]
        if isinstance(n, F.Const):
            if n.v != int(n.v):
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a fractional constant {n.v} in an integer program")
            r = emit("const", imm=int(n.v))
        elif isinstance(n, F.IndexValue):
            r = emit("idx", slot(n.index))
        elif isinstance(n, F.Load) and n.data is None:
            if n.mask is None:
                r = emit("load", slot(n.index), 0, int_arg(n.arg))
            else:
                other = n.other.v if isinstance(n.other, F.Const) else (n.other or 0)
                if not isinstance(other, (int, float)) or other != int(other):
                    raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a masked load whose fill is not an integer")
                cnd = gen_cond(n.mask)
                r = emit("loadm", slot(n.index), cnd, int_arg(n.arg), imm=int(other))
        elif isinstance(n, F.Load):
            if n.mask is not None:
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a masked load through a loaded position")
            pos = gen(n.data)
            if n.index.terms:
                pos = emit("add", pos, emit("idx", slot(n.index)))
            elif n.index.const:
                pos = emit("add", pos, gen(F.Const(n.index.const)))
            r = emit("loadi", pos, 0, int_arg(n.arg))
        elif isinstance(n, F.Op):
            if n.name in _IBIN or n.name in _CMP:
                a, b = gen(n.args[0]), gen(n.args[1])
                r = emit(_IBIN.get(n.name) or _CMP[n.name], a, b)
            elif n.name == "invert":
                r = emit("inv", gen(n.args[0]))
            elif n.name == "neg":
                r = emit("sub", gen(F.Const(0)), gen(n.args[0]))
            elif n.name == "where":
                cnd = gen(n.args[0])
                a, b = gen(n.args[1]), gen(n.args[2])
                r = emit("where", a, b, cnd)
            else:
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {n.name} in an integer program")
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: {type(n).__name__} in an integer program")
        memo[k] = r
        return r

    regs = [gen(e) for e in exprs]
    return code, regs, slot, maps


def _lower_int_table(spec, prog):
    """The MoE routing tables (validation/pytorchsim/layer_op_gmm_*/01_* to 03_*, layer_op_combine_*/00_* to
    02_*): integer programs over a [rows = xnumel, cols = r0_numel] space whose stores are per element,
    a row total (tl.sum over r), or an inclusive running total over r (tl.associative_scan with a + b; in
    a looped reduction, the block scan plus a carry that adds each block's last element, Inductor's
    split-scan form).  Each store becomes an output of one PTSIM_KIND_INT_TABLE descriptor."""
    cols = _lookup(spec, prog, "r0_numel", "rnumel")
    if cols is None:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: an integer table without a reduction extent")
    rows, cols = int(_lookup(spec, prog, "xnumel") or 1), int(cols)
    rblock = prog.block.get("r") or _lookup(spec, prog, "R0_BLOCK", "RBLOCK")
    rblock = int(rblock) if rblock is not None else cols

    def along_r(sc):
        if not (sc.axis == 1 or (sc.axis in (0, -1) and rows == 1)):
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a scan along axis {sc.axis}")

    outs = []
    for st in prog.stores:
        if st.mask is not None:
            raise Refused(Reason.MASKED_STORE_NOT_A_BOX, f"{spec.name}: a masked store in an integer program")
        v = st.value
        if isinstance(v, F.Reduce):
            if v.op != "add":
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: an integer {v.op} reduction")
            if "r" in st.index.vars():
                raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: a row total stored at every r")
            mode, e = "sum", v.value
        elif isinstance(v, F.Scan):
            along_r(v)
            if prog.loops or rblock != cols:
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a scan restarted in every block")
            mode, e = "scan", v.value
        elif isinstance(v, F.Op) and v.name == "add" and len(v.args) == 2 and isinstance(v.args[0], F.Carry) \
                and isinstance(v.args[1], F.Scan):
            c, sc = v.args
            along_r(sc)
            upd = prog.carries.get(c)
            lp = c.loop
            if not (c.init == 0 and isinstance(upd, F.Op) and upd.name == "add" and upd.args[0] is c
                    and isinstance(upd.args[1], F.ChunkLast) and upd.args[1].value is sc
                    and lp.start == 0 and lp.step == rblock and lp.stop == cols and cols % rblock == 0):
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a block scan whose carry is not the "
                                                            f"running total of the blocks before")
            mode, e = "scan", sc.value
        else:
            mode, e = "elem", v
            if "r" not in st.index.vars() and cols != 1:
                raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: an element store without the r index")
        if any(isinstance(n, (F.Scan, F.Reduce, F.Carry, F.ChunkLast)) for n in walk(e)):
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{spec.name}: a nested scan or reduction")
        outs.append((st, mode, e))
    if len(outs) > D.ITAB_OUTS:
        raise Refused(Reason.DESCRIPTOR_CANNOT_STATE, f"{spec.name}: {len(outs)} stores (at most {D.ITAB_OUTS})")
    code, regs, slot, maps = _itab_program(spec, cols, [e for _, _, e in outs])
    out_maps = [slot(st.index) for st, _, _ in outs]   # store indices share the table with the loads
    d = D.new(D.INT_TABLE, _manifest_args(spec), spec.grid, units=rows, unit_size=1)
    q = d.p.itab
    q.rows, q.cols, q.ncode, q.nout = rows, cols, len(code), len(outs)
    for i, (_, m) in enumerate(maps):
        q.maps[i] = m
    for i, ((st, mode, _), reg, m) in enumerate(zip(outs, regs, out_maps)):
        o = q.out[i]
        o.arg, o.map, o.reg, o.mode = st.arg, m, reg, D.ITAB_MODE[mode]
    for i, ins in enumerate(code):
        q.code[i] = ins
    return Lowered(d, D.describe(d))
