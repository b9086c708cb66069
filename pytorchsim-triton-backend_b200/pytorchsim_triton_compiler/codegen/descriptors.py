"""Launch descriptors: the "binary" the B200 lowering emits where the reference's codegen emits a RISC-V ELF
(pytorchsim_triton_compiler/codegen/build.py:467-502 in the reference).  A descriptor is the packed
`ptsim_desc` struct of include/ptsim_b200.h; this module mirrors it with ctypes, builds one per tile-program
class, and reads one back.  The struct layout is checked against the library's own sizeof at load time
(runtime/native.py), so a mismatch between the two sides fails loudly instead of misreading fields."""
import ctypes as C

ABI_VERSION = 1
MAGIC = 0x42535450  # "PTSB"

MAX_ARGS, MAX_MAPS, MAX_DIGITS, MAX_CODE, MAX_REGS = 16, 8, 4, 32, 8

# Kinds (PTSIM_KIND_*).
ELEMENTWISE, ROW_SOFTMAX, ROW_RMSNORM, QKNORM_ROPE, GEMM, ATTN_PREFILL, REDUCE_ALL, ATTN_DECODE = 1, 2, 3, 4, 5, 6, 7, 8
ROW_DIVSUM, TOPK, SORT, GATHER_ROWS, GROUPED_GEMM, GATHER_SUM, INT_TABLE, ROW_SUM = 9, 10, 11, 12, 13, 14, 15, 16
KIND_NAME = {ELEMENTWISE: "elementwise", ROW_SOFTMAX: "row_softmax", ROW_RMSNORM: "row_rmsnorm",
             QKNORM_ROPE: "qknorm_rope", GEMM: "gemm", ATTN_PREFILL: "attn_prefill", REDUCE_ALL: "reduce_all",
             ATTN_DECODE: "attn_decode", ROW_DIVSUM: "row_divsum", TOPK: "topk", SORT: "sort",
             GATHER_ROWS: "gather_rows", GROUPED_GEMM: "grouped_gemm", GATHER_SUM: "gather_sum",
             INT_TABLE: "int_table", ROW_SUM: "row_sum"}

# Element types (PTSIM_DT_*), keyed by kernel.json dtype names (contract/kernel_object.py NP_DTYPE keys).
DTYPE_CODE = {"float32": 0, "bfloat16": 1, "float16": 2, "int32": 3, "int64": 4, "int16": 5, "int8": 6,
              "uint8": 7, "float64": 8, "bool": 6}

# Vector-unit opcodes (PTSIM_OP_*).
OP = {"load": 1, "const": 2, "add": 3, "sub": 4, "mul": 5, "div": 6, "neg": 7, "exp": 8, "rsqrt": 9,
      "sqrt": 10, "max": 11, "min": 12, "rbf16": 13, "abs": 14, "store": 15}
OP_NAME = {v: k for k, v in OP.items()}

RED_SUM, RED_MAX = 0, 1

# Status codes (PTSIM_E_*).
OK, E_DESC, E_ARGS, E_CUDA, E_UNSUPPORTED, E_OOB, E_RESOURCE, E_TIMEOUT = 0, 1, 2, 3, 4, 200, 201, 202
STATUS_NAME = {OK: "OK", E_DESC: "BAD_DESCRIPTOR", E_ARGS: "BAD_ARGUMENTS", E_CUDA: "CUDA_ERROR",
               E_UNSUPPORTED: "UNSUPPORTED", E_OOB: "INVALID_SPAD_ACCESS", E_RESOURCE: "STACK_OVERFLOW",
               E_TIMEOUT: "WAIT_TIMEOUT"}


class Map(C.Structure):
    _fields_ = [("arg", C.c_int32), ("ndigit", C.c_int32), ("offset", C.c_int64),
                ("div", C.c_int64 * MAX_DIGITS), ("mod", C.c_int64 * MAX_DIGITS), ("stride", C.c_int64 * MAX_DIGITS)]


class Insn(C.Structure):
    _fields_ = [("op", C.c_uint8), ("dst", C.c_uint8), ("a", C.c_uint8), ("b", C.c_uint8), ("imm", C.c_float)]


VPROG_LOADS, VPROG_CODE = 4, 16


class VLoad(C.Structure):
    _fields_ = [("arg", C.c_int32), ("pad0", C.c_int32), ("offset", C.c_int64), ("stride", C.c_int64)]


class VProg(C.Structure):
    """ptsim_vprog: a fused fp32 program over one index (the M = 1 matmul's prologue / epilogue, a reduction's
    operand)."""
    _fields_ = [("ncode", C.c_int32), ("nload", C.c_int32), ("load", VLoad * VPROG_LOADS), ("code", Insn * VPROG_CODE)]


class EwParams(C.Structure):
    _fields_ = [("numel", C.c_int64), ("nmap", C.c_int32), ("ncode", C.c_int32), ("store_map", C.c_int32),
                ("pure_copy", C.c_int32), ("map", Map * MAX_MAPS), ("code", Insn * MAX_CODE)]


class RowParams(C.Structure):
    _fields_ = [("rows", C.c_int64), ("cols", C.c_int64), ("in_row_stride", C.c_int64), ("out_row_stride", C.c_int64),
                ("in_arg", C.c_int32), ("out_arg", C.c_int32), ("weight_arg", C.c_int32), ("res_arg_p1", C.c_int32),
                ("eps", C.c_float), ("inv_cols", C.c_float)]


class QkParams(C.Structure):
    _fields_ = [("tokens", C.c_int64), ("heads", C.c_int64), ("dim", C.c_int64), ("out_tok_stride", C.c_int64),
                ("out_head_stride", C.c_int64), ("in_arg", C.c_int32), ("weight_arg", C.c_int32),
                ("cos_arg", C.c_int32), ("sin_arg", C.c_int32), ("out_arg", C.c_int32), ("no_norm", C.c_int32),
                ("eps", C.c_float), ("pad1", C.c_float)]


class GemmParams(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("lda", C.c_int64), ("ldb", C.c_int64),
                ("ldc", C.c_int64), ("ldr", C.c_int64), ("a_arg", C.c_int32), ("b_arg", C.c_int32),
                ("c_arg", C.c_int32), ("r_arg", C.c_int32), ("b_kmajor", C.c_int32), ("pad0", C.c_int32),
                ("pro", VProg), ("epi", VProg)]


class AttnParams(C.Structure):
    _fields_ = [("batch", C.c_int64), ("hq", C.c_int64), ("hkv", C.c_int64), ("seq", C.c_int64), ("dim", C.c_int64),
                ("q_arg", C.c_int32), ("k_arg", C.c_int32), ("v_arg", C.c_int32), ("o_arg", C.c_int32),
                ("causal", C.c_int32), ("pad0", C.c_int32), ("scale", C.c_float), ("pad1", C.c_float),
                ("ref_bq", C.c_int64), ("ref_bkv", C.c_int64)]


class ReduceParams(C.Structure):
    _fields_ = [("numel", C.c_int64), ("in_arg", C.c_int32), ("out_arg", C.c_int32), ("op", C.c_int32),
                ("pad0", C.c_int32), ("pro", VProg)]


class SelectParams(C.Structure):
    _fields_ = [("rows", C.c_int64), ("cols", C.c_int64), ("k", C.c_int64), ("cols_padded", C.c_int64),
                ("in_arg", C.c_int32), ("val_arg", C.c_int32), ("idx_arg", C.c_int32), ("descending", C.c_int32),
                ("float_keys", C.c_int32), ("pad0", C.c_int32)]


MAX_ICODE = 32
IOP = {"load": 1, "const": 2, "add": 3, "sub": 4, "mul": 5, "div": 6, "mod": 7, "inv": 8, "lt": 9, "le": 10,
       "gt": 11, "ge": 12, "eq": 13, "ne": 14, "where": 15, "and": 16, "or": 17, "xor": 18, "shr": 19, "shl": 20,
       "loadi": 21, "loadm": 22, "idx": 23}
IOP_NAME = {v: k for k, v in IOP.items()}


class IInsn(C.Structure):
    _fields_ = [("op", C.c_uint8), ("dst", C.c_uint8), ("a", C.c_uint8), ("b", C.c_uint8), ("c", C.c_uint8),
                ("pad0", C.c_uint8), ("pad1", C.c_uint8), ("pad2", C.c_uint8), ("imm", C.c_int64)]


class GatherParams(C.Structure):
    _fields_ = [("rows", C.c_int64), ("cols", C.c_int64), ("table_rows", C.c_int64), ("out_arg", C.c_int32),
                ("table_arg", C.c_int32), ("idx_arg", C.c_int32), ("ncode", C.c_int32), ("idx_map", Map),
                ("code", IInsn * MAX_ICODE)]


class GGemmParams(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("groups", C.c_int64), ("programs", C.c_int64),
                ("ldb", C.c_int64), ("ldg", C.c_int64), ("a_arg", C.c_int32), ("b_arg", C.c_int32), ("c_arg", C.c_int32),
                ("group_arg", C.c_int32), ("start_arg", C.c_int32), ("rows_arg", C.c_int32)]


GSUM_MAPS = 4


class GsumParams(C.Structure):
    _fields_ = [("rows", C.c_int64), ("cols", C.c_int64), ("terms", C.c_int64), ("table_rows", C.c_int64),
                ("out_arg", C.c_int32), ("table_arg", C.c_int32), ("w_arg", C.c_int32), ("ncode", C.c_int32),
                ("w_map", Map), ("maps", Map * GSUM_MAPS), ("code", IInsn * MAX_ICODE),
                ("wdiv", C.c_int32), ("nres", C.c_int32), ("res_arg", C.c_int32 * 2), ("wdiv_arg", C.c_int32),
                ("pad0", C.c_int32), ("wdiv_offset", C.c_int64), ("wdiv_stride", C.c_int64)]


ITAB_MAPS, ITAB_OUTS = 5, 4
FLAG_INTERPRET = 1   # desc.flags: INT_TABLE on the element interpreter only
FLAG_TEST_STALL = 2  # desc.flags: pipelined kernels withhold one stage and time out in 1 ms (timeout tests)
ITAB_MODE = {"elem": 0, "sum": 1, "scan": 2}
ITAB_MODE_NAME = {v: k for k, v in ITAB_MODE.items()}


class ItabOut(C.Structure):
    _fields_ = [("arg", C.c_int32), ("map", C.c_int32), ("reg", C.c_int32), ("mode", C.c_int32)]


class ItabParams(C.Structure):
    _fields_ = [("rows", C.c_int64), ("cols", C.c_int64), ("ncode", C.c_int32), ("nout", C.c_int32),
                ("maps", Map * ITAB_MAPS), ("out", ItabOut * ITAB_OUTS), ("code", IInsn * MAX_ICODE)]


class Params(C.Union):
    _fields_ = [("ew", EwParams), ("row", RowParams), ("qk", QkParams), ("gemm", GemmParams),
                ("attn", AttnParams), ("red", ReduceParams), ("sel", SelectParams), ("gat", GatherParams),
                ("ggemm", GGemmParams), ("gsum", GsumParams), ("itab", ItabParams)]


class Desc(C.Structure):
    _fields_ = [("magic", C.c_uint32), ("version", C.c_uint32), ("kind", C.c_uint32), ("flags", C.c_uint32),
                ("nargs", C.c_int32), ("pad0", C.c_int32), ("arg_dtype", C.c_int32 * MAX_ARGS),
                ("arg_numel", C.c_int64 * MAX_ARGS), ("grid", C.c_int64 * 3), ("units", C.c_int64),
                ("unit_size", C.c_int64), ("workspace_bytes", C.c_int64), ("p", Params)]


SIZE = C.sizeof(Desc)

# Workspace of a REDUCE_ALL launch: one fp32 partial per pass-1 CTA, at most 1024 of them.
REDUCE_WORKSPACE_BYTES = 1024 * 4


def new(kind, args, grid, units, unit_size, workspace_bytes=0):
    """A zeroed descriptor of `kind` over the manifest arguments `args` ([{name, dtype, shape}])."""
    import math
    if len(args) > MAX_ARGS:
        raise ValueError(f"{len(args)} tensor arguments; the executor takes at most {MAX_ARGS}")
    d = Desc()
    d.magic, d.version, d.kind = MAGIC, ABI_VERSION, kind
    d.nargs = len(args)
    for i, a in enumerate(args):
        if a["dtype"] not in DTYPE_CODE:
            raise ValueError(f"argument {a['name']} has dtype {a['dtype']}, which the executor does not carry")
        d.arg_dtype[i] = DTYPE_CODE[a["dtype"]]
        d.arg_numel[i] = math.prod(a["shape"])
    g = (list(grid) + [1, 1, 1])[:3]
    for i in range(3):
        d.grid[i] = int(g[i])
    d.units, d.unit_size, d.workspace_bytes = int(units), int(unit_size), int(workspace_bytes)
    return d


def to_bytes(d):
    return bytes(C.string_at(C.addressof(d), SIZE))


def from_bytes(blob):
    if len(blob) != SIZE:
        raise ValueError(f"descriptor of {len(blob)} bytes; this build writes {SIZE}")
    d = Desc.from_buffer_copy(blob)
    if d.magic != MAGIC or d.version != ABI_VERSION:
        raise ValueError(f"not a version-{ABI_VERSION} PTSB descriptor (magic 0x{d.magic:08x}, version {d.version})")
    return d


def describe_vprog(v):
    return {"loads": [(l.arg, l.offset, l.stride) for l in list(v.load)[:v.nload]],
            "code": [(OP_NAME.get(i.op, i.op), i.dst, i.a, i.b, i.imm) for i in list(v.code)[:v.ncode]]}


def describe(d):
    """A JSON-able summary of descriptor `d` (what kernel.json records next to the blob)."""
    out = {"kind": KIND_NAME.get(d.kind, d.kind), "units": d.units, "unit_size": d.unit_size,
           "grid": list(d.grid), "workspace_bytes": d.workspace_bytes}
    if d.kind == ELEMENTWISE:
        e = d.p.ew
        out["numel"] = e.numel
        out["pure_copy"] = bool(e.pure_copy)
        out["maps"] = [{"arg": m.arg, "offset": m.offset,
                        "digits": [(m.div[k], m.mod[k], m.stride[k]) for k in range(m.ndigit)]}
                       for m in list(e.map)[:e.nmap]]
        out["code"] = [(OP_NAME.get(i.op, i.op), i.dst, i.a, i.b, i.imm) for i in list(e.code)[:e.ncode]]
    elif d.kind in (ROW_SOFTMAX, ROW_RMSNORM):
        r = d.p.row
        out.update(rows=r.rows, cols=r.cols, eps=r.eps)
        if r.res_arg_p1:
            out["residual"] = r.res_arg_p1 - 1
    elif d.kind == QKNORM_ROPE:
        q = d.p.qk
        out.update(tokens=q.tokens, heads=q.heads, dim=q.dim, eps=q.eps,
                   out_strides=[q.out_tok_stride, q.out_head_stride])
        if q.no_norm:
            out["no_norm"] = True
    elif d.kind == GEMM:
        g = d.p.gemm
        out.update(M=g.M, N=g.N, K=g.K, residual=g.r_arg >= 0, b_kmajor=bool(g.b_kmajor))
        for nm in ("pro", "epi"):
            if getattr(g, nm).ncode:
                out[nm] = describe_vprog(getattr(g, nm))
    elif d.kind == ATTN_PREFILL:
        a = d.p.attn
        out.update(batch=a.batch, hq=a.hq, hkv=a.hkv, seq=a.seq, dim=a.dim, causal=bool(a.causal), scale=a.scale)
    elif d.kind == ATTN_DECODE:
        a = d.p.attn
        out.update(hkv=a.hkv, group=a.hq // max(1, a.hkv), seq=a.seq, dim=a.dim, scale=a.scale,
                   ref_bkv=a.ref_bkv)
    elif d.kind in (ROW_DIVSUM, ROW_SUM):
        out.update(rows=d.p.row.rows, cols=d.p.row.cols)
    elif d.kind in (TOPK, SORT):
        e = d.p.sel
        out.update(rows=e.rows, cols=e.cols, cols_padded=e.cols_padded, descending=bool(e.descending))
        if d.kind == TOPK:
            out["k"] = e.k
        else:
            out["float_keys"] = bool(e.float_keys)
    elif d.kind == GATHER_ROWS:
        gp = d.p.gat
        out.update(rows=gp.rows, cols=gp.cols, table_rows=gp.table_rows,
                   program=[(IOP_NAME.get(i.op, i.op), i.dst, i.a, i.b, i.c, i.imm) for i in list(gp.code)[:gp.ncode]])
    elif d.kind == GROUPED_GEMM:
        q = d.p.ggemm
        out.update(M=q.M, N=q.N, K=q.K, groups=q.groups, programs=q.programs)
    elif d.kind == GATHER_SUM:
        q = d.p.gsum
        out.update(rows=q.rows, cols=q.cols, terms=q.terms, table_rows=q.table_rows,
                   program=[(IOP_NAME.get(i.op, i.op), i.dst, i.a, i.b, i.c, i.imm) for i in list(q.code)[:q.ncode]])
        if q.wdiv:
            out["weight_divisor"] = (q.wdiv_arg, q.wdiv_offset, q.wdiv_stride)
        if q.nres:
            out["residuals"] = list(q.res_arg)[:q.nres]
    elif d.kind == INT_TABLE:
        q = d.p.itab
        out.update(rows=q.rows, cols=q.cols,
                   outputs=[(ITAB_MODE_NAME.get(o.mode, o.mode), o.arg, o.map, o.reg) for o in list(q.out)[:q.nout]],
                   program=[(IOP_NAME.get(i.op, i.op), i.dst, i.a, i.b, i.c, i.imm) for i in list(q.code)[:q.ncode]])
    elif d.kind == REDUCE_ALL:
        out.update(numel=d.p.red.numel, op="max" if d.p.red.op == RED_MAX else "sum")
        if d.p.red.pro.ncode:
            out["pro"] = describe_vprog(d.p.red.pro)
    return out
