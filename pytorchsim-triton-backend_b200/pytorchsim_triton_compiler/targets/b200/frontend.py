"""The B200 lowering's front end: a symbolic evaluation of a Triton kernel's Python source into a small
tile-program IR (index maps + a value DAG), standing where the reference runs patched Triton 3.8 and its
TTGIR -> linalg -> pytorchsim passes (pytorchsim_triton_compiler/frontend.py:24-27, passes/lower.py:35-55).

Why the source and not TTIR: the validation bundle's kernels use blocks of up to 2**24 elements, past
stock Triton's tensor limit (the reference's Triton is patched for its NPU), so they cannot be traced to
TTIR here.  Their bodies are straight-line Inductor/Triton code over tl.* calls, which this module walks
statement by statement.

The IR:
  index expressions (Index): const + sum coeff * digit(var, div, mod), digit = (var // div) % mod, over
    the launch's global row index 'x' (pid * XBLOCK + arange), the reduction index 'r', and program ids;
  values (Node): Load(arg, index, mask, other), Const, Op(name, *args), Reduce(op, value), Dot(a, b);
    integer programs add IndexValue(index) (an index used as data), Scan(op, value, axis) (an inclusive
    scan along the block), ChunkLast(value) (a scan's last element in the block) and Carry (an integer
    loop-carried value as the loop body sees it);
  Store(arg, index, value, mask) records.
Anything outside that (an index the algebra cannot state, a call it does not know) raises Refused, the
reference's refusal discipline (contract/stop.py); nothing is guessed."""
import ast
import inspect
import math
import textwrap

from ...contract.stop import Reason, Refused

# ---------------------------------------------------------------------------------------------------
# Index algebra
# ---------------------------------------------------------------------------------------------------


class Digit(tuple):
    """(var, div, mod): the value (var // div) % mod; mod None means unbounded."""
    __slots__ = ()

    def __new__(cls, var, div=1, mod=None):
        return tuple.__new__(cls, (var, int(div), None if mod is None else int(mod)))

    var = property(lambda s: s[0])
    div = property(lambda s: s[1])
    mod = property(lambda s: s[2])


class Index:
    """An integer tensor expression: const + sum(coeff * digit)."""

    def __init__(self, terms=None, const=0):
        self.terms = {k: v for k, v in (terms or {}).items() if v != 0}
        self.const = int(const)

    @staticmethod
    def var(name):
        return Index({Digit(name): 1})

    def __add__(self, o):
        o = as_index(o)
        t = dict(self.terms)
        for k, v in o.terms.items():
            t[k] = t.get(k, 0) + v
        return Index(t, self.const + o.const)

    __radd__ = __add__

    def __neg__(self):
        return Index({k: -v for k, v in self.terms.items()}, -self.const)

    def __sub__(self, o):
        return self + (-as_index(o))

    def __rsub__(self, o):
        return as_index(o) + (-self)

    def scale(self, c):
        return Index({k: v * c for k, v in self.terms.items()}, self.const * c)

    def single(self):
        """The lone digit of an expression that is exactly one digit with coefficient 1, else None."""
        if self.const == 0 and len(self.terms) == 1:
            (d, c), = self.terms.items()
            if c == 1:
                return d
        return None

    def floordiv(self, k):
        k = int(k)
        if not self.terms:
            return Index(const=self.const // k)
        d = self.single()
        if d is None:
            raise Refused(Reason.INDEX_NOT_AFFINE, f"floor division of {self} by {k} is not a digit")
        if d.mod is None:
            return Index({Digit(d.var, d.div * k, None): 1})
        if d.mod % k:
            raise Refused(Reason.INDEX_NOT_AFFINE, f"({d.var} // {d.div}) % {d.mod} // {k}: {k} does not divide {d.mod}")
        return Index({Digit(d.var, d.div * k, d.mod // k): 1})

    def mod(self, m):
        m = int(m)
        if not self.terms:
            return Index(const=self.const % m)
        d = self.single()
        if d is None:
            raise Refused(Reason.INDEX_NOT_AFFINE, f"{self} % {m} is not a digit")
        if d.mod is not None and d.mod % m:
            raise Refused(Reason.INDEX_NOT_AFFINE, f"digit mod {d.mod} taken mod {m}")
        return Index({Digit(d.var, d.div, m): 1})

    def vars(self):
        return {d.var for d in self.terms}

    def coeff_of(self, var):
        return {d: c for d, c in self.terms.items() if d.var == var}

    def __repr__(self):
        parts = [f"{c}*({d.var}//{d.div}%{d.mod})" for d, c in self.terms.items()]
        return " + ".join(parts + [str(self.const)])


def as_index(v):
    if isinstance(v, Index):
        return v
    if isinstance(v, (bool, int)):
        return Index(const=int(v))
    if isinstance(v, Arange):
        raise Refused(Reason.INDEX_NOT_AFFINE, "an arange used outside a block index")
    raise Refused(Reason.INDEX_NOT_AFFINE, f"{type(v).__name__} used as an index")


class Arange:
    """tl.arange(0, n), not yet placed as a row (x) or reduction (r) block index."""

    def __init__(self, n, dim=None):
        self.n, self.dim = int(n), dim


class Pid:
    """tl.program_id(axis) times a factor."""

    def __init__(self, axis, factor=1):
        self.axis, self.factor = axis, int(factor)


class LoopVar:
    """The induction variable of a loop over [start, stop) by step."""

    def __init__(self, name, start, stop, step):
        self.name, self.start, self.stop, self.step = name, start, stop, step


# ---------------------------------------------------------------------------------------------------
# Values
# ---------------------------------------------------------------------------------------------------


class Node:
    kind = "node"


class Const(Node):
    kind = "const"

    def __init__(self, v):
        self.v = float(v)


class Load(Node):
    kind = "load"

    def __init__(self, arg, index, mask=None, other=None, data=None):
        # data: a value node added to the affine index (an index loaded from memory, as index_select has)
        self.arg, self.index, self.mask, self.other, self.data = arg, index, mask, other, data


class Op(Node):
    kind = "op"

    def __init__(self, name, *args):
        self.name, self.args = name, args


class Reduce(Node):
    kind = "reduce"

    def __init__(self, op, value):
        self.op, self.value = op, value


class Dot(Node):
    kind = "dot"

    def __init__(self, a, b):
        self.a, self.b = a, b


class IndexValue(Node):
    """An index expression used as an integer value (tmp = (x0).to(tl.int64); tmp == loaded)."""
    kind = "index"

    def __init__(self, index):
        self.index = index


class Scan(Node):
    """tl.associative_scan(value, axis, combine) with an additive combine: the inclusive running sum along the
    block's `axis` (within one block of a looped reduction)."""
    kind = "scan"

    def __init__(self, op, value, axis):
        self.op, self.value, self.axis = op, value, axis


class ChunkLast(Node):
    """The last element of `value` along the reduction block (triton_helpers.select_one(v, rbase == RBLOCK - 1)):
    for a Scan, the block's total."""
    kind = "chunk_last"

    def __init__(self, value):
        self.value = value


class Carry(Node):
    """An integer value carried across the iterations of `loop` (a name holding an integer tl.full before the
    loop and reassigned in its body), as one iteration sees it on entry.  `init` is its value before the
    loop; the body's update is recorded in Program.carries."""
    kind = "carry"

    def __init__(self, name, init, loop):
        self.name, self.init, self.loop = name, init, loop


class IntFull(int):
    """The value of an integer tl.full / tl.zeros: a loop-carried integer accumulator starts from one."""


class Cond:
    """A mask: a comparison of an index with a constant, or a conjunction of masks."""

    def __init__(self, op, index=None, value=None, parts=()):
        self.op, self.index, self.value, self.parts = op, index, value, tuple(parts)


class Ptr:
    """A pointer argument plus an element index (affine) and an optional data-dependent offset (a value node)."""

    def __init__(self, arg, index=None, data=None):
        self.arg, self.index, self.data = arg, index if index is not None else Index(), data


class DataIndex:
    """An affine index plus a value node: the element offset of a gather (x0 + C * loaded_index)."""

    def __init__(self, index, data):
        self.index, self.data = index, data


class Store:
    def __init__(self, arg, index, value, mask):
        self.arg, self.index, self.value, self.mask = arg, index, value, mask


class DType:
    def __init__(self, name):
        self.name = name


_DTYPES = {"float32": "float32", "float16": "float16", "bfloat16": "bfloat16", "int32": "int32", "int64": "int64",
           "int1": "bool", "int8": "int8", "int16": "int16", "uint8": "uint8", "float64": "float64"}

# ---------------------------------------------------------------------------------------------------
# The evaluator
# ---------------------------------------------------------------------------------------------------


class Program:
    """The front end's result: the stores, every Dot met, loops seen, constants assigned by name."""

    def __init__(self):
        self.stores, self.dots, self.loops = [], [], []
        self.assigned = {}   # name -> last constant value assigned in the body (M = 4096, eps, ...)
        self.calls = set()   # every tl./libdevice. call name met
        self.block = {}      # axis -> block size of a pid * BLOCK + arange(BLOCK) index
        self.carries = {}    # Carry -> its value at the end of the loop body (integer loop-carried values)


def kernel_source(fn):
    """(source text, function name) of a @triton.jit kernel or a plain function."""
    inner = fn
    for _ in range(4):
        if hasattr(inner, "src") and isinstance(getattr(inner, "src"), str):
            return textwrap.dedent(inner.src), getattr(inner, "__name__", None) or inner.fn.__name__
        if hasattr(inner, "fn"):
            inner = inner.fn
            continue
        break
    return textwrap.dedent(inspect.getsource(inner)), inner.__name__


def kernel_globals(fn):
    """The module globals of a @triton.jit kernel (where its @triton.jit helpers live), or {}."""
    inner = fn
    for _ in range(4):
        g = getattr(inner, "__globals__", None)
        if isinstance(g, dict):
            return g
        inner = getattr(inner, "fn", None)
        if inner is None:
            break
    return {}


def combine_op(helper):
    """'add' when the @triton.jit function `helper` returns the sum of its two arguments (Inductor's
    _triton_helper_fn_add0), else None."""
    try:
        src, name = kernel_source(helper)
    except (TypeError, OSError):
        return None
    fn = next((n for n in ast.walk(ast.parse(src)) if isinstance(n, ast.FunctionDef)), None)
    if fn is None or len(fn.args.args) != 2:
        return None
    a, b = (x.arg for x in fn.args.args)
    env = {}
    for st in fn.body:
        if isinstance(st, ast.Assign) and len(st.targets) == 1 and isinstance(st.targets[0], ast.Name):
            env[st.targets[0].id] = st.value
        elif isinstance(st, ast.Return) and st.value is not None:
            e = st.value
            while isinstance(e, ast.Name) and e.id in env:
                e = env[e.id]
            if isinstance(e, ast.BinOp) and isinstance(e.op, ast.Add) and isinstance(e.left, ast.Name) \
                    and isinstance(e.right, ast.Name) and {e.left.id, e.right.id} == {a, b}:
                return "add"
            return None
        elif not isinstance(st, (ast.Expr, ast.Pass)):
            return None
    return None


class Evaluator:
    def __init__(self, spec, prog, globals_=None):
        self.spec, self.prog = spec, prog
        self.env = {}
        self.acc_init = {}
        self.globals = globals_ or {}

    # ---- entry ---------------------------------------------------------------------------------
    def run(self, src, name):
        tree = ast.parse(src)
        fn = next((n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef) and n.name == name), None)
        if fn is None:
            fn = next(n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef))
        tensor_i = 0
        scalars = self.spec.extra.get("scalar_values", {})
        for a in fn.args.args:
            nm = a.arg
            sig = self.spec.signature.get(nm)
            if sig is None:
                if nm in self.spec.constexprs:
                    self.env[nm] = self.spec.constexprs[nm]
                continue
            if sig == "constexpr" or nm in self.spec.constexprs:
                self.env[nm] = self.spec.constexprs.get(nm)
            elif sig.startswith("*"):
                self.env[nm] = Ptr(tensor_i)
                tensor_i += 1
            else:
                self.env[nm] = scalars.get(nm)
        self.block(fn.body)
        return self.prog

    def block(self, stmts):
        for s in stmts:
            if self.stmt(s) == "return":
                return "return"

    # ---- statements ------------------------------------------------------------------------------
    def stmt(self, s):
        if isinstance(s, ast.Assign):
            v = self.expr(s.value)
            for t in s.targets:
                self.assign(t, v)
        elif isinstance(s, ast.AnnAssign):
            if s.value is not None:
                self.assign(s.target, self.expr(s.value))
        elif isinstance(s, ast.AugAssign):
            cur = self.expr(s.target)
            self.assign(s.target, self.binop(s.op, cur, self.expr(s.value)))
        elif isinstance(s, ast.Expr):
            self.expr(s.value)
        elif isinstance(s, ast.For):
            self.loop(s)
        elif isinstance(s, ast.If):
            c = self.expr(s.test)
            if isinstance(c, (bool, int)) and not isinstance(c, Node):
                return self.block(s.body if c else s.orelse)
            # A data- or loop-dependent branch: both arms describe the same tile program shape.
            self.block(s.body)
            self.block(s.orelse)
        elif isinstance(s, ast.Return):
            return "return"
        elif isinstance(s, ast.Pass):
            pass
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"statement {type(s).__name__} at line {s.lineno}")

    def assign(self, target, v):
        if isinstance(target, ast.Tuple) and isinstance(v, (list, tuple)) and len(v) == len(target.elts):
            for t, x in zip(target.elts, v):
                self.assign(t, x)
            return
        if isinstance(target, ast.Name):
            if isinstance(v, Arange) and v.dim is None:
                # A 1-D block index: the program names which axis it walks (x*: rows, r*: reduction).
                v = Arange(v.n, "r" if target.id.startswith("r") else "x")
            self.env[target.id] = v
            if isinstance(v, (int, float)) and not isinstance(v, bool):
                self.prog.assigned[target.id] = v
        else:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"assignment to {type(target).__name__}")

    def loop(self, s):
        if not isinstance(s.target, ast.Name):
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, "a loop over a tuple")
        it = s.iter
        if not (isinstance(it, ast.Call)):
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, "a loop over a non-range")
        args = [self.expr(a) for a in it.args]
        if len(args) == 1:
            start, stop, step = 0, args[0], 1
        elif len(args) == 2:
            start, stop, step = args[0], args[1], 1
        else:
            start, stop, step = args[0], args[1], args[2]
        lv = LoopVar(s.target.id, start, stop, step)
        self.prog.loops.append(lv)
        before = dict(self.env)
        self.env[s.target.id] = lv
        # Integer loop-carried names: an integer tl.full before the loop, reassigned in the body.
        assigned = {t.id for st in s.body for n in ast.walk(st) if isinstance(n, ast.Assign)
                    for t in n.targets if isinstance(t, ast.Name)}
        carries = {}
        for name in sorted(assigned):
            if isinstance(self.env.get(name), IntFull):
                carries[name] = self.env[name] = Carry(name, int(self.env[name]), lv)
        self.block(s.body)
        for name, c in carries.items():
            v = self.env.get(name)
            if v is c:
                self.env[name] = before[name]
                continue
            self.prog.carries[c] = v
            if isinstance(v, Op) and v.name in ("add", "max", "min") and len(v.args) == 2 and v.args[0] is c:
                self.env[name] = Op("acc_" + v.name, v.args[1])
        # Accumulators: a name holding a constant before the loop and op(previous, x) after one pass.
        for name, v in list(self.env.items()):
            old = before.get(name)
            if isinstance(old, Const) and isinstance(v, Op) and v.name in ("add", "max", "min") and len(v.args) == 2 \
                    and v.args[0] is old:
                self.env[name] = Op("acc_" + v.name, v.args[1])

    # ---- expressions -----------------------------------------------------------------------------
    def expr(self, e):
        if isinstance(e, ast.Constant):
            return e.value
        if isinstance(e, ast.Name):
            if e.id in self.env:
                return self.env[e.id]
            if e.id in ("True", "False", "None"):
                return {"True": True, "False": False, "None": None}[e.id]
            return _Module(e.id)
        if isinstance(e, ast.Attribute):
            base = self.expr(e.value)
            if isinstance(base, _Module):
                return _Module(base.name + "." + e.attr)
            if e.attr == "dtype" and isinstance(base, Ptr):
                return _PtrDtype(base.arg)
            if isinstance(base, _PtrDtype) and e.attr == "element_ty":
                return DType(self.spec.args[base.arg].dtype)
            return _Bound(base, e.attr)
        if isinstance(e, ast.BinOp):
            return self.binop(e.op, self.expr(e.left), self.expr(e.right))
        if isinstance(e, ast.UnaryOp):
            v = self.expr(e.operand)
            if isinstance(e.op, ast.USub):
                if isinstance(v, (int, float)):
                    return -v
                if isinstance(v, Index):
                    return -v
                return Op("neg", self.value(v))
            if isinstance(e.op, ast.Not):
                return not v
            if isinstance(e.op, ast.Invert):
                if isinstance(v, int) and not isinstance(v, bool):
                    return ~v
                if isinstance(v, Node):
                    return Op("invert", v)
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"unary {type(e.op).__name__}")
        if isinstance(e, ast.Compare):
            if len(e.ops) != 1:
                raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, "a chained comparison")
            a, b = self.expr(e.left), self.expr(e.comparators[0])
            return self.compare(e.ops[0], a, b)
        if isinstance(e, ast.BoolOp):
            vals = [self.expr(v) for v in e.values]
            if all(isinstance(v, (bool, int)) for v in vals):
                return all(vals) if isinstance(e.op, ast.And) else any(vals)
            return Cond("and", parts=[v for v in vals if isinstance(v, Cond)])
        if isinstance(e, ast.Subscript):
            # [:, None] / [None, :] / [:] place a block index on the row or reduction axis.
            v = self.expr(e.value)
            if isinstance(v, Arange):
                sl = e.slice
                elts = sl.elts if isinstance(sl, ast.Tuple) else [sl]
                if len(elts) == 2:
                    first_is_none = isinstance(elts[0], ast.Constant) and elts[0].value is None
                    return Arange(v.n, "r" if first_is_none else "x")
                return Arange(v.n, v.dim)
            return v
        if isinstance(e, ast.Call):
            return self.call(e)
        if isinstance(e, ast.Tuple) or isinstance(e, ast.List):
            return [self.expr(x) for x in e.elts]
        if isinstance(e, ast.IfExp):
            c = self.expr(e.test)
            if isinstance(c, (bool, int)):
                return self.expr(e.body if c else e.orelse)
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, "a data-dependent conditional expression")
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"expression {type(e).__name__}")

    def compare(self, op, a, b):
        a = a.v if isinstance(a, Const) else a
        b = b.v if isinstance(b, Const) else b
        if isinstance(a, (int, float)) and isinstance(b, (int, float)):
            return {ast.Lt: a < b, ast.LtE: a <= b, ast.Gt: a > b, ast.GtE: a >= b, ast.Eq: a == b,
                    ast.NotEq: a != b}[type(op)]
        name = {ast.Lt: "lt", ast.LtE: "le", ast.Gt: "gt", ast.GtE: "ge", ast.Eq: "eq", ast.NotEq: "ne"}[type(op)]
        if isinstance(a, (Index, Arange, Pid, LoopVar)) and isinstance(b, (int, float)):
            idx = self.index_of(a)
            if name == "lt" and self.is_extent(idx, b):
                return Cond("bounds", idx, b)
            return Cond(name, idx, b)
        if isinstance(a, (Index, Arange, Pid, LoopVar)) and isinstance(b, (Index, Arange, Pid, LoopVar)):
            return Cond(name, self.index_of(a) - self.index_of(b), 0)
        idx_like = (Index, Arange, Pid, LoopVar)
        if (isinstance(a, idx_like) and isinstance(b, Node)) or (isinstance(a, Node) and isinstance(b, idx_like)):
            # loaded data against an index (an expert id against the row's expert number)
            return Cond("data", None, Op("cmp_" + name, self.value(a), self.value(b)))
        if isinstance(a, (Node, int, float)) and isinstance(b, (Node, int, float)):
            # a comparison of data values: kept as a value node (0/1) for where() and integer programs
            return Cond("data", None, Op("cmp_" + name, self.value(a), self.value(b)))
        return Cond("data", None, None)

    def is_extent(self, idx, n):
        """Whether `idx < n` only guards the launch's own extent: idx is the global row (x) or reduction (r)
        index and n its numel (a scalar or constexpr named as the pointwise lowering reads the extent), so the
        mask holds for every element the launch stores (the store is clamped to n)."""
        d = idx.single()
        if d is None or d.div != 1 or d.mod is not None:
            return False
        names = {"x": ("xnumel", "n", "N", "numel", "n_elements"), "r": ("r0_numel", "rnumel")}.get(d.var, ())
        return any(isinstance(self.env.get(nm), int) and self.env.get(nm) == n for nm in names)

    def index_of(self, v):
        if isinstance(v, Index):
            return v
        if isinstance(v, (bool, int)):
            return Index(const=int(v))
        if isinstance(v, Arange):
            return Index.var(v.dim or "x") if v.dim else Index.var("x")
        if isinstance(v, Pid):
            return Index.var(f"pid{v.axis}").scale(v.factor)
        if isinstance(v, LoopVar):
            return Index.var("loop:" + v.name)
        raise Refused(Reason.INDEX_NOT_AFFINE, f"{type(v).__name__} as an index")

    def value(self, v):
        """`v` as a value node."""
        if isinstance(v, Node):
            return v
        if isinstance(v, Cond) and v.op == "data" and isinstance(v.value, Node):
            return v.value   # a comparison of data values as 0 / 1
        if isinstance(v, (Index, Arange, Pid, LoopVar)):
            return IndexValue(self.index_of(v))
        if isinstance(v, DataIndex):
            return Op("add", IndexValue(v.index), v.data)
        if isinstance(v, Cond) and v.op in ("lt", "le", "gt", "ge", "eq", "ne") and isinstance(v.index, Index):
            return Op("cmp_" + v.op, IndexValue(v.index), Const(v.value))   # an index comparison as 0 / 1
        if isinstance(v, (int, float)) and not isinstance(v, bool):
            return Const(v)
        if isinstance(v, bool):
            return Const(1.0 if v else 0.0)
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"{type(v).__name__} used as a value")

    def binop(self, op, a, b):
        num = (int, float)
        if isinstance(a, num) and isinstance(b, num) and not isinstance(a, bool) and not isinstance(b, bool):
            return _fold(op, a, b)
        # Block indices: pid * BLOCK + arange(BLOCK) is the global index of that axis.
        if isinstance(op, ast.Mult):
            if isinstance(a, Pid) and isinstance(b, int):
                return Pid(a.axis, a.factor * b)
            if isinstance(b, Pid) and isinstance(a, int):
                return Pid(b.axis, b.factor * a)
        if isinstance(op, ast.Add):
            for p, q in ((a, b), (b, a)):
                if isinstance(p, Pid) and isinstance(q, Arange) and p.factor == q.n:
                    self.prog.block[q.dim or "x"] = q.n
                    return Index.var(q.dim or "x")
                if isinstance(p, LoopVar) and isinstance(q, Arange) and p.step == q.n:
                    self.prog.block[q.dim or "r"] = q.n
                    return Index.var(q.dim or "r")
                if isinstance(p, int) and p == 0 and isinstance(q, Arange):
                    return q
        if _is_index(a) and _is_index(b) and not (isinstance(a, Node) or isinstance(b, Node)):
            ia, ib = self.index_of(a), self.index_of(b)
            if isinstance(op, ast.Add):
                return ia + ib
            if isinstance(op, ast.Sub):
                return ia - ib
            if isinstance(op, ast.Mult):
                if not ib.terms:
                    return ia.scale(ib.const)
                if not ia.terms:
                    return ib.scale(ia.const)
                raise Refused(Reason.INDEX_NOT_AFFINE, "a product of two index tensors")
            if isinstance(op, ast.FloorDiv) and not ib.terms:
                return ia.floordiv(ib.const)
            if isinstance(op, ast.Mod) and not ib.terms:
                return ia.mod(ib.const)
            raise Refused(Reason.INDEX_NOT_AFFINE, f"index operator {type(op).__name__}")
        if isinstance(a, Ptr) and _is_index(b):
            return Ptr(a.arg, a.index + self.index_of(b), a.data)
        if isinstance(b, Ptr) and _is_index(a):
            return Ptr(b.arg, b.index + self.index_of(a), b.data)
        if isinstance(op, ast.Add):
            for p, q in ((a, b), (b, a)):
                if isinstance(p, Ptr) and isinstance(q, DataIndex) and p.data is None:
                    return Ptr(p.arg, p.index + q.index, q.data)
                if isinstance(p, Ptr) and isinstance(q, Node) and not isinstance(q, Const) and p.data is None:
                    return Ptr(p.arg, p.index, q)   # a pointer offset by a loaded value (an index load)
                if isinstance(p, (Index, Arange, Pid, LoopVar)) and isinstance(q, Node) and not isinstance(q, Const):
                    return DataIndex(self.index_of(p), q)
                if isinstance(p, DataIndex) and _is_index(q):
                    return DataIndex(p.index + self.index_of(q), p.data)
        name = {ast.Add: "add", ast.Sub: "sub", ast.Mult: "mul", ast.Div: "div", ast.FloorDiv: "idiv",
                ast.Mod: "imod", ast.BitAnd: "iand", ast.BitOr: "ior", ast.BitXor: "ixor", ast.RShift: "ishr",
                ast.LShift: "ishl"}.get(type(op))
        if name is None:
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"value operator {type(op).__name__}")
        return Op(name, self.value(a), self.value(b))

    # ---- calls -----------------------------------------------------------------------------------
    def call(self, e):
        f = self.expr(e.func)
        if isinstance(f, _Module) and f.name.split(".")[-1] == "device_assert":
            # a bounds assertion of the reference; the executor's own bounds checks record PTSIM_E_OOB
            return None
        args = [self.expr(a) for a in e.args]
        kw = {k.arg: self.expr(k.value) for k in e.keywords}
        if isinstance(f, _Bound):
            return self.method(f.obj, f.attr, args, kw)
        if not isinstance(f, _Module):
            raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, "a call of a computed function")
        name = f.name.split(".")[-1]
        self.prog.calls.add(name)
        if name == "program_id":
            return Pid(int(args[0] if args else kw.get("axis", 0)))
        if name == "arange":
            return Arange(int(args[1]) - int(args[0]))
        if name in ("full", "zeros"):
            fill = args[1] if name == "full" and len(args) > 1 else kw.get("value", 0)
            dt = args[2] if len(args) > 2 else kw.get("dtype")
            is_int = isinstance(dt, _Module) and _DTYPES.get(dt.name.split(".")[-1], "") in ("int32", "int64", "bool", "int8", "int16", "uint8")
            if isinstance(fill, bool) or isinstance(fill, (Index, Pid, Arange, LoopVar)):
                return fill
            if is_int:
                return IntFull(int(fill))
            return Const(float(fill))
        if name in ("cdiv",):
            return -(-int(args[0]) // int(args[1]))
        if name in ("min", "max") and f.name in ("min", "max"):
            if all(isinstance(a, (int, float)) for a in args):
                return (min if name == "min" else max)(args)
        if name == "float" and f.name == "float":
            return float(args[0])
        if name in ("range", "static_range"):
            return args  # handled by loop()
        if name == "load":
            ptr = args[0]
            if not isinstance(ptr, Ptr):
                raise Refused(Reason.POINTER_BASE_UNTRACED, "a load through an untraced pointer")
            mask = args[1] if len(args) > 1 else kw.get("mask")
            other = args[2] if len(args) > 2 else kw.get("other")
            if isinstance(mask, Cond) and mask.op == "bounds":
                mask = None
            return Load(ptr.arg, ptr.index, mask if isinstance(mask, Cond) else None, other, ptr.data)
        if name == "store":
            ptr = args[0]
            if not isinstance(ptr, Ptr):
                raise Refused(Reason.POINTER_BASE_UNTRACED, "a store through an untraced pointer")
            val = args[1] if len(args) > 1 else kw.get("value")
            mask = args[2] if len(args) > 2 else kw.get("mask")
            if isinstance(mask, Cond) and mask.op == "bounds":
                mask = None
            self.prog.stores.append(Store(ptr.arg, ptr.index, self.value(val), mask if isinstance(mask, Cond) else None))
            return None
        if name == "dot":
            d = Dot(self.value(args[0]), self.value(args[1]))
            self.prog.dots.append(d)
            return d
        if name in ("broadcast_to", "promote_to_tensor", "max_contiguous", "multiple_of", "assume", "reshape",
                    "view", "expand_dims", "static_assert", "debug_barrier"):
            return args[0] if args else None
        if name in ("exp", "exp2", "rsqrt", "sqrt", "abs", "log", "sigmoid", "cos", "sin"):
            return Op(name, self.value(args[0]))
        if name in ("maximum", "minimum"):
            return Op("max" if name == "maximum" else "min", self.value(args[0]), self.value(args[1]))
        if name == "where":
            if self._first_iteration_guard(args[0]):
                # where(roffset > 0, carry + v, v) with the carry 0 before the loop: carry + v on every pass
                a1, a2 = self.value(args[1]), self.value(args[2])
                if isinstance(a1, Op) and a1.name == "add" and isinstance(a1.args[0], Carry) and a1.args[0].init == 0 \
                        and a1.args[1] is a2 and a1.args[0].loop.name == args[0].index.single()[0][len("loop:"):]:
                    return a1
            if isinstance(args[0], Cond) and args[0].op == "bounds":
                return self.value(args[1])
            if isinstance(args[0], bool):
                pick = args[1] if args[0] else args[2]
                return pick if isinstance(pick, (int, float)) else self.value(pick)
            return Op("where", args[0] if isinstance(args[0], Cond) else Cond("data"), self.value(args[1]), self.value(args[2]))
        if name in ("sum", "max2", "min2") or (name in ("max", "min") and "." in f.name):
            axis = args[1] if len(args) > 1 else kw.get("axis")
            op = {"sum": "add", "max2": "max", "min2": "min", "max": "max", "min": "min"}[name]
            v = self.value(args[0])
            if isinstance(v, Op) and v.name == "acc_" + op:
                v = v.args[0]
            return Reduce(op, v)
        if name == "associative_scan":
            vals = args[0] if args else kw.get("input")
            axis = args[1] if len(args) > 1 else kw.get("axis")
            fn = args[2] if len(args) > 2 else kw.get("combine_fn")
            if not isinstance(vals, list) or len(vals) != 1 or not isinstance(axis, int):
                raise Refused(Reason.MATH_UNLOWERED, f"{f.name} over {len(vals) if isinstance(vals, list) else '?'} values")
            helper = self.globals.get(fn.name) if isinstance(fn, _Module) else None
            if helper is None or combine_op(helper) != "add":
                raise Refused(Reason.MATH_UNLOWERED, f"{f.name} with a combine function other than a + b")
            return [Scan("add", self.value(vals[0]), axis)]
        if name == "select_one":
            cond = args[1] if len(args) > 1 else None
            rb = self.prog.block.get("r") or self.env.get("R0_BLOCK") or self.env.get("RBLOCK")
            if isinstance(cond, Cond) and cond.op == "eq" and isinstance(cond.index, Index) and cond.index.const == 0 \
                    and cond.index.terms == {Digit("r"): 1} and isinstance(rb, int) and cond.value == rb - 1:
                return ChunkLast(self.value(args[0]))
            raise Refused(Reason.MATH_UNLOWERED, f"{f.name} of other than the block's last element")
        if name in ("fma",):
            return Op("add", Op("mul", self.value(args[0]), self.value(args[1])), self.value(args[2]))
        if name.startswith("atomic"):
            raise Refused(Reason.ATOMICS, f"{f.name}: atomics have no tile program on this executor")
        raise Refused(Reason.MATH_UNLOWERED, f"call of {f.name}")

    def _first_iteration_guard(self, c):
        """Whether `c` is `loopvar > 0` for a loop starting at 0 (false exactly on the first pass)."""
        if not (isinstance(c, Cond) and c.op == "gt" and c.value == 0 and isinstance(c.index, Index)):
            return False
        d = c.index.single()
        if d is None or c.index.const != 0 or not str(d[0]).startswith("loop:") or d[1] != 1 or d[2] is not None:
            return False
        lv = next((l for l in self.prog.loops if l.name == d[0][len("loop:"):]), None)
        return lv is not None and lv.start == 0 and isinstance(lv.step, int) and lv.step > 0

    def method(self, obj, attr, args, kw):
        if attr == "to":
            dt = args[0] if args else kw.get("dtype")
            if isinstance(obj, (Index, Arange, Pid, LoopVar, int)):
                return obj
            v = self.value(obj)
            if isinstance(dt, DType) and dt.name == "bfloat16":
                return Op("rbf16", v)
            if isinstance(dt, _Module):
                tname = _DTYPES.get(dt.name.split(".")[-1])
                if tname == "bfloat16":
                    return Op("rbf16", v)
                if tname in ("float32", "float64", None):
                    return v
                if tname in ("float16",):
                    return Op("rf16", v)
            return v
        if attr in ("broadcast_to", "reshape", "expand_dims"):
            return obj
        raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"method .{attr}()")


class _Module:
    def __init__(self, name):
        self.name = name


class _Bound:
    def __init__(self, obj, attr):
        self.obj, self.attr = obj, attr


class _PtrDtype:
    def __init__(self, arg):
        self.arg = arg


def _is_index(v):
    return isinstance(v, (Index, Arange, Pid, LoopVar)) or (isinstance(v, int) and not isinstance(v, bool))


def _fold(op, a, b):
    if isinstance(op, ast.Add):
        return a + b
    if isinstance(op, ast.Sub):
        return a - b
    if isinstance(op, ast.Mult):
        return a * b
    if isinstance(op, ast.Div):
        return a / b
    if isinstance(op, ast.FloorDiv):
        return a // b
    if isinstance(op, ast.Mod):
        return a % b
    if isinstance(op, ast.Pow):
        return a ** b
    raise Refused(Reason.PROGRAM_CLASS_UNKNOWN, f"constant operator {type(op).__name__}")


def trace(spec, fn=None):
    """The tile program of `spec`'s kernel (its Triton source, symbolically evaluated)."""
    if fn is None:
        fn = load_kernel(spec)
    src, name = kernel_source(fn)
    return Evaluator(spec, Program(), kernel_globals(fn)).run(src, name)


def load_kernel(spec):
    """spec.kernel(), importing an Inductor-generated kernel module (written for torch 2.14's runtime
    helpers, which select a GPU driver at import) with those two helpers stubbed for the duration of the
    import: the module is only read here, never launched through Triton."""
    import contextlib
    try:
        from torch._inductor.runtime import triton_helpers
    except Exception:  # noqa: BLE001 -- a kernel file that needs no Inductor runtime still loads
        return spec.kernel()
    saved = {n: getattr(triton_helpers, n) for n in ("skip_gpu_driver_setup", "set_driver_to_gpu")
             if hasattr(triton_helpers, n)}
    triton_helpers.skip_gpu_driver_setup = contextlib.nullcontext
    triton_helpers.set_driver_to_gpu = lambda: None
    try:
        return spec.kernel()
    finally:
        for n in ("skip_gpu_driver_setup", "set_driver_to_gpu"):
            if n in saved:
                setattr(triton_helpers, n, saved[n])
            else:
                delattr(triton_helpers, n)
