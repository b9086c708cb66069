"""The kernel-file contract: a kernel file defines a module-level `SPEC = KernelSpec(...)` naming its Triton
kernel, the kernel's signature and constexprs, each tensor argument's role / dtype / shape, the launch grid,
a torch reference with its tolerances and an input generator.

The field names and their meaning are the reference's (pytorchsim_triton_compiler/contract/kernel_spec.py),
so kernel files written for it load here unchanged; the fields that steer the reference's scratchpad and
timing graph (graph_prefetch, on_chip, prefetch, expect_ir*, expect_stage) are accepted and checked for
consistency but do not change how the B200 executor runs the program.

A JSON spec (`spec_to_json` / `spec_from_json`) carries the fields a compile reads beyond the kernel's
source: it is what the Triton plugin passes as its `pytorchsim_spec` option."""
import dataclasses
import hashlib
import importlib.machinery
import json
import math
import os
import types
from typing import Callable

from .kernel_object import ITEMSIZE

IN, OUT, INOUT = "in", "out", "inout"
ROLES = (IN, OUT, INOUT)
EXPECTATIONS = ("pass", "refuse", "blocked", "open")
PINNED_STAGES = ("", "togcheck", "timing")
AXES = ("x", "y", "z")


def is_read(arg):
    return arg.role in (IN, INOUT)


def is_written(arg):
    return arg.role in (OUT, INOUT)


@dataclasses.dataclass
class Arg:
    """One tensor argument of the kernel, in signature order."""
    name: str
    role: str
    dtype: str
    shape: tuple

    @property
    def numel(self):
        return math.prod(self.shape)

    @property
    def nbytes(self):
        return self.numel * ITEMSIZE[self.dtype]


def _arg_indices(spec, value, what, inputs_only=False):
    """`value` as a tuple of distinct indices into spec.args (inputs only, if asked); ValueError otherwise."""
    got = tuple(value)
    n = len(spec.args)
    problems = [a for a in got if not isinstance(a, int) or not 0 <= a < n]
    if inputs_only:
        problems += [a for a in got if isinstance(a, int) and 0 <= a < n and spec.args[a].role != IN]
    if problems or len(set(got)) != len(got):
        kind = "inputs" if inputs_only else "arguments"
        raise ValueError(f"{spec.name}: KernelSpec.{what} lists distinct indices of {kind}, got {value!r}")
    return got


@dataclasses.dataclass
class KernelSpec:
    name: str
    kernel: Callable
    signature: dict
    constexprs: dict
    args: list
    grid: tuple
    reference: Callable
    make_inputs: Callable
    rtol: float = 1e-4
    atol: float = 1e-4
    expect: str = "pass"
    expect_why: str = ""
    expect_ir: dict = dataclasses.field(default_factory=dict)
    expect_ir_on: dict = dataclasses.field(default_factory=dict)
    expect_stage: str = ""
    expect_stop: object = None
    parallel_axes: tuple = ()
    extra: dict = dataclasses.field(default_factory=dict)
    grid_rule: bool = True
    ttir: str = ""
    graph_prefetch: object = None
    on_chip: tuple = ()
    prefetch: tuple = ()

    def __post_init__(self):
        from .stop import Stop
        axes = tuple(self.parallel_axes) or AXES[:max(1, len(self.grid))]
        if not set(axes) <= set(AXES) or len(set(axes)) < len(axes):
            raise ValueError(f"{self.name}: parallel_axes are distinct x/y/z, outermost first, got {axes!r}")
        self.parallel_axes = axes
        if self.graph_prefetch is not None:
            self.graph_prefetch = _arg_indices(self, self.graph_prefetch, "graph_prefetch")
        self.on_chip = _arg_indices(self, self.on_chip, "on_chip")
        self.prefetch = _arg_indices(self, self.prefetch, "prefetch", inputs_only=True)
        if set(self.prefetch) & (set(self.on_chip) | set(self.graph_prefetch or ())):
            raise ValueError(f"{self.name}: an argument in prefetch is also on_chip or in graph_prefetch")
        for a in self.args:
            if a.role not in ROLES:
                raise ValueError(f"{self.name}: argument {a.name} has role {a.role!r}, not one of {ROLES}")
        if self.expect not in EXPECTATIONS:
            raise ValueError(f"{self.name}: expect is one of {EXPECTATIONS}, got {self.expect!r}")
        if self.expect_stage not in PINNED_STAGES:
            raise ValueError(f"{self.name}: expect_stage is one of {PINNED_STAGES}, got {self.expect_stage!r}")
        passing = self.expect == "pass"
        if not passing and not self.expect_why:
            raise ValueError(f"{self.name}: a kernel expected to stop states why (expect_why)")
        if passing and self.expect_stop is not None:
            raise ValueError(f"{self.name}: a passing kernel declares no expect_stop")
        if not passing and not isinstance(self.expect_stop, Stop):
            raise ValueError(f"{self.name}: a kernel expected to stop declares where, as a contract.stop.Stop")

    def expect_ir_for(self, machine_name):
        """expect_ir with the counts stated for one machine laid over it."""
        merged = {fn: dict(counts) for fn, counts in (self.expect_ir or {}).items()}
        for fn, counts in (self.expect_ir_on or {}).get(machine_name, {}).items():
            merged.setdefault(fn, {}).update(counts)
        return merged

    def inputs(self):
        return [a for a in self.args if is_read(a)]

    def outputs(self):
        return [a for a in self.args if is_written(a)]


JSON_FIELDS = ("name", "signature", "args", "grid", "grid_rule", "graph_prefetch", "on_chip", "prefetch",
               "parallel_axes", "extra")

# Triton's type names in TTIR (the element type of a !tt.ptr, or a scalar) and in a kernel signature, and
# the kernel.json dtype each signature token stands for.
_IR_TYPE_TO_TOKEN = {"f64": "fp64", "f32": "fp32", "f16": "fp16", "bf16": "bf16", "i64": "i64", "i32": "i32",
                     "i16": "i16", "i8": "i8", "i1": "i1"}
_TOKEN_TO_DTYPE = {"fp64": "float64", "fp32": "float32", "fp16": "float16", "bf16": "bfloat16", "i64": "int64",
                   "i32": "int32", "i16": "int16", "i8": "int8", "i1": "bool"}


def _split_params(text):
    """The comma-separated parameters of a parameter list, ignoring commas inside <> () {} brackets."""
    out, depth, cur = [], 0, []
    for ch in text:
        if ch in "<({":
            depth += 1
        elif ch in ">)}":
            depth -= 1
        if ch == "," and depth == 0:
            out.append("".join(cur).strip())
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        out.append("".join(cur).strip())
    return out


def signature_from_ttir(ttir):
    """(kernel name, signature) read from the `tt.func` header of a Triton IR file: pointer parameters
    become "*<token>", scalars "<token>"."""
    with open(ttir) as fh:
        header = next((line for line in fh if "tt.func" in line), None)
    if header is None:
        raise ValueError(f"{ttir}: no tt.func in the file")
    at = header.index("@") + 1
    open_paren = header.index("(", at)
    name = header[at:open_paren].strip()
    depth, close = 0, None
    for i in range(open_paren, len(header)):
        depth += {"(": 1, ")": -1}.get(header[i], 0)
        if depth == 0:
            close = i
            break
    signature = {}
    for param in _split_params(header[open_paren + 1:close]):
        pname, _, ptype = param.partition(":")
        pname, ptype = pname.strip().lstrip("%"), ptype.strip().split(" ")[0].split("{")[0].strip()
        pointer = ptype.startswith("!tt.ptr<")
        elem = ptype[len("!tt.ptr<"):].split(">")[0].split(",")[0].strip() if pointer else ptype
        token = _IR_TYPE_TO_TOKEN.get(elem)
        if token is None:
            raise ValueError(f"{ttir}: parameter {pname} of type {ptype} has no Triton signature token")
        signature[pname] = ("*" if pointer else "") + token
    return name, signature


def spec_to_json(spec):
    """The JSON_FIELDS of `spec` as JSON text."""
    def plain(field, value):
        if field == "args":
            return [{"name": a.name, "role": a.role, "dtype": a.dtype, "shape": list(a.shape)} for a in value]
        return list(value) if isinstance(value, tuple) else value
    return json.dumps({f: plain(f, getattr(spec, f)) for f in JSON_FIELDS})


def spec_from_json(text, ttir=""):
    """A KernelSpec from JSON_FIELDS text; a missing name or signature is read from the TTIR at `ttir`.
    Each tensor argument's dtype defaults to its pointer's element type."""
    fields = json.loads(text)
    extra_keys = set(fields) - set(JSON_FIELDS)
    if extra_keys:
        raise ValueError(f"a JSON spec holds only {', '.join(JSON_FIELDS)}; it also has {', '.join(sorted(extra_keys))}")
    if not fields.get("name") or not fields.get("signature"):
        ir_name, ir_sig = signature_from_ttir(ttir)
        fields.setdefault("name", ir_name)
        fields["name"] = fields["name"] or ir_name
        fields["signature"] = fields.get("signature") or ir_sig
    pointer_params = [(p, _TOKEN_TO_DTYPE[tok[1:]]) for p, tok in fields["signature"].items() if tok.startswith("*")]
    stated = fields.pop("args")
    if len(stated) != len(pointer_params):
        raise ValueError(f"{fields['name']}: {len(stated)} tensor arguments stated, the kernel takes "
                         f"{len(pointer_params)} pointers")
    args = [Arg(s.get("name") or p, s["role"], s.get("dtype") or dt, tuple(s["shape"]))
            for s, (p, dt) in zip(stated, pointer_params)]
    fields["grid"] = tuple(fields["grid"])
    if fields.get("parallel_axes") is not None:
        fields["parallel_axes"] = tuple(fields["parallel_axes"])
    return KernelSpec(kernel=None, constexprs={}, args=args, reference=None, make_inputs=None, ttir=ttir, **fields)


def load_spec(path):
    """The SPEC of a kernel file, or of a JSON spec (`*.json`, its TTIR beside it as `*.ttir`).  A kernel
    file is executed as a module of its own, named by a hash of its path so two files never share one."""
    path = os.path.abspath(path)
    if path.endswith(".json"):
        with open(path) as fh:
            return spec_from_json(fh.read(), os.path.splitext(path)[0] + ".ttir")
    modname = "ptsim_kernel_file_" + hashlib.sha1(path.encode()).hexdigest()[:16]
    loader = importlib.machinery.SourceFileLoader(modname, path)
    module = types.ModuleType(modname)
    module.__file__ = path
    module.__loader__ = loader
    loader.exec_module(module)
    spec = getattr(module, "SPEC", None)
    if spec is None or not hasattr(spec, "args"):
        raise SystemExit(f"{path}: a kernel file defines SPEC = KernelSpec(...) at module level")
    spec.extra.setdefault("source_path", path)
    return spec
