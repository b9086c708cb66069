"""What a kernel file declares (the reference's contract/kernel_spec.py:24-214): the Triton kernel, its
signature and constexprs, each tensor argument's role/dtype/shape, the launch grid, a torch reference and
an input generator with tolerances.  Kernel files written for the reference load unchanged."""
import dataclasses
import importlib.util
import json
import math
import os
import re
from typing import Callable

from .kernel_object import ITEMSIZE

IN, OUT, INOUT = "in", "out", "inout"


def is_read(arg):
    return arg.role in (IN, INOUT)


def is_written(arg):
    return arg.role in (OUT, INOUT)


@dataclasses.dataclass
class Arg:
    """One tensor argument."""
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
        if not self.parallel_axes:
            self.parallel_axes = ("x", "y", "z")[:max(1, len(self.grid))]
        axes = tuple(self.parallel_axes)
        if any(a not in ("x", "y", "z") for a in axes) or len(set(axes)) != len(axes):
            raise ValueError(f"KernelSpec.parallel_axes is distinct 'x'/'y'/'z', outermost first; got {axes!r}")
        self.parallel_axes = axes

        def indices(value, what, inputs_only=False):
            got = tuple(value)
            ok = all(isinstance(a, int) and 0 <= a < len(self.args) for a in got) and len(set(got)) == len(got)
            if ok and inputs_only:
                ok = all(self.args[a].role == IN for a in got)
            if not ok:
                raise ValueError(f"KernelSpec.{what} holds distinct argument indices, not {value!r}: {self.name}")
            return got

        if self.graph_prefetch is not None:
            self.graph_prefetch = indices(self.graph_prefetch, "graph_prefetch")
        self.on_chip = indices(self.on_chip, "on_chip")
        self.prefetch = indices(self.prefetch, "prefetch", inputs_only=True)
        if set(self.prefetch) & (set(self.on_chip) | set(self.graph_prefetch or ())):
            raise ValueError(f"KernelSpec.prefetch overlaps on_chip or graph_prefetch: {self.name}")
        if self.expect not in ("pass", "refuse", "blocked", "open"):
            raise ValueError(f"KernelSpec.expect is pass/refuse/blocked/open, not {self.expect!r}")
        if self.expect_stage not in ("", "togcheck", "timing"):
            raise ValueError(f"KernelSpec.expect_stage is '', 'togcheck' or 'timing', not {self.expect_stage!r}")
        if self.expect != "pass" and not self.expect_why:
            raise ValueError(f"a kernel that is not expected to pass says why (expect_why): {self.name}")
        from .stop import Stop
        if (self.expect == "pass") != (self.expect_stop is None):
            raise ValueError(f"only a refuse/blocked/open kernel states expect_stop: {self.name}")
        if self.expect_stop is not None and not isinstance(self.expect_stop, Stop):
            raise ValueError(f"KernelSpec.expect_stop is a contract.stop.Stop: {self.name}")

    def expect_ir_for(self, machine_name):
        out = {f: dict(c) for f, c in (self.expect_ir or {}).items()}
        for f, counts in self.expect_ir_on.get(machine_name, {}).items():
            out.setdefault(f, {}).update(counts)
        return out

    def inputs(self):
        return [a for a in self.args if is_read(a)]

    def outputs(self):
        return [a for a in self.args if is_written(a)]


JSON_FIELDS = ("name", "signature", "args", "grid", "grid_rule", "graph_prefetch", "on_chip", "prefetch",
               "parallel_axes", "extra")

_TTIR_TOKEN = {"f64": "fp64", "f32": "fp32", "f16": "fp16", "bf16": "bf16", "i64": "i64", "i32": "i32",
               "i16": "i16", "i8": "i8", "i1": "i1"}
_TOKEN_DTYPE = {"fp64": "float64", "fp32": "float32", "fp16": "float16", "bf16": "bfloat16", "i64": "int64",
                "i32": "int32", "i16": "int16", "i8": "int8", "i1": "bool"}


def signature_from_ttir(ttir):
    """(name, signature) of the tt.func in the Triton IR file `ttir`."""
    with open(ttir) as f:
        head = next((line for line in f if "tt.func" in line), None)
    if head is None:
        raise ValueError(f"{ttir} holds no tt.func")
    name = re.search(r"@(\w+)\(", head).group(1)
    sig = {}
    for m in re.finditer(r"%(\w+): (?:!tt\.ptr<(\w+)>|(\w+))", head):
        elem, scalar = m.group(2), m.group(3)
        tok = _TTIR_TOKEN.get(elem or scalar)
        if tok is None:
            raise ValueError(f"{ttir}: parameter {m.group(1)} has type {elem or scalar}, which has no Triton token")
        sig[m.group(1)] = ("*" + tok) if elem else tok
    return name, sig


def spec_from_json(text, ttir=""):
    """A KernelSpec from JSON_FIELDS' JSON (the Triton backend's pytorchsim_spec option)."""
    got = json.loads(text)
    unknown = sorted(set(got) - set(JSON_FIELDS))
    if unknown:
        raise ValueError(f"a JSON spec holds {', '.join(JSON_FIELDS)}, not {', '.join(unknown)}")
    if not got.get("name") or not got.get("signature"):
        name, sig = signature_from_ttir(ttir)
        got["name"] = got.get("name") or name
        got["signature"] = got.get("signature") or sig
    pointers = [(n, _TOKEN_DTYPE[t[1:]]) for n, t in got["signature"].items() if t.startswith("*")]
    wanted = got.pop("args")
    if len(wanted) != len(pointers):
        raise ValueError(f"{got['name']}: the spec states {len(wanted)} tensors, its kernel takes {len(pointers)}")
    args = [Arg(a.get("name") or n, a["role"], a.get("dtype") or d, tuple(a["shape"])) for a, (n, d) in zip(wanted, pointers)]
    got["grid"] = tuple(got["grid"])
    if got.get("parallel_axes") is not None:
        got["parallel_axes"] = tuple(got["parallel_axes"])
    return KernelSpec(kernel=None, constexprs={}, args=args, reference=None, make_inputs=None, ttir=ttir, **got)


def spec_to_json(spec):
    """The JSON_FIELDS of `spec` as text (what the Triton backend passes as pytorchsim_spec)."""
    out = {}
    for f in JSON_FIELDS:
        v = getattr(spec, f)
        if f == "args":
            v = [{"name": a.name, "role": a.role, "dtype": a.dtype, "shape": list(a.shape)} for a in v]
        elif isinstance(v, tuple):
            v = list(v)
        out[f] = v
    return json.dumps(out)


def load_spec(path):
    """Import a kernel file and return its SPEC; a .json file is a JSON spec with its .ttir beside it."""
    if path.endswith(".json"):
        with open(path) as f:
            return spec_from_json(f.read(), os.path.splitext(os.path.abspath(path))[0] + ".ttir")
    modspec = importlib.util.spec_from_file_location("pytorchsim_kernel_" + os.path.basename(path).replace(".", "_"), path)
    mod = importlib.util.module_from_spec(modspec)
    modspec.loader.exec_module(mod)
    if not hasattr(mod, "SPEC"):
        raise SystemExit(f"{path}: a kernel file defines a module-level SPEC (KernelSpec)")
    spec = mod.SPEC
    spec.extra.setdefault("source_path", os.path.abspath(path))
    return spec
