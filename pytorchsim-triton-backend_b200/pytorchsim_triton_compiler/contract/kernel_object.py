"""The kernel object a device launches: a directory holding kernel.json (the manifest) and the executable
artifact, with one flat .raw file per tensor argument at launch time (bf16 stored as uint16 bits).

The manifest's fields keep the reference's names and meaning (pytorchsim_triton_compiler/contract/
kernel_object.py): name, args (name, role, dtype, shape), scalars (name, ctype, default), grid, grid_bound,
abi.parallel_axes, artifacts, graph_prefetch, format 11; the dtype tables NP_DTYPE / ITEMSIZE are the .raw
ABI.  The B200 object differs in two places:
  - its artifact is `desc` (desc.bin, a packed ptsim_desc of include/ptsim_b200.h) where the reference has
    `elf`, and a `b200` section records the lowered program class;
  - a scalar's `default` is also the value the descriptor was lowered with: the executor folds scalars
    into the descriptor, so a launch that passes another value is refused (check_launch_scalars) rather
    than silently run with the old one."""
import json
import math
import os

MANIFEST = "kernel.json"
DESC_FILE = "desc.bin"
FORMAT = 11

# Bits of the program key each grid axis's program id occupies (x from bit 0, y from 21, z from 42).
PROGRAM_KEY_SHIFT = {"x": 0, "y": 21, "z": 42}
_AXIS_ID_LIMIT = 1 << PROGRAM_KEY_SHIFT["y"]

# .raw element types: the numpy dtype each kernel.json dtype is stored as, and its size in bytes.
NP_DTYPE = {
    "float64": "float64", "float32": "float32", "float16": "float16",
    "bfloat16": "uint16", "float8_e5m2": "uint8", "float8_e4m3fn": "uint8",
    "int64": "int64", "int32": "int32", "int16": "int16", "int8": "int8",
    "uint64": "uint64", "uint32": "uint32", "uint16": "uint16", "uint8": "uint8",
    "bool": "int8",
}
ITEMSIZE = {
    "float64": 8, "float32": 4, "float16": 2, "bfloat16": 2, "float8_e5m2": 1, "float8_e4m3fn": 1,
    "int64": 8, "int32": 4, "int16": 2, "int8": 1,
    "uint64": 8, "uint32": 4, "uint16": 2, "uint8": 1,
    "bool": 1,
}
assert NP_DTYPE.keys() == ITEMSIZE.keys(), "every .raw dtype needs a numpy type and a size"

# C types of the kernel's scalar parameters, by Triton signature token.
SCALAR_CTYPE = {"i32": "int32_t", "i64": "int64_t", "fp32": "float", "fp64": "double", "i1": "int32_t"}
FLOAT_CTYPES = ("float", "double", "_Float16")


class ObjectError(RuntimeError):
    """A kernel object that is missing, malformed, or launched in a way its compile did not allow."""


def numel(arg):
    return math.prod(arg["shape"])


def nbytes(arg):
    return numel(arg) * ITEMSIZE[arg["dtype"]]


def grid3(grid):
    """A launch grid as (x, y, z), missing axes 1."""
    x, y, z = (tuple(grid) + (1, 1, 1))[:3]
    return x, y, z


def argv_order(manifest):
    """The tensor arguments' names in launch order."""
    return [a["name"] for a in manifest["args"]]


def writable(manifest):
    """The arguments a launch writes (out and inout)."""
    return [a for a in manifest["args"] if a["role"] != "in"]


def splittable(manifest):
    """Whether the grid may run as independent ranges: no argument is both read and written, so no
    program can read another's store."""
    return all(a["role"] != "inout" for a in manifest["args"])


def refuse_grid_past_bound(manifest, grid):
    """(x, y, z) of `grid`, or ObjectError when the compile did not allow it: an axis larger than the
    manifest's grid_bound, an axis with no program loop (not in abi.parallel_axes) that is not 1, or a
    program id too large for its program-key field."""
    got = grid3(grid)
    bound = list(manifest.get("grid_bound") or [None, None, None])
    looped = manifest.get("abi", {}).get("parallel_axes", list("xyz"))
    problems = []
    for axis, extent, limit in zip("xyz", got, bound):
        if limit is not None and extent > limit:
            problems.append(f"{axis}={extent} exceeds its bound {limit}")
        if axis not in looped and extent != 1:
            problems.append(f"{axis}={extent} but the program has no loop over {axis}")
        if extent > _AXIS_ID_LIMIT:
            problems.append(f"{axis}={extent} does not fit the program key")
    if problems:
        raise ObjectError(f"{manifest.get('name')}: grid {got} refused ({'; '.join(problems)}); lowered for "
                          f"default grid {grid3(manifest['grid'])}, grid_bound {manifest.get('grid_bound')}")
    return got


# ---- scalars ------------------------------------------------------------------------------------------

def scalar_table(spec):
    """The manifest's `scalars`: each non-pointer, non-constexpr parameter of the kernel in signature order,
    its C type (spec.extra["scalar_args"] overrides the token's), and the value the lowering folded into
    the descriptor (spec.extra["scalar_values"], or None when the program does not depend on it)."""
    lowered = spec.extra.get("scalar_values", {})
    ctypes = dict(spec.extra.get("scalar_args", []))
    table = []
    for param, token in spec.signature.items():
        if token == "constexpr" or token.startswith("*"):
            continue
        ctype = ctypes.get(param, SCALAR_CTYPE.get(token))
        if ctype is None:
            raise ValueError(f"{spec.name}: scalar parameter {param} has type {token}, which has no C type here")
        table.append({"name": param, "ctype": ctype, "default": lowered.get(param)})
    return table


def _same_scalar(ctype, a, b):
    if ctype in FLOAT_CTYPES:
        import numpy as np
        cast = np.float32 if ctype == "float" else np.float64
        return bool(cast(a) == cast(b)) or (a != a and b != b)
    return int(a) == int(b)


def check_launch_scalars(manifest, values):
    """Refuse a launch whose scalar values differ from those the descriptor was lowered with.  `values`:
    {name: value}, or a sequence in the manifest's scalar order (the Triton launcher's positional scalars).
    A scalar lowered without a value (the program does not read it) takes any value."""
    if values is None:
        return
    table = manifest.get("scalars", [])
    if not isinstance(values, dict):
        values = list(values)
        if len(values) != len(table):
            raise ObjectError(f"{manifest.get('name')}: {len(values)} scalar values for the kernel's "
                              f"{len(table)} scalar parameters")
        values = {s["name"]: v for s, v in zip(table, values)}
    known = {s["name"]: s for s in table}
    unknown = sorted(set(values) - set(known))
    if unknown:
        raise ObjectError(f"{manifest.get('name')}: no scalar parameter named {', '.join(unknown)}")
    for name, value in values.items():
        s = known[name]
        if s["default"] is not None and not _same_scalar(s["ctype"], value, s["default"]):
            raise ObjectError(f"{manifest.get('name')}: scalar {name} = {value!r} at launch, but the descriptor "
                              f"was lowered with {s['default']!r}; lower the kernel again with this value")


# ---- the manifest and its compile ---------------------------------------------------------------------

def _manifest_view(manifest):
    return {
        "argument order": argv_order(manifest),
        "scalar parameters": [s["name"] for s in manifest.get("scalars", [])],
        "default grid": grid3(manifest["grid"]),
        "argument sizes": [numel(a) for a in manifest["args"]],
        "written arguments": [a["name"] for a in writable(manifest)],
        "graph_prefetch": manifest.get("graph_prefetch"),
    }


def _spec_view(spec):
    return {
        "argument order": [a.name for a in spec.args],
        "scalar parameters": [s["name"] for s in scalar_table(spec)],
        "default grid": grid3(spec.grid),
        "argument sizes": [a.numel for a in spec.args],
        "written arguments": [a.name for a in spec.args if a.role != "in"],
        "graph_prefetch": None if spec.graph_prefetch is None else list(spec.graph_prefetch),
    }


def refuse_if_it_disagrees(manifest, spec):
    """ObjectError when the kernel object in hand was not compiled from `spec` (another compile wrote it)."""
    mine, theirs = _manifest_view(manifest), _spec_view(spec)
    differ = [k for k in mine if mine[k] != theirs[k]]
    if differ:
        raise ObjectError(f"{spec.name}: the kernel object does not match its spec ({', '.join(differ)} "
                          f"differ); it was written by another compile")


def describe(spec, lowered, artifacts, grid_bound=None):
    """The manifest of a lowered kernel; `lowered` is the lowering's summary (program class, units)."""
    manifest = {"format": FORMAT, "name": spec.name, "grid": list(spec.grid),
                "grid_bound": list(grid_bound) if grid_bound is not None else None,
                "target": {"name": "b200", "arch": "sm_100a"}}
    manifest["args"] = [dict(name=a.name, role=a.role, dtype=a.dtype, shape=list(a.shape)) for a in spec.args]
    manifest["scalars"] = scalar_table(spec)
    manifest["abi"] = {"parallel_axes": list(spec.parallel_axes)}
    manifest["artifacts"] = {kind: rel for kind, rel in artifacts.items() if rel}
    manifest["graph_prefetch"] = None if spec.graph_prefetch is None else list(spec.graph_prefetch)
    manifest["b200"] = lowered
    return manifest


def write(workdir, spec, lowered, blob, grid_bound=None):
    """Write desc.bin and kernel.json of a lowered kernel into `workdir`; returns kernel.json's path."""
    os.makedirs(workdir, exist_ok=True)
    with open(os.path.join(workdir, DESC_FILE), "wb") as fh:
        fh.write(blob)
    path = os.path.join(workdir, MANIFEST)
    text = json.dumps(describe(spec, lowered, {"desc": DESC_FILE}, grid_bound), indent=2)
    with open(path, "w") as fh:
        fh.write(text + "\n")
    return path


def read(workdir):
    """The manifest in `workdir`; ObjectError when there is none or it is not this format."""
    path = os.path.join(workdir, MANIFEST)
    if not os.path.isfile(path):
        raise ObjectError(f"{path}: no manifest; this directory holds no compiled kernel object")
    with open(path) as fh:
        text = fh.read()
    try:
        manifest = json.loads(text)
    except json.JSONDecodeError as e:
        raise ObjectError(f"{path}: not JSON ({e})") from None
    if manifest.get("format") != FORMAT:
        raise ObjectError(f"{path}: manifest format {manifest.get('format')!r}, this executor reads {FORMAT}")
    return manifest


def artifact(workdir, kind, required=True, manifest=None):
    """Path of the object's artifact `kind` (e.g. "desc"), or None when it has none and it is optional."""
    manifest = read(workdir) if manifest is None else manifest
    kinds = manifest.get("artifacts", {})
    if kinds.get(kind):
        return os.path.join(workdir, kinds[kind])
    if required:
        raise ObjectError(f"{workdir}: the kernel object has no {kind!r} artifact (it has: "
                          f"{', '.join(sorted(kinds)) or 'none'})")
    return None


def read_desc(workdir, manifest=None):
    """The launch descriptor (desc.bin bytes) of the kernel object in `workdir`."""
    with open(artifact(workdir, "desc", manifest=manifest), "rb") as fh:
        return fh.read()
