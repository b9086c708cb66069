"""The kernel object a device reads (the reference's contract/kernel_object.py): kernel.json, the manifest
of one compiled kernel, and the .raw ABI of its tensors (one flat file per argument, bf16 as uint16 bits).

B200 edition: the object's executable artifact is `desc` (desc.bin, a packed launch descriptor of
include/ptsim_b200.h) in place of the reference's `elf`; the manifest records the lowered program class
under `b200`.  Every field a device or a launcher reads in the reference -- name, args (name, role, dtype,
shape), scalars, grid, grid_bound, abi.parallel_axes, artifacts -- keeps its name and meaning."""
import json
import math
import os

MANIFEST = "kernel.json"
DESC_FILE = "desc.bin"

FORMAT = 11
"""The reference's manifest format number; a B200 manifest adds the `b200` section and the `desc` artifact."""

PROGRAM_KEY_SHIFT = {"x": 0, "y": 21, "z": 42}

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

if set(NP_DTYPE) != set(ITEMSIZE):
    raise ImportError("NP_DTYPE and ITEMSIZE must answer for the same dtypes")

SCALAR_CTYPE = {"i32": "int32_t", "i64": "int64_t", "fp32": "float"}
FLOAT_CTYPES = ("float", "double", "_Float16")


class ObjectError(RuntimeError):
    pass


def numel(arg):
    return math.prod(arg["shape"])


def nbytes(arg):
    return numel(arg) * ITEMSIZE[arg["dtype"]]


def grid3(grid):
    g = list(grid) + [1, 1, 1]
    return g[0], g[1], g[2]


def program_key_fits(grid):
    """Whether every program id of `grid` packs into its PROGRAM_KEY_SHIFT field."""
    return all(g <= 1 << PROGRAM_KEY_SHIFT["y"] for g in grid3(grid))


def refuse_grid_past_bound(manifest, grid):
    """`grid` padded to three axes, or ObjectError when an axis exceeds kernel.json's grid_bound, an axis with
    no program loop is not 1, or a program id does not fit the program key."""
    got = grid3(grid)
    bound = manifest.get("grid_bound")
    over = [f"{a}={g} (bound {b})" for a, g, b in zip("xyz", got, bound or [None] * 3) if b is not None and g > b]
    axes = manifest.get("abi", {}).get("parallel_axes", "xyz")
    loose = [f"{a}={g} is on an axis with no program loop" for a, g in zip("xyz", got) if a not in axes and g != 1]
    if over or loose or not program_key_fits(got):
        raise ObjectError(f"{manifest.get('name')}: launch grid {tuple(got)} is refused; compiled for grids within "
                          f"{tuple(bound) if bound else None} (grid_bound), default {tuple(grid3(manifest['grid']))}: "
                          f"{', '.join(over + loose) or 'a program id past the key'}")
    return got


def argv_order(manifest):
    """Tensor argument names in the order a launch takes their buffers."""
    return [a["name"] for a in manifest["args"]]


def writable(manifest):
    return [a for a in manifest["args"] if a["role"] in ("out", "inout")]


def splittable(manifest):
    """Whether the launch grid may be cut into ranges run independently: no argument is read and written."""
    return not any(a["role"] == "inout" for a in manifest["args"])


def parameters(spec):
    """("tensor", k) / ("scalar", k) for each non-constexpr parameter of the kernel, in signature order."""
    out, t, k = [], 0, 0
    for sig in spec.signature.values():
        if sig == "constexpr":
            continue
        if sig.startswith("*"):
            out.append(("tensor", t))
            t += 1
        else:
            out.append(("scalar", k))
            k += 1
    return out


def runtime_scalars(spec):
    """(name, C type, default) of each scalar parameter, in signature order."""
    values = spec.extra.get("scalar_values", {})
    declared = dict(spec.extra.get("scalar_args", []))
    out = []
    for name, sig in spec.signature.items():
        if sig == "constexpr" or sig.startswith("*"):
            continue
        ctype = declared.get(name) or SCALAR_CTYPE.get(sig)
        if ctype is None:
            raise ValueError(f"kernel {spec.name}: no C type known for scalar '{name}: {sig}'")
        out.append((name, ctype, values.get(name)))
    return out


def scalar_entries(spec):
    return [{"name": n, "ctype": c, "default": d} for n, c, d in runtime_scalars(spec)]


def scalar_value(manifest, s, values=None):
    v = (values or {}).get(s["name"], s["default"])
    if v is None:
        raise ObjectError(f"{manifest['name']}: scalar '{s['name']}' has no value for this launch and no default")
    return v


def _prefetch_list(graph_prefetch):
    return None if graph_prefetch is None else list(graph_prefetch)


def disagreements(manifest, spec):
    """Every question both the manifest and the spec answer, answered differently."""
    return [what for what, mine, theirs in (
        ("argv_order", argv_order(manifest), [a.name for a in spec.args]),
        ("scalars", [x["name"] for x in manifest.get("scalars", [])], [n for n, _, _ in runtime_scalars(spec)]),
        ("grid3", grid3(manifest["grid"]), grid3(spec.grid)),
        ("numel", [numel(a) for a in manifest["args"]], [a.numel for a in spec.args]),
        ("writable", [a["name"] for a in writable(manifest)], [a.name for a in spec.outputs()]),
        ("graph_prefetch", [manifest.get("graph_prefetch")], [_prefetch_list(spec.graph_prefetch)]),
    ) if list(mine) != list(theirs)]


def refuse_if_it_disagrees(manifest, spec):
    bad = disagreements(manifest, spec)
    if bad:
        raise ObjectError(f"{spec.name}: the manifest and the spec disagree about {', '.join(bad)}; the object was "
                          f"written by a different compile")


def describe(spec, lowered, artifacts, grid_bound=None):
    """The manifest of one lowered kernel: `lowered` is the lowering's summary (program class, units)."""
    return {
        "format": FORMAT,
        "name": spec.name,
        "grid": list(spec.grid),
        "grid_bound": None if grid_bound is None else list(grid_bound),
        "target": {"name": "b200", "arch": "sm_100a"},
        "args": [{"name": a.name, "role": a.role, "dtype": a.dtype, "shape": list(a.shape)} for a in spec.args],
        "scalars": scalar_entries(spec),
        "abi": {"parallel_axes": list(spec.parallel_axes)},
        "artifacts": {k: v for k, v in artifacts.items() if v},
        "graph_prefetch": _prefetch_list(spec.graph_prefetch),
        "b200": lowered,
    }


def write(workdir, spec, lowered, blob, grid_bound=None):
    """Write desc.bin and kernel.json into `workdir`; return the manifest's path."""
    os.makedirs(workdir, exist_ok=True)
    with open(os.path.join(workdir, DESC_FILE), "wb") as fh:
        fh.write(blob)
    path = os.path.join(workdir, MANIFEST)
    with open(path, "w") as fh:
        json.dump(describe(spec, lowered, {"desc": DESC_FILE}, grid_bound), fh, indent=2)
        fh.write("\n")
    return path


def read(workdir):
    path = os.path.join(workdir, MANIFEST)
    try:
        with open(path) as fh:
            got = json.load(fh)
    except OSError as e:
        raise ObjectError(f"{path}: {e.strerror}. A kernel object carries its own manifest; this directory was not "
                          f"produced by a compile that reached the binary stage.")
    except json.JSONDecodeError as e:
        raise ObjectError(f"{path}: not valid JSON ({e})")
    if got.get("format") != FORMAT:
        raise ObjectError(f"{path}: manifest format {got.get('format')!r}; this build reads format {FORMAT}")
    return got


def artifact(workdir, kind, required=True, manifest=None):
    got = read(workdir) if manifest is None else manifest
    rel = got.get("artifacts", {}).get(kind)
    if not rel:
        if not required:
            return None
        have = ", ".join(sorted(got.get("artifacts", {}))) or "none"
        raise ObjectError(f"{workdir}: this kernel object has no `{kind}`. It has: {have}.")
    return os.path.join(workdir, rel)


def read_desc(workdir, manifest=None):
    """The descriptor blob of the kernel object in `workdir`."""
    with open(artifact(workdir, "desc", manifest=manifest), "rb") as fh:
        return fh.read()
