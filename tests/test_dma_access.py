"""The DMA-access trace (runtime/dma_access.py), on the host: for every committed kernel object,

  - every element a map stream names lies inside its tensor (a masked load's map may reach outside: the
    program's mask keeps those reads from happening);
  - the write footprints of a launch cut into unit ranges are the whole launch's, range by range (the split
    the multi-GPU launch relies on);
  - the headline programs move the bytes their roofline counts;
  - the trace file a launch leaves under the runtime directory reads back, with the grouped GEMM's rows
    resolved from its group tables.
The GPU test (tests/test_gpu_canary.py) checks the write footprints against what the kernels write."""
import json
import os

import numpy as np
import pytest

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.runtime import cuda as RC
from pytorchsim_triton_compiler.runtime import dma_access as DA

HERE = os.path.dirname(os.path.abspath(__file__))
OBJ = os.path.join(HERE, "golden", "objects")
NAMES = sorted(os.listdir(OBJ))


def load(name):
    m = ko.read(os.path.join(OBJ, name))
    return m, D.from_bytes(ko.read_desc(os.path.join(OBJ, name), m))


@pytest.mark.parametrize("name", NAMES)
def test_streams_stay_inside_their_tensors(name):
    m, d = load(name)
    names = [a["name"] for a in m["args"]]
    numel = {a["name"]: ko.numel(a) for a in m["args"]}
    for s in DA.streams(d, 0, d.units, names):
        assert s["arg"] in numel
        b = DA.bounds(s["access"])
        if b is None or s["access"]["map"].get("masked"):
            continue
        assert b[0] >= 0 and b[1] < numel[s["arg"]], f"{name}: {s['dir']} of {s['arg']} leaves the tensor"


def small(name):
    m, d = load(name)
    return d.units >= 2 and sum(ko.numel(a) for a in m["args"]) <= (8 << 20)


@pytest.mark.parametrize("name", [n for n in NAMES if small(n)])
def test_split_ranges_write_what_the_whole_launch_writes(name):
    m, d = load(name)
    names = [a["name"] for a in m["args"]]

    def writes(lo, hi):
        out = {}
        for s in DA.streams(d, lo, hi, names):
            e = DA.elements(s["access"])
            if s["dir"] == "write" and e is not None:
                out.setdefault(s["arg"], []).append(e)
        return {k: np.unique(np.concatenate(v)) for k, v in out.items()}

    whole = writes(0, d.units)
    parts = [writes(lo, hi) for lo, hi in RC.split(d.units, 3)]
    for arg, w in whole.items():
        got = np.unique(np.concatenate([p[arg] for p in parts if arg in p]))
        assert np.array_equal(got, w), f"{name}: the ranges' writes of {arg} differ from the whole launch's"


def test_headline_programs_move_their_roofline_bytes():
    for name, want in (("softmax_4096x4096", 2 * 2 * 4096 * 4096), ("rmsnorm_4096x4096", 2 * 2 * 4096 * 4096 + 2 * 4096)):
        m, d = load(name)
        dt = {a["name"]: a["dtype"] for a in m["args"]}
        size = {"bfloat16": 2, "float32": 4}
        got = sum(s["elements"] * size[dt[s["arg"]]] for s in DA.streams(d, 0, d.units, [a["name"] for a in m["args"]]))
        assert got == want, f"{name}: {got} bytes, the roofline counts {want}"


def test_trace_file_with_resolved_grouped_gemm_rows(tmp_path):
    M, N, K, G, P = 300, 64, 64, 4, 3
    d = B.grouped_gemm(M, N, K, G, P)
    m = {"name": "grouped", "args": [{"name": f"a{i}", "dtype": {1: "bfloat16", 3: "int32"}[d.arg_dtype[i]],
                                      "shape": [d.arg_numel[i]]} for i in range(d.nargs)]}
    p = d.p.ggemm
    host = {f"a{i}": np.zeros(d.arg_numel[i], dtype=np.int32 if d.arg_dtype[i] == 3 else np.uint16) for i in range(d.nargs)}
    host[f"a{p.group_arg}"][:P] = [2, 0, 2]                 # group 2 listed twice: its rows once
    host[f"a{p.start_arg}"][:G + 1] = [0, 100, 150, 250, 300]
    host[f"a{p.rows_arg}"][:G + 1] = [100, 50, 100, 50, 0]
    DA.write(str(tmp_path), m, d, [(0, 0, d.units)], host)
    t = json.load(open(tmp_path / "dma_access" / "trace.json"))
    assert t["format"] == DA.FORMAT and t["kind"] == "grouped_gemm"
    st = {(s["arg"], s["dir"]): s for s in t["ranges"][0]["streams"]}
    c = st[(f"a{p.c_arg}", "write")]["access"]["indirect"]
    assert c["resolved_rows"] == [[0, 100], [150, 250]] and c["rows"] == 200 and c["row_elems"] == N
