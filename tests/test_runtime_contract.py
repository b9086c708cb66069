"""The launcher contract, driven with fakes as the reference's own cases drive runtime/spike.launch
(tests/runtime/spike_launch_cases.py:28-119, triton_backend_cases.py:86-106): unit ranges split at
total*w//n, written bytes merge when ranges are disjoint, a clash reruns the grid on one device, an inout
argument keeps the launch on one device, a grid past grid_bound is refused, and the Triton-side launcher
registry hands (binary, kernel_object, grid, args) to whoever registered."""
import json
import os
import tempfile

import numpy as np
import pytest

from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.contract.kernel_spec import KernelSpec, Arg, load_spec, spec_from_json, spec_to_json
from pytorchsim_triton_compiler.runtime import cuda as RC
from pytorchsim_triton_compiler.runtime import device
import pytorchsim_triton_backend.driver as drv


def manifest(n, role="out", grid=None, bound=None):
    return {"name": "k", "grid": [grid or n], "grid_bound": bound, "scalars": [], "abi": {"parallel_axes": ["x"]},
            "args": [{"name": "o", "role": role, "dtype": "uint8", "shape": [n]}]}


def test_split_edges_match_the_reference_rule():
    assert RC.split(8, 4) == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert RC.split(5, 3) == [(0, 1), (1, 3), (3, 5)]
    assert RC.split(2, 4) == [(0, 1), (1, 2)]


def test_inout_is_one_device():
    said = []
    assert RC.jobs(manifest(8, role="inout"), 8, said.append, want=4, ndev=8) == 1
    assert "read as well as written" in said[0]
    assert RC.jobs(manifest(8), 8, said.append, want=None, ndev=8) == 8
    assert RC.jobs(manifest(8), 3, said.append, want=None, ndev=8) == 3


def test_disjoint_ranges_merge_to_the_whole():
    m = manifest(8)
    base = {"o": np.zeros(8, dtype=np.uint8)}

    def part(lo, hi):
        b = np.zeros(8, dtype=np.uint8)
        b[lo:hi] = np.arange(lo, hi) + 1
        return {"o": b}

    got = RC.merge(m, base, [part(lo, hi) for lo, hi in RC.split(8, 4)])
    assert list(got["o"]) == list(range(1, 9))


def test_a_clash_is_not_splittable():
    m = manifest(8)
    base = {"o": np.zeros(8, dtype=np.uint8)}
    a, b = np.zeros(8, dtype=np.uint8), np.zeros(8, dtype=np.uint8)
    a[0], b[0] = 1, 2
    with pytest.raises(RC.NotSplittable):
        RC.merge(m, base, [{"o": a}, {"o": b}])


def test_grid_past_bound_is_refused():
    m = manifest(8, bound=[8, 1, 1])
    assert ko.refuse_grid_past_bound(m, (8,)) == (8, 1, 1)
    with pytest.raises(ko.ObjectError):
        ko.refuse_grid_past_bound(m, (9,))
    with pytest.raises(ko.ObjectError):
        ko.refuse_grid_past_bound(m, (8, 2))  # an axis with no program loop


def test_launch_without_a_gpu_fails_loudly():
    m = manifest(8)
    with tempfile.TemporaryDirectory() as d:
        raw = os.path.join(d, "o.raw")
        np.zeros(8, dtype=np.uint8).tofile(raw)
        from pytorchsim_triton_compiler.codegen import build as B
        from pytorchsim_triton_compiler.codegen import descriptors as D
        blob = D.to_bytes(B.copy_map(8, 8, [(1, 8, 1)], dtype="uint8"))
        with pytest.raises(RC.CudaError):
            RC.launch(blob, m, d, {"o": raw}, devices=[], log=lambda *_: None)


def test_device_registry():
    assert device.get("cuda").name == "cuda"
    with pytest.raises(device.DeviceError):
        device.get("spike")


def test_launcher_registry_hands_the_launch_over():
    class Src:
        signature = {"x": "*fp32", "y": "*fp32", "o": "*fp32", "n": "constexpr"}
        constants = {(3,): 8}

    class Meta:
        kernel_object = json.dumps({"name": "add_kernel", "grid": [3]})
        artifacts = None

    seen = []
    drv.set_launcher(lambda binary, kobj, grid, args, artifacts=None: seen.append((binary, json.loads(kobj), grid, args)))
    try:
        drv._Launcher(Src(), Meta())(3, 1, 1, 0, b"PTSB", None, None, None, None, "a", "b", "c", 8)
        assert seen[0][0] == b"PTSB" and seen[0][2] == (3, 1, 1) and seen[0][3] == ("a", "b", "c")
        assert seen[0][1]["constexprs"] == {"n": 8}
        os.environ["PYTORCHSIM_COLLECT_FAILURES"] = "1"
        drv._Launcher(Src(), Meta())(3, 1, 1, 0, b"PTSB", None, None, None, None, "a", "b", "c", 8)
        assert len(seen) == 1
    finally:
        os.environ.pop("PYTORCHSIM_COLLECT_FAILURES", None)
        drv.set_launcher(None)
    with pytest.raises(RuntimeError, match="set_launcher"):
        drv._Launcher(Src(), Meta())


def test_manifest_disagreement_is_refused():
    spec = KernelSpec(name="k", kernel=None, signature={"o": "*u8"}, constexprs={}, args=[Arg("o", "out", "uint8", (8,))],
                      grid=(8,), reference=None, make_inputs=None)
    m = manifest(8)
    ko.refuse_if_it_disagrees(m, spec)
    m2 = manifest(9)
    with pytest.raises(ko.ObjectError):
        ko.refuse_if_it_disagrees(m2, spec)


def test_json_spec_round_trip():
    spec = KernelSpec(name="k", kernel=None, signature={"x": "*bf16", "o": "*bf16", "n": "i32"}, constexprs={},
                      args=[Arg("x", "in", "bfloat16", (16,)), Arg("o", "out", "bfloat16", (16,))], grid=(2,),
                      reference=None, make_inputs=None, extra={"scalar_values": {"n": 16}})
    back = spec_from_json(spec_to_json(spec))
    assert [a.name for a in back.args] == ["x", "o"] and back.grid == (2,) and back.extra["scalar_values"] == {"n": 16}
