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


def _scalar_manifest():
    m = manifest(8)
    m["scalars"] = [{"name": "n", "ctype": "int32_t", "default": 8}, {"name": "eps", "ctype": "float", "default": 1e-6},
                    {"name": "unused", "ctype": "int64_t", "default": None}]
    return m


def test_launch_scalars_must_match_the_lowered_values():
    """The descriptor holds the scalars it was lowered with (spike.launch passes them per launch,
    runtime/spike.py:44-56,100-110 in the reference): the same values pass, another value is refused with a
    message that says to lower again, an unknown name is refused, a scalar the program does not read takes
    anything."""
    m = _scalar_manifest()
    ko.check_launch_scalars(m, None)
    ko.check_launch_scalars(m, {"n": 8, "eps": 1e-6, "unused": 12345})
    ko.check_launch_scalars(m, [8, float("1e-6"), 0])
    with pytest.raises(ko.ObjectError, match="lower the kernel again"):
        ko.check_launch_scalars(m, {"n": 9})
    with pytest.raises(ko.ObjectError, match="lowered with"):
        ko.check_launch_scalars(m, {"eps": 1e-5})
    with pytest.raises(ko.ObjectError, match="no scalar parameter"):
        ko.check_launch_scalars(m, {"m": 1})
    with pytest.raises(ko.ObjectError, match="scalar values"):
        ko.check_launch_scalars(m, [8])


def test_launch_from_files_refuses_a_changed_scalar():
    """runtime.cuda.launch refuses before it touches a device (so on a host without one, too)."""
    m = _scalar_manifest()
    with tempfile.TemporaryDirectory() as d:
        raw = os.path.join(d, "o.raw")
        np.zeros(8, dtype=np.uint8).tofile(raw)
        from pytorchsim_triton_compiler.codegen import build as B
        from pytorchsim_triton_compiler.codegen import descriptors as D
        blob = D.to_bytes(B.copy_map(8, 8, [(1, 8, 1)], dtype="uint8"))
        with pytest.raises(RC.CudaError, match="scalar n = 7"):
            RC.launch(blob, m, d, {"o": raw}, devices=[], log=lambda *_: None, scalar_values={"n": 7})


def test_triton_launcher_refuses_a_changed_scalar():
    """cuda_launcher checks Triton's positional scalars (and those Triton specialised into constexprs)
    against the lowered values before any launch."""
    import torch
    m = manifest(8)
    m["scalars"] = [{"name": "n", "ctype": "int32_t", "default": 8}]
    o = torch.zeros(8, dtype=torch.uint8)
    with pytest.raises(ko.ObjectError, match="scalar n = 4"):
        drv.cuda_launcher(b"", json.dumps(m), (8, 1, 1), (o, 4))
    with pytest.raises(ko.ObjectError, match="scalar n = 1"):
        drv.cuda_launcher(b"", json.dumps({**m, "constexprs": {"n": 1}}), (8, 1, 1), (o,))
    with pytest.raises(RuntimeError, match="scalar arguments"):
        drv.cuda_launcher(b"", json.dumps(m), (8, 1, 1), (o,))


def test_every_descriptor_kind_names_its_outputs():
    """HostPipeline copies back what written_args names: every kind the executor runs has an answer that
    agrees with the builder's output argument."""
    from pytorchsim_triton_compiler.codegen import build as B
    from pytorchsim_triton_compiler.codegen import descriptors as D
    cases = {
        D.ELEMENTWISE: (B.elementwise_add(64), [2]), D.ROW_SOFTMAX: (B.row_softmax(4, 128), [1]),
        D.ROW_RMSNORM: (B.row_rmsnorm(4, 128), [2]), D.QKNORM_ROPE: (B.qknorm_rope(4, 2), [4]),
        D.GEMM: (B.gemm(128, 128, 64), [2]), D.ATTN_PREFILL: (B.attention(1, 2, 1, 128), [3]),
        D.REDUCE_ALL: (B.reduce_all(1024), [1]), D.ATTN_DECODE: (B.attention_decode(2, 4, 128), [3]),
        D.ROW_DIVSUM: (B.row_divsum(4, 8), [1]), D.TOPK: (B.topk(4, 128, 8), [1, 2]),
        D.SORT: (B.sort(2, 64), [1, 2]), D.GATHER_ROWS: (B.gather_rows_floordiv(16, 64, 8, 2), [2]),
        D.GROUPED_GEMM: (B.grouped_gemm(64, 64, 64, 4, 4), [5]),
        D.GATHER_SUM: (B.combine_gather_sum(8, 64, 2, 4), [6]),
        D.INT_TABLE: (B.expert_counts(64, 8), [1, 2]), D.ROW_SUM: (B.row_sum(4, 8), [1]),
    }
    assert set(cases) == set(D.KIND_NAME)
    for kind, (desc, want) in cases.items():
        assert desc.kind == kind
        assert RC.written_args(desc) == want, D.KIND_NAME[kind]
    bad = B.elementwise_add(64)
    bad.kind = 99
    with pytest.raises(RC.CudaError, match="no known outputs"):
        RC.written_args(bad)


def test_cli_target_lists_every_kind(capsys):
    from pytorchsim_triton_compiler import cli
    from pytorchsim_triton_compiler.codegen import descriptors as D
    cli.target()
    got = json.loads(capsys.readouterr().out)
    assert got["kinds"] == [D.KIND_NAME[k] for k in sorted(D.KIND_NAME)] and len(got["kinds"]) == 16


def test_signature_from_ttir(tmp_path):
    ttir = tmp_path / "k.ttir"
    ttir.write_text('#loc = loc("k.py":1:0)\nmodule {\n  tt.func public @add_kernel(%arg0: !tt.ptr<f32> '
                    '{tt.divisibility = 16 : i32} loc("x"(#loc)), %arg1: !tt.ptr<bf16> loc("y"(#loc)), '
                    '%arg2: i32 {tt.divisibility = 16 : i32} loc("n"(#loc))) attributes {noinline = false} {\n')
    from pytorchsim_triton_compiler.contract.kernel_spec import signature_from_ttir
    assert signature_from_ttir(str(ttir)) == ("add_kernel", {"arg0": "*fp32", "arg1": "*bf16", "arg2": "i32"})


def test_stop_and_failure_records(tmp_path):
    from pytorchsim_triton_compiler.contract import failure
    from pytorchsim_triton_compiler.contract.stop import Reason, Refused, Stop
    assert Stop("lower", Reason.ATOMICS) == Stop("lower", Reason.ATOMICS)
    Stop("lower", "triton.CompilationError")
    with pytest.raises(ValueError):
        Stop("lower", "NotDotted")
    with pytest.raises(TypeError):
        Refused("atomics", "a string is not a Reason")
    with pytest.raises(AttributeError):
        Stop("lower", Reason.ATOMICS).step = "x"
    assert failure.found(str(tmp_path)) is None
    failure.leave(str(tmp_path), "cuda", failure.DEVICE, "kernel said so", code=202)
    rec = failure.found(str(tmp_path))
    assert (rec.stage, rec.kind, rec.facts) == ("cuda", "device", {"code": 202})
    assert json.load(open(tmp_path / failure.FILE))["format"] == failure.FORMAT
    failure.forget(str(tmp_path))
    assert failure.found(str(tmp_path)) is None
