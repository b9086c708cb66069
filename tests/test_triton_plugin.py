"""The Triton backend plugin as a caller reaches it (the reference's tests/runtime/triton_backend_cases.py):
triton.compile with pytorchsim_spec runs Triton's front end and the B200 lowering and yields the launch
descriptor with its kernel object; a refused program is a RuntimeError naming the compiler gap, never
OutOfResources; a launch goes to the registered launcher (constexpr arguments dropped, their values named in
the kernel object) or raises.  Fake launchers on the CPU, as the reference tests it; the GPU case launches
through cuda_launcher on real tensors and checks the result against the oracle."""
import json
import os

import pytest

triton = pytest.importorskip("triton")

from pytorchsim_triton_backend import register  # noqa: E402
from pytorchsim_triton_compiler.codegen import descriptors as D  # noqa: E402
from pytorchsim_triton_compiler.contract.kernel_spec import load_spec, spec_to_json  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ADD = os.path.join(HERE, "kernels", "vector_add.py")
SOFTMAX = os.path.join(HERE, "kernels", "row_softmax.py")
ATOMIC = os.path.join(HERE, "kernels", "atomic_accumulate.py")

register()


def _compile(path, device_type="cpu", with_spec=True, derive=False, constexprs=None, spec_text=None, **options):
    from triton.backends.compiler import GPUTarget
    from triton.compiler.compiler import ASTSource
    spec = load_spec(path)
    text = spec_to_json(spec) if spec_text is None else spec_text
    if derive:
        got = json.loads(text)
        got.pop("name"), got.pop("signature")
        got["args"] = [{"role": a["role"], "shape": a["shape"]} for a in got["args"]]
        text = json.dumps(got)
    src = ASTSource(fn=spec.kernel(), signature=spec.signature, constexprs={**spec.constexprs, **(constexprs or {})})
    opts = {**({"pytorchsim_spec": text} if with_spec else {}), **options}
    return triton.compile(src, target=GPUTarget(device_type, 0, 0), options=opts)


def _launcher(seen, what):
    from triton.backends.pytorchsim.driver import set_launcher
    set_launcher(lambda binary, kobj, grid, args, artifacts=None: seen.append(what(binary, kobj, grid, args)))


def test_small_kernel_yields_a_descriptor():
    got = _compile(ADD)
    blob = got.asm["obj"]
    d = D.from_bytes(blob)
    kobj = json.loads(got.metadata.kernel_object)
    assert d.kind == D.ELEMENTWISE and d.p.ew.numel == 1 << 16
    assert kobj["name"] == got.name == "add_kernel"
    assert [a["name"] for a in kobj["args"]] == ["x_ptr", "y_ptr", "o_ptr"]


def test_launch_goes_to_the_registered_launcher():
    from pytorchsim_triton_backend.driver import activated
    seen = []
    with activated():
        _launcher(seen, lambda b, k, g, a: (bytes(b[:4]), json.loads(k)["name"], g, a))
        _compile(ADD)[(64, 1, 1)]("a", "b", "c", 8)
    assert seen == [(D.MAGIC.to_bytes(4, "little"), "add_kernel", (64, 1, 1), ("a", "b", "c", 8))]


def test_launch_without_a_launcher_raises():
    from triton.backends.pytorchsim.driver import set_launcher
    from pytorchsim_triton_backend.driver import activated
    with activated():
        set_launcher(None)
        with pytest.raises(RuntimeError, match="set_launcher"):
            _compile(ADD)[(1, 1, 1)]("a", "b", "c", 8)


def test_launch_drops_constexpr_arguments_and_names_their_values():
    from pytorchsim_triton_backend.driver import activated
    seen = []
    with activated():
        _launcher(seen, lambda b, k, g, a: (a, json.loads(k).get("constexprs")))
        got = _compile(ADD)
        sig = list(got.src.signature.values())
        got[(64, 1, 1)](*[("p%d" % i) if t != "constexpr" else 1024 for i, t in enumerate(sig)])
    assert seen == [(tuple("p%d" % i for i, t in enumerate(sig) if t != "constexpr"), {"BLOCK": 1024})]


def test_a_compiler_gap_is_an_error_not_a_dropped_config():
    from triton.runtime.errors import OutOfResources
    try:
        _compile(ATOMIC)
    except OutOfResources as e:  # pragma: no cover -- the failure this test exists to catch
        pytest.fail(f"dropped as a capacity limit: {e}")
    except RuntimeError as e:
        assert "compiler gap (atomics)" in str(e), str(e)
    else:
        pytest.fail("an atomic accumulation compiled")


def test_internal_error_stays_a_runtime_error():
    with pytest.raises(RuntimeError, match="pytorchsim-triton-compiler failed"):
        _compile(ADD, spec_text=json.dumps({"args": []}))


def test_compile_without_a_spec_is_not_launchable():
    from pytorchsim_triton_backend.driver import activated
    with activated():
        _launcher([], lambda *a: None)
        got = _compile(ADD, with_spec=False)
        assert got.name == "add_kernel" and got.metadata.kernel_object == ""
        with pytest.raises(RuntimeError, match="without pytorchsim_spec"):
            got[(1, 1, 1)]("a", "b", "c", 8)


def test_spec_without_signature_reads_it_off_the_ir():
    full, derived = _compile(ADD), _compile(ADD, derive=True)
    a, b = json.loads(full.metadata.kernel_object), json.loads(derived.metadata.kernel_object)
    assert [(x["role"], x["dtype"], x["shape"]) for x in a["args"]] == [(x["role"], x["dtype"], x["shape"]) for x in b["args"]]
    assert a["name"] == b["name"] and [x["name"] for x in b["args"]] == ["x_ptr", "y_ptr", "o_ptr"]
    assert full.asm["obj"] == derived.asm["obj"]


def test_every_reference_target_name_compiles():
    blobs = {t: _compile(ADD, device_type=t).asm["obj"] for t in ("cpu", "npu", "b200")}
    assert len(set(blobs.values())) == 1


def test_a_kernel_compiles_at_two_configs():
    spec = load_spec(SOFTMAX)
    xb = spec.constexprs.get("XBLOCK")
    assert xb is not None
    a = D.from_bytes(_compile(SOFTMAX).asm["obj"])
    b = D.from_bytes(_compile(SOFTMAX, constexprs={"XBLOCK": xb // 2},
                              spec_text=json.dumps({**json.loads(spec_to_json(spec)), "grid": [spec.grid[0] * 2]})).asm["obj"])
    assert a.kind == b.kind == D.ROW_SOFTMAX
    assert (a.p.row.rows, a.p.row.cols) == (b.p.row.rows, b.p.row.cols) and a.grid[0] * 2 == b.grid[0]


def test_backend_hash_follows_the_pipeline_source():
    from triton.backends.compiler import GPUTarget
    from triton.backends.pytorchsim.compiler import CPUBackend, _pipeline_fingerprint
    import pytorchsim_triton_compiler as package
    probe = os.path.join(os.path.dirname(package.__file__), "_fingerprint_probe.py")
    before = CPUBackend(GPUTarget("cpu", 0, 0)).hash()
    try:
        with open(probe, "w") as f:
            f.write("X = 1\n")
        _pipeline_fingerprint.cache_clear()
        after = CPUBackend(GPUTarget("cpu", 0, 0)).hash()
    finally:
        os.remove(probe)
        _pipeline_fingerprint.cache_clear()
    assert before != after


def test_keep_option_leaves_the_workdir(tmp_path, monkeypatch):
    import shutil
    # A private Triton cache: a cached compile from an earlier run would name a workdir that run removed.
    monkeypatch.setenv("TRITON_CACHE_DIR", str(tmp_path / "triton-cache"))
    gone, kept = _compile(ADD), _compile(ADD, pytorchsim_keep_workdir=True)
    work = kept.metadata.workdir
    try:
        assert sorted(os.listdir(work)) == ["desc.bin", "kernel.json", "spec.json", "spec.ttir"]
        assert "workdir" not in gone.metadata._asdict()
    finally:
        shutil.rmtree(work, ignore_errors=True)


def test_timing_graph_is_refused():
    with pytest.raises(RuntimeError, match="timing graph"):
        _compile(ADD, pytorchsim_tog=True)


@pytest.mark.gpu
def test_plugin_launch_runs_on_the_b200():
    """triton.compile -> kernel[grid](tensors) -> cuda_launcher -> the executor, bit exact against x + y."""
    import torch
    from pytorchsim_triton_backend.driver import activated, cuda_launcher, set_launcher
    from oracle import programs as O
    n = 1 << 16
    g = torch.Generator().manual_seed(5)
    x, y = torch.randn(n, generator=g), torch.randn(n, generator=g)
    xs, ys, o = x.cuda(), y.cuda(), torch.zeros(n, device="cuda")
    with activated():
        set_launcher(cuda_launcher)
        try:
            _compile(ADD)[(64, 1, 1)](xs, ys, o, n)
        finally:
            set_launcher(None)
    assert torch.equal(o.cpu(), O.vector_add(x, y))


@pytest.mark.gpu
def test_plugin_launch_writes_a_strided_output_view():
    """A written argument that is a non-contiguous view runs on a contiguous copy, and the result is copied
    back into the caller's view; the elements between the view's elements keep their values."""
    import torch
    from pytorchsim_triton_backend.driver import activated, cuda_launcher, set_launcher
    from oracle import programs as O
    n = 1 << 16
    g = torch.Generator().manual_seed(6)
    x, y = torch.randn(n, generator=g), torch.randn(n, generator=g)
    backing = torch.full((2 * n,), -7.0, device="cuda")
    o = backing[::2]
    assert not o.is_contiguous()
    with activated():
        set_launcher(cuda_launcher)
        try:
            _compile(ADD)[(64, 1, 1)](x.cuda(), y.cuda(), o, n)
        finally:
            set_launcher(None)
    assert torch.equal(o.cpu(), O.vector_add(x, y))
    assert bool((backing[1::2] == -7.0).all())
