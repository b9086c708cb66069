"""ptsim_launch_reduce_noalloc: the whole-tensor reduction for callers that cannot allocate device memory
(a foreign-language binding holding only the raw pointers it was handed, a host whose memory pool owns
the GPU, a caller that may not synchronise the device as cudaMalloc does).  Its pass-1 partials live in
a fixed 4 KiB array inside the library.  Checked here against ptsim_launch with a caller workspace, on
two calls in a row with different inputs (the second call must not see the first one's partials), with
the tolerances of the other reduction tests: bit-exact for max, 1e-5 of the sum of magnitudes for sum.
This file is collected last."""
import pytest
import torch

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.runtime import native

pytestmark = pytest.mark.gpu


def _with_workspace(blob, x, stream):
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    n = native.workspace_size(blob, 0)
    ws = torch.empty(max(1, n), dtype=torch.uint8, device="cuda")
    native.launch(blob, [x.data_ptr(), out.data_ptr()], 0, D.from_bytes(blob).units, ws.data_ptr(), n, stream)
    native.sync(stream)
    return out


@pytest.mark.parametrize("numel,op", [(16_777_216, "sum"), (16_777_216, "max"), (1000, "sum"), (4099, "max")])
def test_noalloc_reduce_matches_launch(numel, op):
    native.init(0)
    stream = torch.cuda.current_stream().cuda_stream
    blob = D.to_bytes(B.reduce_all(numel, op))
    for call, seed in enumerate((31, 32)):
        g = torch.Generator().manual_seed(seed)
        x = (torch.randn(numel, generator=g) * (call + 1)).to(torch.bfloat16).cuda()
        want = _with_workspace(blob, x, stream)
        got = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
        native.launch_reduce_noalloc(blob, [x.data_ptr(), got.data_ptr()], stream)
        native.sync(stream)
        w, r = float(want.item()), float(got.item())
        if op == "max":
            assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (call + 1, r, w)
        else:
            assert abs(r - w) <= 1e-5 * float(x.float().abs().sum()), (call + 1, r, w)


def test_noalloc_rejects_scratch_beyond_the_array():
    native.init(0)
    d = B.reduce_all(1024, "sum")
    d.workspace_bytes = 64 << 10          # declares more scratch than the 4 KiB array holds
    blob = D.to_bytes(d)
    x = torch.ones(1024, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(1, device="cuda")
    with pytest.raises(native.ExecutorError) as e:
        native.launch_reduce_noalloc(blob, [x.data_ptr(), out.data_ptr()], 0)
    assert e.value.code == D.E_RESOURCE and "static scratch" in str(e.value)
    assert float(out.item()) == 0.0


def test_noalloc_rejects_other_kinds():
    native.init(0)
    blob = D.to_bytes(B.elementwise_add(1024))
    t = [torch.zeros(1024, device="cuda") for _ in range(3)]
    with pytest.raises(native.ExecutorError) as e:
        native.launch_reduce_noalloc(blob, [a.data_ptr() for a in t], 0)
    assert e.value.code == D.E_UNSUPPORTED
