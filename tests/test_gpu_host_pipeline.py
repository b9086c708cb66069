"""runtime.cuda.HostPipeline: launches over host tensors (copies in, kernels, copies back on separate
streams, row launches cut into unit ranges) must write exactly what a device-resident launch writes."""
import pytest
import torch

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.runtime import cuda as RC
from tests._helpers import bits_equal, randn

pytestmark = pytest.mark.gpu


def _device_run(desc, host):
    ts = [t.cuda() for t in host]
    RC.launch_tensors(D.to_bytes(desc), ts)
    return [t.cpu() for t in ts]


@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_pipelined_rows_match_device_launch(chunks):
    rows, cols = 1000, 4096
    x = randn(rows * cols, 11).pin_memory()
    w = (randn(cols, 12).float() * 0.02 + 1.0).to(torch.bfloat16).pin_memory()
    xr = randn(rows * cols, 13).pin_memory()
    d_s = B.row_softmax(rows, cols, xblock=64)
    d_r = B.row_rmsnorm(rows, cols, 1e-6)
    ys = torch.zeros(rows * cols, dtype=torch.bfloat16).pin_memory()
    yr = torch.zeros(rows * cols, dtype=torch.bfloat16).pin_memory()
    pipe = RC.HostPipeline(0, chunks=chunks)
    pipe.submit(D.to_bytes(d_s), [x, ys])
    pipe.submit(D.to_bytes(d_r), [xr, w, yr])
    pipe.wait()
    assert bits_equal(ys, _device_run(d_s, [x, torch.zeros_like(x)])[1])
    assert bits_equal(yr, _device_run(d_r, [xr, w, torch.zeros_like(xr)])[2])


def test_pipelined_whole_launch_kinds():
    M, N, K = 256, 512, 256
    a = randn(M * K, 14)
    b = randn(K * N, 15)
    d = B.gemm(M, N, K)
    c = torch.zeros(M * N, dtype=torch.bfloat16)
    pipe = RC.HostPipeline(0)
    pipe.submit(D.to_bytes(d), [a, b, c])
    x = randn(1 << 20, 16)
    s = torch.zeros(1)
    dr = B.reduce_all(1 << 20, "max")
    pipe.submit(D.to_bytes(dr), [x, s])
    pipe.wait()
    assert bits_equal(c, _device_run(d, [a, b, torch.zeros_like(c)])[2])
    assert bits_equal(s, _device_run(dr, [x, torch.zeros(1)])[1])


def test_pipeline_refuses_device_tensors():
    d = B.elementwise_add(16)
    pipe = RC.HostPipeline(0)
    with pytest.raises(RC.CudaError):
        pipe.submit(D.to_bytes(d), [torch.zeros(16, device="cuda"), torch.zeros(16), torch.zeros(16)])


def test_pipelined_moe_kinds():
    """Kinds with two outputs (top-k values and indices), integer tables (expert counts and running counts)
    and the combine's gather-sum: the pipeline copies back every written argument, bit for bit what a
    device-resident launch writes."""
    g = torch.Generator().manual_seed(17)
    rows, cols, k = 512, 128, 8
    x = torch.randn(rows * cols, generator=g)
    d_t = B.topk(rows, cols, k)
    d_c = B.expert_counts(4096, 128)
    ids = torch.randint(0, 128, (4096,), generator=g)
    outs_t = [torch.zeros(rows * k), torch.zeros(rows * k, dtype=torch.int64)]
    outs_c = [torch.zeros(128, dtype=torch.int64), torch.zeros(4096 * 128, dtype=torch.int64)]
    pipe = RC.HostPipeline(0)
    pipe.submit(D.to_bytes(d_t), [x] + outs_t)
    pipe.submit(D.to_bytes(d_c), [ids] + outs_c)
    pipe.wait()
    want_t = _device_run(d_t, [x, torch.zeros(rows * k), torch.zeros(rows * k, dtype=torch.int64)])
    want_c = _device_run(d_c, [ids, torch.zeros(128, dtype=torch.int64), torch.zeros(4096 * 128, dtype=torch.int64)])
    assert bits_equal(outs_t[0], want_t[1]) and bits_equal(outs_t[1], want_t[2])
    assert bits_equal(outs_c[0], want_c[1]) and bits_equal(outs_c[1], want_c[2])
