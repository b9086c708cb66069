"""Parity of every executor kernel class with the CPU oracle, through the C ABI (ptsim_launch via ctypes),
on seeded inputs, under the parity bars of oracle/tolerance.py: bit exact for copies and fp32 adds; bf16
results within 1e-2 relative, with no absolute floor and at most 2 ulps for element- and row-wise programs,
a floor of 2^-10 of the row's RMS for GEMM outputs, and attention within the envelope of the reference's
own block-size variation (ATTENTION); fp32 sums within 1e-5 of the summands' magnitudes.  Shapes include the BASELINE.json configurations
(vector add 1,048,576; softmax / RMSNorm 4096 x 4096; GEMM 4096^3 and the M sweep) and ragged edges."""
import math

import pytest
import torch

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.runtime import cuda as RC
from oracle import programs as O
from oracle.tolerance import ATTENTION, CONTRACTION, FP32_SUM, POINTWISE
from tests._helpers import bits_equal, parity, randn

pytestmark = pytest.mark.gpu

def run(desc, tensors):
    ts = [t.cuda() for t in tensors]
    RC.launch_tensors(D.to_bytes(desc), ts)
    return [t.cpu() for t in ts]


@pytest.mark.parametrize("n", [1024, 1_048_576, 1_000_003])
def test_vector_add_bit_exact(n):
    g = torch.Generator().manual_seed(0)
    x, y = torch.randn(n, generator=g), torch.randn(n, generator=g)
    out = run(B.elementwise_add(n), [x, y, torch.zeros(n)])[2]
    assert bits_equal(out, O.vector_add(x, y))


@pytest.mark.parametrize("tokens,heads", [(2048, 8), (128, 8), (2048, 32)])
def test_relayout_copies_bit_exact(tokens, heads):
    dim = 128
    n = tokens * heads * dim
    x = randn(n, 1)
    # 05: out[h, t, d] = in[t, h, d]: flat out index i -> d = i % 128, t = (i // 128) % T, h = i // (T*128)
    d05 = B.copy_map(n, n, [(1, dim, 1), (dim, tokens, heads * dim), (tokens * dim, heads, dim)])
    out = run(d05, [x, torch.zeros(n, dtype=torch.bfloat16)])[1]
    assert bits_equal(out, O.token_to_head_major(x, tokens, heads, dim))
    # 07: out[t, h, d] = in[h, t, d]
    d07 = B.copy_map(n, n, [(1, dim, 1), (dim, heads, tokens * dim), (heads * dim, tokens, dim)])
    out = run(d07, [x, torch.zeros(n, dtype=torch.bfloat16)])[1]
    assert bits_equal(out, O.heads_to_token_major(x, tokens, heads, dim))


@pytest.mark.parametrize("tokens,inter", [(64, 12288), (2048, 12288), (3, 24)])
def test_silu_mul(tokens, inter):
    x = randn(tokens * 2 * inter, 2)
    out = run(B.silu_mul(tokens, inter, block=1 << 21), [x, torch.zeros(tokens * inter, dtype=torch.bfloat16)])[1]
    parity(out, O.silu_mul(x, tokens, inter), POINTWISE, name=f"silu_mul {tokens}x{inter}")


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (32, 128), (7, 384), (64, 6144), (16, 8192), (5, 100), (1, 4096)])
def test_softmax(rows, cols):
    x = randn(rows * cols, 3)
    out = run(B.row_softmax(rows, cols), [x, torch.zeros_like(x)])[1]
    parity(out, O.softmax_rows(x, rows, cols), POINTWISE, name=f"softmax {rows}x{cols}")


def test_softmax_nan_propagates():
    rows, cols = 4, 256
    x = randn(rows * cols, 4)
    x[cols + 17] = float("nan")
    out = run(B.row_softmax(rows, cols), [x, torch.zeros_like(x)])[1].float().view(rows, cols)
    assert torch.isnan(out[1]).all() and not torch.isnan(out[0]).any()


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (2048, 4096), (8, 128), (3, 1000)])
def test_rmsnorm(rows, cols):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(rows * cols, generator=g).to(torch.bfloat16)
    w = (torch.randn(cols, generator=g) * 0.02 + 1.0).to(torch.bfloat16)
    out = run(B.row_rmsnorm(rows, cols, 1e-6), [x, w, torch.zeros_like(x)])[2]
    parity(out, O.rmsnorm_rows(x, w, rows, cols, 1e-6), POINTWISE, name=f"rmsnorm {rows}x{cols}")


@pytest.mark.parametrize("tokens,heads", [(2048, 32), (2048, 8), (16, 4)])
def test_qknorm_rope(tokens, heads):
    g = torch.Generator().manual_seed(6)
    x = torch.randn(tokens * heads * 128, generator=g).to(torch.bfloat16)
    w = torch.randn(128, generator=g).to(torch.bfloat16)
    cos, sin = O.rope_tables(tokens)
    out = run(B.qknorm_rope(tokens, heads), [x, w, cos, sin, torch.zeros_like(x)])[4]
    parity(out, O.qknorm_rope(x, w, cos, sin, tokens, heads, 1e-6), POINTWISE, row=128,
           name=f"qknorm_rope {tokens}x{heads}")


@pytest.mark.parametrize("numel,op", [(16_777_216, "sum"), (16_777_216, "max"), (1024, "sum"), (1000, "max")])
def test_reduce_all(numel, op):
    x = randn(numel, 7)
    out = run(B.reduce_all(numel, op), [x, torch.zeros(1)])[1]
    want = O.reduce_all(x, op)
    if op == "max":
        assert bits_equal(out, want)
    else:
        # fp32 sums of N(0,1) values in different orders: bound by the accumulated rounding, relative to
        # the sum of magnitudes (the 1e-5 fp32 bar of the reference, tests/cases/workloads/softmax.py:84).
        parity(out, want, FP32_SUM, magnitude=float(x.float().abs().sum()), name=f"reduce_all {numel}")


def _gemm_case(M, N, K, residual=False, b_kmajor=False, seed=8):
    g = torch.Generator().manual_seed(seed)
    std = 1.0 / math.sqrt(K)   # A, B ~ N(0, 1/sqrt(K))
    a = (torch.randn(M * K, generator=g) * std).to(torch.bfloat16)
    b = (torch.randn(K * N, generator=g) * std).to(torch.bfloat16)
    r = torch.randn(M * N, generator=g).to(torch.bfloat16) if residual else None
    d = B.gemm(M, N, K, residual=residual, b_kmajor=b_kmajor)
    ins = ([r] if residual else []) + [a, b, torch.zeros(M * N, dtype=torch.bfloat16)]
    out = run(d, ins)[-1]
    want = O.gemm(a, b, M, N, K, residual=r, b_kn=not b_kmajor)
    parity(out, want, CONTRACTION, row=N, name=f"gemm M={M} N={N} K={K} residual={residual} b_kmajor={b_kmajor}")


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (128, 4096, 4096), (512, 4096, 4096),
                                   (2048, 4096, 4096), (4096, 4096, 4096), (300, 1000, 200), (2048, 1024, 4096)])
def test_gemm(M, N, K):
    _gemm_case(M, N, K)


@pytest.mark.parametrize("M,N,K", [(2048, 4096, 4096), (256, 512, 12288)])
def test_gemm_residual(M, N, K):
    _gemm_case(M, N, K, residual=True)


@pytest.mark.parametrize("M,N,K", [(512, 1024, 512), (256, 384, 128), (2048, 4096, 512)])
def test_gemm_b_kmajor(M, N, K):
    _gemm_case(M, N, K, b_kmajor=True)


@pytest.mark.parametrize("M,N,K,residual", [(2100, 2560, 520, False), (2304, 4096, 1024, True), (8192, 4096, 256, False)])
def test_gemm_pair_tiles(M, N, K, residual):
    """Shapes with at least one 256 x 256 output tile per cluster run on the 2-CTA kernel: ragged M, N
    and K, the residual epilogue, and many tiles per cluster."""
    _gemm_case(M, N, K, residual=residual)


@pytest.mark.parametrize("batch,hq,hkv,seq,causal", [(1, 4, 1, 256, True), (2, 8, 2, 512, True),
                                                     (1, 2, 2, 256, False), (1, 32, 8, 1024, True),
                                                     (1, 4, 2, 384, True), (2, 2, 1, 128, True),
                                                     (1, 2, 1, 768, False)])
def test_attention(batch, hq, hkv, seq, causal):
    dim = 128
    g = torch.Generator().manual_seed(9)
    q = torch.randn(batch * hq * seq * dim, generator=g).to(torch.bfloat16)
    k = torch.randn(batch * hkv * seq * dim, generator=g).to(torch.bfloat16)
    v = torch.randn(batch * hkv * seq * dim, generator=g).to(torch.bfloat16)
    d = B.attention(batch, hq, hkv, seq, dim, causal)
    out = run(d, [q, k, v, torch.zeros_like(q)])[3]
    want = O.attention_prefill(q, k, v, batch, hq, hq // hkv, seq, dim, min(1024, seq), min(1024, seq), causal,
                               1.0 / math.sqrt(dim))
    parity(out, want, ATTENTION, row=dim, name=f"attention b{batch} hq{hq} hkv{hkv} s{seq} causal={causal}")


def test_unit_ranges_compose():
    """Running units [0, k) and [k, n) writes what [0, n) writes (the split a multi-GPU launch relies on)."""
    rows, cols = 1000, 4096
    x = randn(rows * cols, 10)
    d = D.to_bytes(B.row_softmax(rows, cols, xblock=128))
    whole = torch.zeros_like(x).cuda()
    xs = x.cuda()
    RC.launch_tensors(d, [xs, whole])
    parts = torch.zeros_like(x).cuda()
    units = D.from_bytes(d).units
    RC.launch_tensors(d, [xs, parts], 0, units // 3)
    RC.launch_tensors(d, [xs, parts], units // 3, units)
    assert bits_equal(parts, whole)
