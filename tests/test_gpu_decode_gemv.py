"""Parity of the decode-side programs on the B200 against the CPU oracle:

  - the M = 1 matmul (gemm_1x* and the Qwen3 decode layer's o-projection, a multiply-reduce program the
    reference runs on its vector unit) on the CUDA-core GEMV path: N-contiguous and K-major matrices,
    ragged N and K, the residual epilogue, fp32 output;
  - one-token GQA attention (attention_decode_*) on the split-key kernel: every group size 1-16, key
    counts from one 64-key tile to 8192, head subsets launched as unit ranges.

Parity bars (oracle/tolerance.py): GEMV outputs as sums of products (1e-2 relative plus 2^-10 of the
output's RMS); decode attention under the ATTENTION bar (per query row of 128 values: 1e-2 relative plus
2^-5 of the row's RMS, the error's RMS within 2^-7 of the output's); the rotary op element-wise (at most 2
ulps); fp32 sums of squares within 1e-5 of themselves.  Unit ranges: bit
exact against the whole launch."""
import math

import pytest
import torch

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.runtime import cuda as RC
from pytorchsim_triton_compiler.runtime import native
from oracle import programs as O
from oracle.tolerance import ATTENTION, CONTRACTION, FP32, FP32_SUM, POINTWISE
from tests._helpers import bits_equal, parity

pytestmark = pytest.mark.gpu

def run(desc, tensors, lo=None, hi=None):
    ts = [t.cuda() for t in tensors]
    if lo is None:
        RC.launch_tensors(D.to_bytes(desc), ts)
    else:
        RC.launch_tensors(D.to_bytes(desc), ts, lo, hi)
    return [t.cpu() for t in ts]


def _gemv_case(N, K, b_kmajor=False, residual=False, out_dtype="bfloat16", seed=21):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(K, generator=g).to(torch.bfloat16)
    b = torch.randn(K * N, generator=g).to(torch.bfloat16)
    r = torch.randn(N, generator=g).to(torch.bfloat16) if residual else None
    d = B.gemv(N, K, b_kmajor=b_kmajor, residual=residual, out_dtype=out_dtype)
    dt = getattr(torch, out_dtype)
    out = run(d, ([r] if residual else []) + [a, b, torch.zeros(N, dtype=dt)])[-1]
    want = O.gemm(a, b, 1, N, K, residual=r, b_kn=not b_kmajor, out_dtype=dt)
    parity(out, want, CONTRACTION if out_dtype == "bfloat16" else FP32,
           name=f"gemv N={N} K={K} b_kmajor={b_kmajor} residual={residual} {out_dtype}")


@pytest.mark.parametrize("K,N", [(4096, 4096), (2048, 2048), (384, 1152), (768, 768), (4096, 2048), (2048, 128),
                                 (3072, 768), (12288, 4096), (8, 8), (200, 72), (1000, 4104)])
def test_gemv(K, N):
    _gemv_case(N, K)


@pytest.mark.parametrize("K,N", [(4096, 4096), (768, 3072), (264, 40), (4096, 12)])
def test_gemv_b_kmajor(K, N):
    _gemv_case(N, K, b_kmajor=True)


def test_gemv_residual_and_fp32_output():
    _gemv_case(4096, 4096, residual=True)
    _gemv_case(1536, 512, out_dtype="float32")


@pytest.mark.parametrize("K,N,residual,out_dtype", [(8192, 8192, False, "bfloat16"), (30000, 2056, True, "bfloat16"),
                                                    (4096, 12296, False, "float32"), (131072, 256, True, "float32")])
def test_gemv_row_streaming(K, N, residual, out_dtype):
    """Matrices from 32M elements stream whole 4 KB row runs with partial columns in scratch: ragged column
    tiles (N not a multiple of 2048), K slices of many rows, the residual and fp32 stores after the sum."""
    _gemv_case(N, K, residual=residual, out_dtype=out_dtype)


def test_gemv_refuses_ragged_columns():
    """N-contiguous rows must be 16-byte vectors: N % 8 != 0 is refused, never approximated."""
    d = B.gemv(12, 64)
    ts = [torch.zeros(64, dtype=torch.bfloat16, device="cuda"), torch.zeros(64 * 12, dtype=torch.bfloat16, device="cuda"),
          torch.zeros(12, dtype=torch.bfloat16, device="cuda")]
    with pytest.raises(native.ExecutorError) as e:
        RC.launch_tensors(D.to_bytes(d), ts)
    assert e.value.code == D.E_UNSUPPORTED


def _decode_inputs(hkv, g, seq, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(hkv * g * 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(hkv * seq * 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(hkv * seq * 128, generator=gen).to(torch.bfloat16)
    o = torch.randn(hkv * g * 128, generator=gen).to(torch.bfloat16)   # inout: fully overwritten
    return q, k, v, o


@pytest.mark.parametrize("hkv,g,seq", [(8, 4, 4096), (8, 4, 8192), (8, 2, 128), (8, 8, 1024), (8, 3, 2048),
                                       (1, 16, 64), (2, 1, 640), (4, 5, 192), (8, 16, 512), (3, 7, 8192)])
def test_attention_decode(hkv, g, seq):
    q, k, v, o = _decode_inputs(hkv, g, seq, 31)
    d = B.attention_decode(hkv, g, seq)
    out = run(d, [q, k, v, o])[3]
    want = O.attention_decode(q, k, v, o, hkv, g, 16, seq, 128, seq, 1 / math.sqrt(128))
    parity(out, want, ATTENTION, row=128, name=f"decode hkv={hkv} G={g} S={seq}")


def test_attention_decode_reference_blocks():
    """A program whose key block BKV is shorter than S (the reference restarts its running max per block):
    the result stays within the bf16 tolerance of the block-for-block oracle."""
    hkv, g, seq, bkv = 8, 4, 2048, 512
    q, k, v, o = _decode_inputs(hkv, g, seq, 32)
    out = run(B.attention_decode(hkv, g, seq, bkv=bkv), [q, k, v, o])[3]
    want = O.attention_decode(q, k, v, o, hkv, g, 16, seq, 128, bkv, 1 / math.sqrt(128))
    parity(out, want, ATTENTION, row=128, name="decode reference blocks")


def test_attention_decode_peaked_scores():
    """Keys aligned with the query (one dominant score per head): the split-key merge carries the
    maximum across chunks without losing the other keys' mass."""
    hkv, g, seq = 4, 4, 4096
    q, k, v, o = _decode_inputs(hkv, g, seq, 33)
    kk = k.view(hkv, seq, 128).float()
    qq = q.view(hkv, g, 128).float()
    for h in range(hkv):
        kk[h, 1234 + 500 * h] = qq[h, 0] * 0.5
    k = kk.to(torch.bfloat16).reshape(-1)
    out = run(B.attention_decode(hkv, g, seq), [q, k, v, o])[3]
    want = O.attention_decode(q, k, v, o, hkv, g, 16, seq, 128, seq, 1 / math.sqrt(128))
    parity(out, want, ATTENTION, row=128, name="decode peaked scores")


def test_attention_decode_unit_ranges_compose():
    """Heads [0, 3) then [3, 8) write exactly what one launch of all 8 writes (the split plan follows the
    whole launch, so each head's chunks and merge order are the same)."""
    hkv, g, seq = 8, 4, 4096
    q, k, v, o = _decode_inputs(hkv, g, seq, 34)
    d = B.attention_decode(hkv, g, seq)
    whole = run(d, [q, k, v, o])[3]
    ts = [t.cuda() for t in (q, k, v, o)]
    RC.launch_tensors(D.to_bytes(d), ts, 0, 3)
    RC.launch_tensors(D.to_bytes(d), ts, 3, 8)
    assert bits_equal(ts[3].cpu(), whole)


def test_attention_decode_workspace_is_required():
    native.init(0)
    d = B.attention_decode(8, 4, 4096)
    blob = D.to_bytes(d)
    assert native.workspace_size(blob, 0) > 0
    ts = [t.cuda() for t in _decode_inputs(8, 4, 4096, 35)]
    with pytest.raises(native.ExecutorError) as e:
        native.launch(blob, [t.data_ptr() for t in ts], 0, 8, 0, 0, torch.cuda.current_stream().cuda_stream)
    assert e.value.code == D.E_RESOURCE


def test_attention_decode_refuses_unsupported():
    """Head dim other than 128 and key counts off the 64-key tile are refused."""
    for d in (B.attention_decode(2, 4, 100), B.attention_decode(2, 4, 256, dim=64)):
        ts = [torch.zeros(int(n), dtype=torch.bfloat16, device="cuda") for n in list(d.arg_numel)[:4]]
        with pytest.raises(native.ExecutorError) as e:
            RC.launch_tensors(D.to_bytes(d), ts)
        assert e.value.code == D.E_UNSUPPORTED


# ---- fused matrix-vector products of the decode layer (vector prologue / output epilogue) -------------------

def _wide_compare(got, want, name):
    """bf16 outputs of K-term sums (one row): the CONTRACTION bar."""
    parity(got, want, CONTRACTION, name=name)


@pytest.mark.parametrize("N,K,residual", [(4096, 4096, False), (24576, 4096, True), (520, 3000, False),
                                          (64, 100000, True), (8, 16, False)])
def test_rmsnorm_gemv(N, K, residual):
    g = torch.Generator().manual_seed(N + K)
    x = torch.randn(K, generator=g).to(torch.bfloat16)
    res = torch.randn(K, generator=g).to(torch.bfloat16)
    w = torch.randn(K, generator=g).to(torch.bfloat16)
    mat = (torch.randn(K * N, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    ss = O.sumsq(x, K, res if residual else None)
    ins = [x] + ([res] if residual else []) + [ss, w, mat, torch.zeros(N, dtype=torch.bfloat16)]
    got = run(B.rmsnorm_gemv(N, K, residual=residual), ins)[-1]
    _wide_compare(got, O.rmsnorm_gemv(x, ss, w, mat, K, N, 1e-6, res=res if residual else None),
                  f"rmsnorm_gemv N={N} K={K} residual={residual}")


@pytest.mark.parametrize("N,K", [(4096, 12288), (1000, 2000), (8, 8)])
def test_silu_gemv(N, K):
    g = torch.Generator().manual_seed(N * 3 + K)
    gu = torch.randn(2 * K, generator=g).to(torch.bfloat16)
    mat = (torch.randn(K * N, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    r1, r2 = (torch.randn(N, generator=g).to(torch.bfloat16) for _ in range(2))
    got = run(B.silu_gemv(N, K), [gu, mat, r1, r2, torch.zeros(N, dtype=torch.bfloat16)])[-1]
    _wide_compare(got, O.silu_gemv(gu, mat, r1, r2, K, N), f"silu_gemv N={N} K={K}")


@pytest.mark.parametrize("n,residual", [(4096, False), (4096, True), (1, False), (1000003, True)])
def test_sumsq(n, residual):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, generator=g).to(torch.bfloat16)
    res = torch.randn(n, generator=g).to(torch.bfloat16)
    ins = [x] + ([res] if residual else []) + [torch.zeros(1)]
    got = run(B.sumsq(n, residual), ins)[-1]
    want = O.sumsq(x, n, res if residual else None)
    parity(got, want, FP32_SUM, magnitude=float(want[0]), name=f"sumsq {n} residual={residual}")


def test_fused_vector_load_out_of_range_is_recorded():
    """A prologue load past its tensor records PTSIM_E_OOB."""
    N, K = 64, 256
    desc = B.rmsnorm_gemv(N, K)
    desc.arg_numel[2] = K - 1                 # the weight row holds one element fewer than the program reads
    ts = [torch.randn(K).to(torch.bfloat16), torch.ones(1), torch.randn(K - 1).to(torch.bfloat16),
          torch.randn(K * N).to(torch.bfloat16), torch.zeros(N, dtype=torch.bfloat16)]
    with pytest.raises(native.ExecutorError) as e:
        RC.launch_tensors(D.to_bytes(desc), [t.cuda() for t in ts])
    assert e.value.code == D.E_OOB


@pytest.mark.parametrize("tokens,heads", [(4096, 32), (1, 4), (333, 8)])
def test_rope_rows(tokens, heads):
    """The rotary embedding layer op: the QK kernel with its norm off."""
    from tests.test_oracle_golden import make_inputs
    g = torch.Generator().manual_seed(tokens)
    n = tokens * heads * 128
    x = torch.randn(n, generator=g).to(torch.bfloat16)
    cos, sin = torch.randn(tokens * 128, generator=g), torch.randn(tokens * 128, generator=g)
    desc = B.qknorm_rope(tokens, heads)
    q = desc.p.qk
    q.no_norm, q.out_tok_stride, q.out_head_stride = 1, heads * 128, 128
    ts = [x, torch.zeros(128, dtype=torch.bfloat16), cos, sin, torch.zeros(n, dtype=torch.bfloat16)]
    got = run(desc, ts)[4]
    parity(got, O.rope_rows(x, cos, sin, tokens, heads), POINTWISE, row=128, name=f"rope {tokens}x{heads}")
