"""The parity bars catch what they must (CPU only).  Each case plants a mistake in an oracle output and checks
that oracle/tolerance.py rejects it, and that an honest result (the same computation in another order or
with the GPU's rounding) passes.  The headline softmax is the case the bars were written for: its outputs
are of order 1e-4, so a fixed absolute floor of 1e-2 (or even 1e-4) accepts nearly any answer."""
import math

import pytest
import torch

from oracle import programs as O
from oracle import tolerance as T


def _softmax_case(rows=64, cols=4096, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows * cols, generator=g).to(torch.bfloat16)
    return x, O.softmax_rows(x, rows, cols)


def _step(t, ulps):
    """t moved by `ulps` bf16 steps away from zero, element by element."""
    b = t.contiguous().view(torch.int16)
    return (b + ulps).view(torch.bfloat16)


def test_softmax_one_ulp_everywhere_is_caught():
    _, want = _softmax_case()
    bad = _step(want, 1)
    # The round-1 bar would have taken it: every element is within rtol 1e-2.
    assert torch.allclose(bad.float(), want.float(), rtol=1e-2, atol=1e-2)
    with pytest.raises(AssertionError, match="differ"):
        T.check(bad, want, T.POINTWISE, name="softmax one ulp")


def test_softmax_small_elements_wrong_are_caught():
    _, want = _softmax_case()
    w = want.float()
    bad = torch.where(w < w.median(), w * 2, w).to(torch.bfloat16)     # half the outputs 100 % wrong
    assert torch.allclose(bad.float(), w, rtol=1e-2, atol=1e-2)        # what the old bar let through
    with pytest.raises(AssertionError):
        T.check(bad, want, T.POINTWISE)


def test_softmax_honest_recomputation_passes():
    """The same softmax in fp64 then rounded to bf16 (another summation order, exact exp) meets the bar."""
    x, want = _softmax_case()
    other = torch.softmax(x.double().view(64, 4096), dim=1).reshape(-1).to(torch.bfloat16)
    st = T.check(other, want, T.POINTWISE)
    assert st["ulp_max"] <= 1 and st["frac_different"] < 0.01


def test_fp32_router_softmax_held_to_1e5():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(128 * 128, generator=g).to(torch.bfloat16)
    want = O.softmax_rows(x, 128, 128, torch.float32)
    T.check(want.double().view(128, 128).float().reshape(-1), want, T.FP32)
    with pytest.raises(AssertionError, match="1e-5"):
        T.check(want * (1 + 1e-4), want, T.FP32)                        # bf16-sized error in an fp32 output


def _gemm_case(M=64, N=256, K=4096, seed=2):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M * K, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    b = (torch.randn(K * N, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    return a, b, O.gemm(a, b, M, N, K)


def test_gemm_bars():
    M, N, K = 64, 256, 4096
    a, b, want = _gemm_case(M, N, K)
    # Another accumulation order (fp64) rounded to bf16 passes.
    other = (a.double().view(M, K) @ b.double().view(K, N)).reshape(-1).to(torch.bfloat16)
    T.check(other, want, T.CONTRACTION, row=N)
    # 2 % off everywhere fails.
    with pytest.raises(AssertionError):
        T.check((want.float() * 1.02).to(torch.bfloat16), want, T.CONTRACTION, row=N)
    # A near-zero element off by 0.3 % of its row's RMS fails (the floor is 2^-10 = 0.1 % of it).
    w = want.float().view(M, N).clone()
    i = int(w[3].abs().argmin())
    w[3, i] += 0.003 * float(w[3].pow(2).mean().sqrt())
    with pytest.raises(AssertionError, match="rms"):
        T.check(w.reshape(-1).to(torch.bfloat16), want, T.CONTRACTION, row=N)
    # Two ulps on 2 % of the elements fails the ulp-fraction clause; one ulp everywhere fails the
    # differing-fraction clause.
    bad = want.clone()
    bad[::50] = _step(bad[::50], 2)
    with pytest.raises(AssertionError, match="ulp"):
        T.check(bad, want, T.CONTRACTION, row=N)
    with pytest.raises(AssertionError, match="differ"):
        T.check(_step(want, 1), want, T.CONTRACTION, row=N)


def _attention_case(S=1024, H=4, G=4, D=128, seed=3):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(H * S * D, generator=g).to(torch.bfloat16)
    k, v = (torch.randn(H // G * S * D, generator=g).to(torch.bfloat16) for _ in range(2))
    return q, k, v, (1, H, G, S, D)


def test_attention_bar_is_the_references_own_envelope():
    """The reference kernel (BQ = BKV = 1024) against itself at other legal key-block sizes, and against the
    exact fp64 softmax: every one meets the ATTENTION bar, which is where the bar's numbers come from."""
    q, k, v, (B, H, G, S, D) = _attention_case()
    sc = 1 / math.sqrt(D)
    ref = O.attention_prefill(q, k, v, B, H, G, S, D, 1024, 1024, True, sc)
    for bkv in (128, 256, 512):
        st = T.check(O.attention_prefill(q, k, v, B, H, G, S, D, bkv, bkv, True, sc), ref, T.ATTENTION, row=D)
        assert st["frac_different"] > 0.05        # the block size alone moves many elements
    Q = q.double().view(H, S, D)
    K = k.double().view(H // G, S, D).repeat_interleave(G, 0)
    V = v.double().view(H // G, S, D).repeat_interleave(G, 0)
    s = (Q @ K.transpose(1, 2) * sc).masked_fill(~torch.ones(S, S, dtype=torch.bool).tril(), -1e300)
    exact = (torch.softmax(s, -1) @ V).reshape(-1).to(torch.bfloat16)
    T.check(exact, ref, T.ATTENTION, row=D)


def test_attention_bar_catches_errors():
    q, k, v, (B, H, G, S, D) = _attention_case(S=256, H=2, G=1)
    want = O.attention_prefill(q, k, v, B, H, G, S, D, 128, 128, True, 1 / math.sqrt(D))
    # 2 % everywhere: the error RMS clause.
    with pytest.raises(AssertionError, match="RMS"):
        T.check((want.float() * 1.02).to(torch.bfloat16), want, T.ATTENTION, row=D)
    # One ulp everywhere: the differing-fraction clause.
    with pytest.raises(AssertionError, match="differ"):
        T.check(_step(want, 1), want, T.ATTENTION, row=D)
    # One late query row off by 10 % of its own (small) scale: the per-row floor, which the old fixed
    # atol = 1e-2 let through.
    w = want.float().view(-1, D).clone()
    last = w.shape[0] - 1
    w[last] += 0.1 * float(w[last].pow(2).mean().sqrt())
    w0 = w.reshape(-1).to(torch.bfloat16)
    assert torch.allclose(w0.float(), want.float(), rtol=1e-2, atol=1e-2)
    with pytest.raises(AssertionError, match="rms"):
        T.check(w0, want, T.ATTENTION, row=D)


def test_rotary_sum_floor():
    """x cos + rot sin cancels to near zero for some elements; the fp32-level floor (2^-16 of the row's RMS)
    admits the fp32 noise there and nothing more."""
    tokens, heads = 64, 4
    g = torch.Generator().manual_seed(5)
    x = torch.randn(tokens * heads * 128, generator=g).to(torch.bfloat16)
    cos, sin = O.rope_tables(tokens)
    want = O.rope_rows(x, cos, sin, tokens, heads)
    # The same sum with each product rounded separately in fp64 (another fp32 evaluation order) passes.
    v = x.double().view(tokens, heads, 128)
    rot = torch.cat([-v[..., 64:], v[..., :64]], dim=2)
    other = (v * cos.double().view(tokens, 1, 128) + rot * sin.double().view(tokens, 1, 128)).reshape(-1)
    T.check(other.to(torch.bfloat16), want, T.POINTWISE, row=128)
    with pytest.raises(AssertionError):
        T.check(_step(want, 1), want, T.POINTWISE, row=128)


def test_exact_and_nan():
    x = torch.arange(100, dtype=torch.int64)
    T.check(x.clone(), x, T.EXACT)
    y = x.clone()
    y[7] += 1
    with pytest.raises(AssertionError, match="bit exact"):
        T.check(y, x, T.EXACT)
    f = torch.randn(64).to(torch.bfloat16)
    f[3] = float("nan")
    T.check(f.clone(), f, T.POINTWISE)
    h = f.clone()
    h[5] = float("nan")
    with pytest.raises(AssertionError, match="NaN"):
        T.check(h, f, T.POINTWISE)


def test_fp32_sum_bar():
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1 << 20, generator=g)
    want = x.sum().reshape(1)
    mag = float(x.abs().sum())
    T.check(x.double().sum().float().reshape(1), want, T.FP32_SUM, magnitude=mag)
    with pytest.raises(AssertionError):
        T.check(want + 1e-4 * mag, want, T.FP32_SUM, magnitude=mag)
