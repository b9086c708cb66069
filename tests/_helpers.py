"""Shared helpers of the parity tests: seeded inputs with the reference's conventions, and the parity
assertion (oracle/tolerance.py), whose failure report follows the reference's verify stage
(tests/runtime/verify.py:28-69 in the reference: max abs / rel error and the worst index)."""
import torch

from oracle import tolerance as T


def randn(numel, seed, dtype=torch.bfloat16, std=1.0, mean=0.0, gen=None):
    g = gen or torch.Generator().manual_seed(seed)
    t = torch.randn(numel, generator=g) * std + mean
    return t.to(dtype)


def make_inputs(args, seed=0):
    """Inputs as the bundle specs' make_inputs build them: one torch.Generator seeded once, randn of each
    read argument's numel in argument order, cast to its dtype; written arguments zero-filled."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for name, role, dtype, numel in args:
        dt = getattr(torch, dtype)
        if role in ("in", "inout"):
            out.append(torch.randn(numel, generator=g).to(dt))
        else:
            out.append(torch.zeros(numel, dtype=dt))
    return out


def parity(got, want, bar, row=None, name="", magnitude=None):
    """Assert that a CUDA result meets its parity bar against the oracle (oracle/tolerance.py: EXACT,
    POINTWISE, CONTRACTION, FP32, FP32_SUM); returns the comparison's statistics."""
    return T.check(got, want, bar, row=row, name=name, magnitude=magnitude)


def bits_equal(got, want):
    a, b = got.detach().cpu().contiguous(), want.detach().cpu().contiguous()
    if a.dtype != b.dtype or a.shape != b.shape:
        return False
    return bool(torch.equal(a.view(torch.uint8), b.view(torch.uint8)))
