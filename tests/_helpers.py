"""Shared helpers of the parity tests: seeded inputs with the reference's conventions and the comparison
report of its verify stage (tests/runtime/verify.py:28-69 in the reference: allclose, max abs/rel error)."""
import torch


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


def compare(got, want, rtol, atol):
    """(ok, report) of a CUDA result against the oracle: torch.allclose plus the reference's error report."""
    g, w = got.detach().float().cpu(), want.detach().float().cpu()
    ok = torch.allclose(g, w, rtol=rtol, atol=atol, equal_nan=True)
    diff = (g - w).abs()
    diff = torch.where(torch.isnan(g) & torch.isnan(w), torch.zeros_like(diff), diff)
    rel = diff / w.abs().clamp_min(1e-12)
    i = int(diff.argmax()) if diff.numel() else 0
    rep = (f"max_abs_err={float(diff.max()) if diff.numel() else 0:.6g} max_rel_err={float(rel.max()) if rel.numel() else 0:.6g}"
           f" worst@{i}: got={float(g.reshape(-1)[i]) if g.numel() else 0!r} want={float(w.reshape(-1)[i]) if w.numel() else 0!r}")
    return ok, rep


def bits_equal(got, want):
    a, b = got.detach().cpu().contiguous(), want.detach().cpu().contiguous()
    if a.dtype != b.dtype or a.shape != b.shape:
        return False
    return bool(torch.equal(a.view(torch.uint8), b.view(torch.uint8)))
