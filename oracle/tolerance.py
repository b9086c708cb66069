"""Parity bars of the B200 executor against the oracle.

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's checker import this module; the
product package never does.

The bars follow the north star: bit exact for copies, indices and integer work; bf16 results within 1e-2
relative; fp32 results within 1e-5 (the reference's own fp32 softmax case uses rtol 1e-5, atol 1e-6:
tests/cases/workloads/softmax.py:84).  A relative bar needs an absolute floor for elements at or near zero.
Here that floor is never a fixed number: it is tied to the output's own scale, or absent, by the kind of
computation that produced the element.

  EXACT        bit for bit.
  POINTWISE    bf16 results that the kernel and the oracle each compute from the same fp32 inputs element by
               element or row by row (softmax, RMSNorm, SiLU x mul, QK-norm + RoPE, rotary, divide by the row
               sum).  Both round one fp32 value to bf16 (RNE); they can disagree only where the fp32 values,
               which differ by a few fp32 ulps (ex2 / rsqrt approximations, summation order), straddle a bf16
               rounding boundary.  Bar: |got - want| <= 1e-2 |want| for every element, every element within
               2 bf16 ulps, and at most 1 % of the elements differing at all.  An output moved by one ulp
               everywhere fails the last clause.  There is no absolute floor, except for programs whose
               element is a sum of two products (the rotary embedding: x cos + rot sin), where it is the fp32
               level, 2^-16 of the row's RMS, and the ulp clause skips elements below 2^-8 of it.
  CONTRACTION  bf16 results of sums of products accumulated in fp32 (GEMM, GEMV, grouped GEMM, the MoE
               combine): the kernel accumulates in another order, which moves an element by a few fp32 ulps
               of the row's magnitude.  Bar: |got - want| <= 1e-2 |want| + 2^-10 rms(want over the element's
               row), at most 0.5 % of the elements more than one bf16 ulp away and at most 5 % differing at
               all.  Measured on the B200: at most 2.7e-5 rms, 0.05 % and 0.7 %.
  ATTENTION    bf16 results of attention (prefill and decode), whose P = exp(s - m) is rounded to bf16 before
               P.V.  Where P is rounded depends on the running maximum m, which depends on the key-block
               size, a free choice of the online softmax: the reference's own kernel run with BKV = 128, 256
               or 512 instead of 1024 differs from itself by up to 0.0086 rms per element, 8 % of elements
               more than one ulp and 0.12 % rms error, and the exact (fp64) softmax differs from it by 0.0074,
               12 % and 0.22 % (tests/test_tolerance.py measures both).  The kernel keeps its own maximum
               (128-key tiles, rescaled lazily), so it is held to that same envelope: |got - want| <=
               1e-2 |want| + 2^-5 rms(row), the error's RMS at most 2^-7 of the output's, at most 30 % of
               the elements more than one bf16 ulp away and at most 75 % differing at all.
  FP32         fp32 results: |got - want| <= 1e-5 |want| + 1e-6 max|want|.
  FP32_SUM     fp32 sums whose order differs: |got - want| <= 1e-5 sum|x| (the summands' magnitudes).

check() returns the comparison's statistics (and writes them as a JSON line to $PTSIM_PARITY_LOG when that
is set) and raises AssertionError with the reference's verify-style report (tests/runtime/verify.py:28-69:
max abs / rel error and the worst index) when the bar is missed.
"""
import json
import os

import torch

EXACT, POINTWISE, CONTRACTION, ATTENTION, FP32, FP32_SUM = ("exact", "pointwise", "contraction", "attention", "fp32",
                                                            "fp32_sum")

BF16_RTOL = 1e-2
FP32_RTOL, FP32_ATOL_OF_MAX = 1e-5, 1e-6
POINTWISE_MAX_ULP = 2
POINTWISE_MAX_FRAC_DIFFERENT = 0.01
POINTWISE_SUM_ATOL_OF_ROW_RMS = 2.0 ** -16
POINTWISE_SUM_ULP_FLOOR_OF_ROW_RMS = 2.0 ** -8
# Sums of products: (absolute floor as a fraction of the row's RMS, max fraction more than one ulp away,
# max fraction differing at all, max RMS of the error as a fraction of the output's RMS).
CONTRACTION_BAR = (2.0 ** -10, 0.005, 0.05, None)
ATTENTION_BAR = (2.0 ** -5, 0.30, 0.75, 2.0 ** -7)

# Program families (the kernel objects' case.json "family") and the bar each one's outputs meet.
FAMILY_BAR = {
    "softmax_rows": POINTWISE, "rmsnorm_rows": POINTWISE, "qknorm_rope": POINTWISE, "rope_rows": POINTWISE,
    "silu_mul": POINTWISE, "row_divsum": POINTWISE,
    "gemm": CONTRACTION, "rmsnorm_gemv": CONTRACTION, "silu_gemv": CONTRACTION, "attention_prefill": ATTENTION,
    "attention_decode": ATTENTION, "grouped_gemm": CONTRACTION, "combine_weighted": CONTRACTION,
    "combine_weighted_fused": CONTRACTION,
    "reduce_all": FP32_SUM, "sumsq": FP32_SUM, "row_sum": FP32,
}


def bar_for(family, dtype):
    """The bar of one output of a program family; `dtype` is the output's kernel.json / torch dtype name."""
    dt = str(dtype).replace("torch.", "")
    bar = FAMILY_BAR.get(family, EXACT)
    if bar in (POINTWISE, CONTRACTION, ATTENTION) and dt == "float32":
        return FP32
    return bar


def _ordered(bits, width):
    """Bit patterns mapped to integers that are ordered like the floats they encode (+0 and -0 both 0)."""
    b = bits.to(torch.int64)
    sign = 1 << (width - 1)
    b = torch.where(b < 0, b + (1 << width), b)          # the unsigned pattern
    return torch.where(b >= sign, -(b - sign), b)


def ulp_distance(got, want):
    """How many representable values of got's dtype (bf16 or fp32) lie between got and want, element by
    element; 0 where both are NaN, a huge value where only one is."""
    g, w = got.detach().cpu().contiguous().reshape(-1), want.detach().cpu().contiguous().reshape(-1)
    if g.dtype == torch.bfloat16:
        w = w.to(torch.bfloat16)
        d = (_ordered(g.view(torch.int16), 16) - _ordered(w.view(torch.int16), 16)).abs()
    else:
        g, w = g.float(), w.float()
        d = (_ordered(g.view(torch.int32), 32) - _ordered(w.view(torch.int32), 32)).abs()
    gn, wn = torch.isnan(g.float()), torch.isnan(w.float())
    d = torch.where(gn & wn, torch.zeros_like(d), d)
    return torch.where(gn ^ wn, torch.full_like(d, 1 << 40), d)


def _report(g, w, diff, what):
    i = int(diff.argmax()) if diff.numel() else 0
    rel = diff / w.abs().clamp_min(1e-30)
    return (f"{what}: max_abs_err={float(diff.max()) if diff.numel() else 0:.6g} "
            f"max_rel_err={float(rel.max()) if rel.numel() else 0:.6g} worst@{i}: "
            f"got={float(g[i]) if g.numel() else 0!r} want={float(w[i]) if w.numel() else 0!r}")


def check(got, want, bar, *, row=None, magnitude=None, name=""):
    """Compare a CUDA result with the oracle's under `bar`.  `row`: elements per row of the output, the unit
    of the row scale (CONTRACTION / ATTENTION: default the whole output; POINTWISE: only for outputs that are
    sums of two products, which then get the fp32-level floor).  `magnitude`: sum |x| of the summands, for
    FP32_SUM."""
    g_raw = got.detach().cpu().contiguous().reshape(-1)
    w_raw = want.detach().cpu().contiguous().reshape(-1)
    stats = {"name": name, "bar": bar, "numel": int(g_raw.numel())}
    if g_raw.numel() != w_raw.numel():
        raise AssertionError(f"{name}: {g_raw.numel()} elements, the oracle has {w_raw.numel()}")
    if bar == EXACT:
        a = g_raw.view(torch.uint8) if g_raw.dtype != torch.bool else g_raw
        b = w_raw.to(g_raw.dtype)
        b = b.view(torch.uint8) if b.dtype != torch.bool else b
        ok = bool(torch.equal(a, b))
        stats["ok"] = ok
        _log(stats)
        if not ok:
            n = int((a != b).sum()) if a.shape == b.shape else -1
            raise AssertionError(f"{name}: not bit exact ({n} differing bytes)")
        return stats
    g, w = g_raw.float(), w_raw.float()
    nan_g, nan_w = torch.isnan(g), torch.isnan(w)
    if not torch.equal(nan_g, nan_w):
        raise AssertionError(f"{name}: NaN in {int((nan_g ^ nan_w).sum())} positions of only one side")
    keep = ~nan_g
    diff = torch.where(keep, (g - w).abs(), torch.zeros_like(g))
    inf_mismatch = torch.isinf(g) | torch.isinf(w)
    inf_ok = torch.where(inf_mismatch, g == w, torch.ones_like(keep))
    if not bool(inf_ok.all()):
        raise AssertionError(f"{name}: infinities differ")
    diff = torch.where(inf_mismatch, torch.zeros_like(diff), diff)
    wa = torch.where(keep & ~inf_mismatch, w.abs(), torch.zeros_like(w))
    msg = []
    if bar == FP32_SUM:
        if magnitude is None:
            raise ValueError("FP32_SUM needs the summands' magnitude")
        bound = FP32_RTOL * float(magnitude)
        stats["need_over_magnitude"] = float(diff.max()) / max(float(magnitude), 1e-30)
        if float(diff.max()) > bound:
            msg.append(f"|got - want| > 1e-5 sum|x| = {bound:.6g}")
    elif bar == FP32:
        atol = FP32_ATOL_OF_MAX * float(wa.max()) if wa.numel() else 0.0
        excess = diff - FP32_RTOL * wa
        stats["need_atol_over_max"] = float(excess.max()) / max(float(wa.max()), 1e-30)
        stats["max_rel"] = float((diff / wa.clamp_min(1e-30)).max())
        if bool((excess > atol).any()):
            msg.append(f"{int((excess > atol).sum())} elements beyond rtol 1e-5 + 1e-6 max|want|")
    elif bar == POINTWISE:
        u = ulp_distance(g_raw, w_raw)
        frac = float((u > 0).float().mean()) if u.numel() else 0.0
        excess = diff - BF16_RTOL * wa
        if row:
            scale = _row_rms(wa, row, name)
            excess = excess - POINTWISE_SUM_ATOL_OF_ROW_RMS * scale
            u = torch.where(wa >= POINTWISE_SUM_ULP_FLOOR_OF_ROW_RMS * scale, u, torch.zeros_like(u))
        stats.update(ulp_max=int(u.max()) if u.numel() else 0, frac_different=frac,
                     frac_over_one_ulp=float((u > 1).float().mean()) if u.numel() else 0.0)
        if bool((excess > 0).any()):
            msg.append(f"{int((excess > 0).sum())} elements beyond rtol 1e-2"
                       + (" + 2^-16 rms(row)" if row else " (no absolute floor)"))
        if stats["ulp_max"] > POINTWISE_MAX_ULP:
            msg.append(f"an element {stats['ulp_max']} bf16 ulps away (bar: {POINTWISE_MAX_ULP})")
        if frac > POINTWISE_MAX_FRAC_DIFFERENT:
            msg.append(f"{100 * frac:.3g}% of elements differ (bar: {100 * POINTWISE_MAX_FRAC_DIFFERENT:g}%)")
    elif bar in (CONTRACTION, ATTENTION):
        floor, max_over_one, max_different, max_rms_err = CONTRACTION_BAR if bar == CONTRACTION else ATTENTION_BAR
        rms = _row_rms(wa, row or w.numel(), name)
        excess = diff - BF16_RTOL * wa
        need = (excess / rms.clamp_min(1e-30)).max() if excess.numel() else torch.tensor(0.0)
        u = ulp_distance(g_raw, w_raw)
        frac1 = float((u > 1).float().mean()) if u.numel() else 0.0
        frac0 = float((u > 0).float().mean()) if u.numel() else 0.0
        out_rms = float(wa.pow(2).mean().sqrt()) if wa.numel() else 0.0
        rms_err = float(diff.pow(2).mean().sqrt()) / max(out_rms, 1e-30) if diff.numel() else 0.0
        stats.update(need_atol_over_row_rms=float(need), frac_over_one_ulp=frac1, frac_different=frac0,
                     rel_rms_err=rms_err)
        bad = excess > floor * rms
        if bool(bad.any()):
            msg.append(f"{int(bad.sum())} elements beyond rtol 1e-2 + {floor:g} rms(row)")
        if frac1 > max_over_one:
            msg.append(f"{100 * frac1:.3g}% of elements more than one bf16 ulp away (bar: {100 * max_over_one:g}%)")
        if frac0 > max_different:
            msg.append(f"{100 * frac0:.3g}% of elements differ (bar: {100 * max_different:g}%)")
        if max_rms_err is not None and rms_err > max_rms_err:
            msg.append(f"error RMS {rms_err:.3g} of the output's (bar: {max_rms_err:g})")
    else:
        raise ValueError(f"unknown bar {bar!r}")
    stats["ok"] = not msg
    _log(stats)
    if msg:
        raise AssertionError(_report(g, w, diff, name or bar) + "; " + "; ".join(msg))
    return stats


def _row_rms(wa, row, name):
    """The RMS of |want| over each element's row, one value per element."""
    if wa.numel() % row:
        raise ValueError(f"{name}: {wa.numel()} elements are not whole rows of {row}")
    return wa.view(-1, row).pow(2).mean(dim=1, keepdim=True).sqrt().expand(-1, row).reshape(-1)


def _log(stats):
    path = os.environ.get("PTSIM_PARITY_LOG")
    if path:
        with open(path, "a") as fh:
            fh.write(json.dumps(stats) + "\n")
