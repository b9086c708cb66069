"""The oracle is pinned: each restatement in oracle/programs.py reproduces the outputs of the reference's own
kernel (its Triton source run by the Triton interpreter, tests/golden/make_golden.py) on the reference's
seeded inputs (make_inputs(torch, seed=0)).  Bit exact where the program is exact (copies, fp32 adds, bf16
+ 1, max, integer tables); otherwise under the parity bars of oracle/tolerance.py (bf16: 1e-2 relative with
no absolute floor and at most 2 ulps for element- and row-wise programs, plus 2^-10 of the row's RMS for
sums of products, the ATTENTION envelope for attention; fp32: 1e-5).  CPU only."""
import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import programs as O
from oracle import tolerance as T

HERE = os.path.dirname(os.path.abspath(__file__))
OBJ = os.path.join(HERE, "golden", "objects")


def golden_cases():
    with open(os.path.join(HERE, "golden", "index.json")) as fh:
        names = json.load(fh)
    out = []
    for n in names:
        with open(os.path.join(OBJ, n, "case.json")) as fh:
            c = json.load(fh)
        if c["golden"]:
            out.append(c)
    return out


def make_inputs(case):
    """The reference's input convention (validation/pytorchsim/*/..._spec.py make_inputs): one generator
    seeded 0, randn(numel) per read argument in argument order, cast to the argument's dtype.  Arguments a
    spec loads from a recording (the MoE dispatch's routing indices) come from the committed fixture and
    draw nothing."""
    g = torch.Generator().manual_seed(0)
    rec = case.get("recorded") or {}
    saved = np.load(os.path.join(HERE, "golden", rec["file"])) if rec else {}
    out = {}
    for a in case["args"]:
        dt = getattr(torch, a["dtype"])
        if a["name"] in rec.get("args", ()):
            out[a["name"]] = torch.from_numpy(saved[a["name"]].copy()).to(dt).reshape(-1)
        elif a["role"] in ("in", "inout"):
            out[a["name"]] = torch.randn(a["numel"], generator=g).to(dt)
        else:
            out[a["name"]] = torch.zeros(a["numel"], dtype=dt)
    return out


def run_oracle(case, ins):
    """(output argument name, oracle output) of the case's program family."""
    o = dict(case["oracle"])
    fam = o.pop("family")
    args = case["args"]
    reads = [a["name"] for a in args if a["role"] in ("in", "inout")]
    outs = [a["name"] for a in args if a["role"] in ("out", "inout")]
    x = [ins[n] for n in reads]
    if fam == "vector_add":
        return outs[0], O.vector_add(x[0], x[1])
    if fam == "add_one":
        return outs[0], O.add_one(x[0])
    if fam == "slice_add_one":
        return outs[0], O.slice_add_one(x[0])
    if fam == "reduce_all":
        return outs[0], O.reduce_all(x[0], o["op"])
    if fam == "softmax_rows":
        return outs[0], O.softmax_rows(x[0], o["rows"], o["cols"], getattr(torch, o.get("out_dtype", "bfloat16")))
    if fam == "combine_weighted":
        return outs[0], O.combine_weighted(x[0], x[1], x[2], x[3], x[4], x[5], o["tokens"], o["hidden"], o["topk"],
                                           o["experts"])
    if fam == "grouped_gemm":
        return outs[0], O.grouped_gemm(x[0], x[1], x[2], x[3], x[4], x[5], o["M"], o["N"], o["K"], o["groups"])
    if fam == "cumsum_int":
        dt = next(getattr(torch, a["dtype"]) for a in args if a["name"] == outs[0])
        return outs[0], O.cumsum_int(x[0], o["n"], dt)
    if fam == "slot_of":
        return outs[0], O.slot_of(x[0], x[1], o["n"], o["experts"])
    if fam == "count_le":
        dt = next(getattr(torch, a["dtype"]) for a in args if a["name"] == outs[0])
        return outs[0], O.count_le(x[0], o["n"], o["rows"], dt)
    if fam == "sumsq":
        return outs[0], O.sumsq(x[0], o["n"], x[1] if len(x) > 1 else None)
    if fam == "rmsnorm_gemv":
        if o.get("residual"):
            return outs[0], O.rmsnorm_gemv(x[0], x[2], x[3], x[4], o["K"], o["N"], o["eps"], res=x[1])
        return outs[0], O.rmsnorm_gemv(x[0], x[1], x[2], x[3], o["K"], o["N"], o["eps"])
    if fam == "silu_gemv":
        return outs[0], O.silu_gemv(x[1], x[2], x[3], x[4], o["K"], o["N"])
    if fam == "row_divsum":
        return outs[0], O.row_divsum(x[0], o["rows"], o["cols"])
    if fam == "dispatch_gather":
        return outs[0], O.dispatch_gather(x[0], x[1], o["tokens"], o["hidden"], o["topk"])
    if fam == "rmsnorm_rows":
        if o.get("residual"):
            return outs[0], O.rmsnorm_rows(x[0], x[2], o["rows"], o["cols"], o["eps"], res=x[1])
        return outs[0], O.rmsnorm_rows(x[0], x[1], o["rows"], o["cols"], o["eps"])
    if fam == "row_sum":
        return outs[0], O.row_sum(x[0], o["rows"], o["cols"])
    if fam == "rope_rows":
        return outs[0], O.rope_rows(x[0], x[1], x[2], o["tokens"], o["heads"])
    if fam == "combine_weighted_fused":
        return outs[0], O.combine_weighted_fused(x[1], x[2], x[3], x[4], x[5], x[6], x[7], x[8], x[0], o["tokens"],
                                                 o["hidden"], o["topk"], o["experts"])
    if fam == "qknorm_rope":
        q = x[1:] if o.get("inout_first") else x    # the decode program's output row comes first, unread
        return outs[0], O.qknorm_rope(q[0], q[1], q[2], q[3], o["tokens"], o["heads"], o["eps"])
    if fam == "token_to_head_major":
        return outs[0], O.token_to_head_major(x[0], o["tokens"], o["heads"], o["dim"])
    if fam == "heads_to_token_major":
        return outs[0], O.heads_to_token_major(x[0], o["tokens"], o["heads"], o["dim"])
    if fam == "silu_mul":
        return outs[0], O.silu_mul(x[0], o["tokens"], o["inter"])
    if fam == "gemm":
        if o["residual"]:
            return outs[0], O.gemm(x[1], x[2], o["M"], o["N"], o["K"], residual=x[0])
        return outs[0], O.gemm(x[0], x[1], o["M"], o["N"], o["K"])
    if fam == "attention_decode":
        return outs[0], O.attention_decode(x[0], x[1], x[2], x[3], o["hkv"], o["g"], o["gp"], o["seq"], o["dim"],
                                           o["bkv"], o["scale"])
    if fam == "attention_prefill":
        bq = case.get("ref_bq") or min(1024, o["seq"])
        return outs[0], O.attention_prefill(x[0], x[1], x[2], o["batch"], o["hq"], o["g"], o["seq"], o["dim"],
                                            bq, bq, o["causal"], o["scale"])
    raise AssertionError(f"no oracle family {fam}")


EXACT = {"vector_add", "add_one", "slice_add_one", "token_to_head_major", "heads_to_token_major", "topk", "sort",
         "dispatch_gather", "expert_counts", "cumsum_int", "slot_of", "group_tables", "count_le"}


def run_oracle_all(case, ins):
    """{output argument name: oracle output} of the case's program family (several for top-k and sort)."""
    o = dict(case["oracle"])
    fam = o.pop("family")
    outs = [a["name"] for a in case["args"] if a["role"] in ("out", "inout")]
    x = [ins[a["name"]] for a in case["args"] if a["role"] in ("in", "inout")]
    if fam == "topk":
        v, i = O.topk_rows(x[0], o["rows"], o["cols"], o["cols_padded"], o["k"], o["largest"])
        return {outs[0]: v, outs[1]: i}
    if fam == "sort":
        v, i = O.sort_rows(x[0], o["rows"], o["cols"], o["descending"], o["float_keys"])
        return {outs[0]: v, outs[1]: i}
    if fam == "expert_counts":
        cnt, run = O.expert_counts(x[0], o["experts"], o["n"])
        return {outs[0]: cnt, outs[1]: run}
    if fam == "group_tables":
        nonempty, prev, count = O.group_tables(x[0], o["n"])
        return {outs[0]: nonempty, outs[1]: prev, outs[2]: count}
    name, got = run_oracle(case, ins)
    return {name: got}


def as_bits(t):
    t = t.contiguous()
    return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def as_float(bits, dtype):
    if dtype == "bfloat16":
        return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16).float()
    return torch.from_numpy(bits).float()


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_kernel(case):
    ins = make_inputs(case)
    for name, got in run_oracle_all(case, ins).items():
        _check_against_gold(case, ins, name, got)


def row_of(case):
    """Elements per row of a contraction family's output (the CONTRACTION bar's scale), or None (one row)."""
    o = case["oracle"]
    fam = o["family"]
    if fam in ("gemm", "grouped_gemm"):
        return o["N"]
    if fam in ("attention_prefill", "attention_decode"):
        return o["dim"]
    if fam in ("combine_weighted", "combine_weighted_fused"):
        return o["hidden"]
    if fam in ("qknorm_rope", "rope_rows"):      # x cos + rot sin: the POINTWISE bar's fp32-level floor
        return o.get("dim", 128)
    return None


def bar_of(case, name):
    """The parity bar (oracle/tolerance.py) of output `name` of a case."""
    o = case["oracle"]
    if o["family"] in EXACT or (o["family"] == "reduce_all" and o["op"] == "max"):
        return T.EXACT
    dt = next(a["dtype"] for a in case["args"] if a["name"] == name)
    return T.bar_for(o["family"], dt)


def magnitude_of(case, ins, want):
    """Sum of the summands' magnitudes of an FP32_SUM output: sum |x| of a whole-tensor sum; a sum of
    squares is its own magnitude."""
    if case["oracle"]["family"] == "reduce_all":
        return float(ins[case["inputs"][0]].float().abs().sum())
    return float(want.float().abs().sum())


def _check_against_gold(case, ins, name, got):
    gold = np.load(os.path.join(HERE, "golden", case["golden"]))
    stride = int(gold[f"{name}__stride"][0])
    want_bits = gold[name]
    dt = next(a["dtype"] for a in case["args"] if a["name"] == name)
    got_bits = as_bits(got.reshape(-1))
    bar = bar_of(case, name)
    if bar == T.EXACT:
        # Exact programs: the whole output's hash matches, not only the sample.
        import hashlib
        assert hashlib.sha256(got_bits.tobytes()).digest() == bytes(gold[f"{name}__sha256"]), case["name"]
        return
    g = as_float(got_bits[::stride], dt)
    w = as_float(want_bits, dt)
    if dt == "bfloat16":
        g, w = g.to(torch.bfloat16), w.to(torch.bfloat16)
    T.check(g, w, bar, row=row_of(case) if stride == 1 else None,
            magnitude=magnitude_of(case, ins, w) if bar == T.FP32_SUM else None, name=case["name"])
