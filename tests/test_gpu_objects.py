"""The reference's own validation programs, run end to end on the B200: each committed kernel object
(tests/golden/objects/, lowered from the reference's kernel source by tests/golden/make_golden.py) goes
through the launch-from-files API (runtime/cuda.py launch: .raw in, .raw out, the reference's spike.launch
shape) on inputs built by the reference's make_inputs convention, and its output is compared with
  - the Triton-interpreter output vectors of the reference's kernel (small cases), and
  - the CPU oracle (every case; for the batch-4 attention, on a subset of heads).
Bit exact for copies, fp32 adds, bf16 + 1 and max; rtol = atol = 1e-2 for bf16 results; fp32 sums within
1e-5 of the sum of magnitudes."""
import hashlib
import json
import math
import os
import tempfile

import numpy as np
import pytest
import torch

from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.runtime import cuda as RC
from tests.test_oracle_golden import EXACT, as_bits, as_float, make_inputs, run_oracle_all

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
OBJ = os.path.join(HERE, "golden", "objects")


def all_cases():
    with open(os.path.join(HERE, "golden", "index.json")) as fh:
        names = json.load(fh)
    return [json.load(open(os.path.join(OBJ, n, "case.json"))) for n in names]


def run_object(case, ins):
    """Write the inputs as .raw files, launch the kernel object from files, read the outputs back."""
    d = os.path.join(OBJ, case["name"])
    m = ko.read(d)
    blob = ko.read_desc(d, m)
    with tempfile.TemporaryDirectory() as rt:
        raw = {}
        for a in m["args"]:
            p = os.path.join(rt, f"{a['name']}.raw")
            t = ins[a["name"]].contiguous()
            (t.view(torch.int16) if t.dtype == torch.bfloat16 else t).numpy().tofile(p)
            raw[a["name"]] = p
        RC.launch(blob, m, rt, raw, log=lambda *_: None, devices=[0])
        out = {}
        for a in m["args"]:
            if a["role"] in ("out", "inout"):
                arr = np.fromfile(raw[a["name"]], dtype=np.dtype(ko.NP_DTYPE[a["dtype"]]))
                t = torch.from_numpy(arr.copy())
                out[a["name"]] = t.view(torch.bfloat16) if a["dtype"] == "bfloat16" else t
        return out


def attention_subset(case, ins, got, heads=(0, 5, 17, 31)):
    """Oracle check of a large attention case on a subset of (batch, query head) pairs."""
    o = case["oracle"]
    B, HQ, G, S, Dh = o["batch"], o["hq"], o["g"], o["seq"], o["dim"]
    q = ins["q_ptr"].view(B, HQ, S, Dh)
    k = ins["k_ptr"].view(B, HQ // G, S, Dh)
    v = ins["v_ptr"].view(B, HQ // G, S, Dh)
    out = got.view(B, HQ, S, Dh)
    for b in range(B):
        for h in heads:
            want = __import__("oracle.programs", fromlist=["x"]).attention_prefill(
                q[b, h].reshape(-1), k[b, h // G].reshape(-1), v[b, h // G].reshape(-1), 1, 1, 1, S, Dh,
                min(1024, S), min(1024, S), o["causal"], o["scale"])
            ok = torch.allclose(out[b, h].float().reshape(-1), want.float(), rtol=1e-2, atol=1e-2)
            assert ok, f"{case['name']} b={b} h={h}: {float((out[b, h].float().reshape(-1) - want.float()).abs().max())}"


@pytest.mark.parametrize("case", all_cases(), ids=lambda c: c["name"])
def test_reference_program_on_b200(case):
    ins = make_inputs(case)
    got_all = run_object(case, ins)
    fam = case["oracle"]["family"]
    if fam == "attention_prefill" and case["oracle"]["batch"] * case["oracle"]["hq"] * case["oracle"]["seq"] > 32 * 2048:
        name = [a["name"] for a in case["args"] if a["role"] in ("out", "inout")][0]
        _check_golden(case, ins, name, got_all[name])
        attention_subset(case, ins, got_all[name])
        return
    for name, want in run_oracle_all(case, ins).items():
        _check_golden(case, ins, name, got_all[name])
        _check_oracle(case, ins, name, got_all[name], want)


def _check_golden(case, ins, name, got):
    fam = case["oracle"]["family"]
    dt = next(a["dtype"] for a in case["args"] if a["name"] == name)
    # 1. The reference kernel's own output (Triton interpreter), where recorded.
    if case["golden"]:
        gold = np.load(os.path.join(HERE, "golden", case["golden"]))
        stride = int(gold[f"{name}__stride"][0])
        gb = as_bits(got.reshape(-1))
        if fam in EXACT or (fam == "reduce_all" and case["oracle"]["op"] == "max"):
            assert hashlib.sha256(gb.tobytes()).digest() == bytes(gold[f"{name}__sha256"]), "differs from the reference kernel"
        elif fam == "reduce_all":
            scale = float(ins[case["inputs"][0]].float().abs().sum())
            assert abs(float(as_float(gb, dt)[0]) - float(as_float(gold[name], dt)[0])) <= 1e-5 * scale
        else:
            g, w = as_float(gb[::stride], dt), as_float(gold[name], dt)
            assert torch.allclose(g, w, rtol=1e-2, atol=1e-2), f"max abs err vs reference kernel {float((g - w).abs().max())}"


def _check_oracle(case, ins, name, got, want):
    fam = case["oracle"]["family"]
    if fam in EXACT or (fam == "reduce_all" and case["oracle"]["op"] == "max"):
        assert torch.equal(got.reshape(-1).view(torch.uint8) if got.dtype != torch.bool else got,
                           want.reshape(-1).to(got.dtype).view(torch.uint8)), "differs from the oracle"
    elif fam == "reduce_all":
        scale = float(ins[case["inputs"][0]].float().abs().sum())
        assert abs(float(got.float()[0]) - float(want.float()[0])) <= 1e-5 * scale
    elif fam == "sumsq":
        assert abs(float(got.float()[0]) - float(want.float()[0])) <= 1e-5 * abs(float(want.float()[0]))
    else:
        g, w = got.float().reshape(-1), want.float().reshape(-1)
        wide = fam in ("gemm", "rmsnorm_gemv", "silu_gemv")   # sums of K products: atol scales with the output
        atol = 1e-2 if not wide else 1e-2 * max(1.0, float(w.pow(2).mean().sqrt()))
        assert torch.allclose(g, w, rtol=1e-2, atol=atol), f"max abs err vs oracle {float((g - w).abs().max())}"
