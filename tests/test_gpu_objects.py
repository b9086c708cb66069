"""The reference's own validation programs, run end to end on the B200: each committed kernel object
(tests/golden/objects/, lowered from the reference's kernel source by tests/golden/make_golden.py) goes
through the launch-from-files API (runtime/cuda.py launch: .raw in, .raw out, the reference's spike.launch
shape) on inputs built by the reference's make_inputs convention, and its output is compared with
  - the Triton-interpreter output vectors of the reference's kernel (small cases), and
  - the CPU oracle (every case, every output element; the batch-4 attention one batch at a time).
Bit exact for copies, fp32 adds, bf16 + 1, max and integer tables; otherwise the parity bars of
oracle/tolerance.py: bf16 within 1e-2 relative (element- and row-wise programs with no absolute floor and at
most 2 ulps; sums of products with a floor of 2^-10 of the row's RMS; attention within the reference's
own block-size envelope), fp32 within 1e-5, fp32 sums within 1e-5 of the summands' magnitudes."""
import hashlib
import json
import os
import tempfile

import numpy as np
import pytest
import torch

from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.runtime import cuda as RC
from oracle import programs as O
from oracle import tolerance as T
from tests.test_oracle_golden import (as_bits, as_float, bar_of, magnitude_of, make_inputs, row_of,
                                      run_oracle_all)

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


def attention_all_heads(case, ins, got):
    """Oracle check of a large attention case on every (batch, query head) pair, one batch at a time (the
    oracle is vectorised over heads), each query row against the ATTENTION bar."""
    o = case["oracle"]
    B, HQ, G, S, Dh = o["batch"], o["hq"], o["g"], o["seq"], o["dim"]
    hkv = HQ // G
    q = ins["q_ptr"].view(B, HQ * S * Dh)
    k = ins["k_ptr"].view(B, hkv * S * Dh)
    v = ins["v_ptr"].view(B, hkv * S * Dh)
    out = got.view(B, HQ * S * Dh)
    bq = min(1024, S)
    for b in range(B):
        want = O.attention_prefill(q[b], k[b], v[b], 1, HQ, G, S, Dh, bq, bq, o["causal"], o["scale"])
        T.check(out[b], want, T.ATTENTION, row=Dh, name=f"{case['name']} batch {b}")


@pytest.mark.parametrize("case", all_cases(), ids=lambda c: c["name"])
def test_reference_program_on_b200(case):
    ins = make_inputs(case)
    got_all = run_object(case, ins)
    fam = case["oracle"]["family"]
    if fam == "attention_prefill" and case["oracle"]["batch"] > 1:
        name = [a["name"] for a in case["args"] if a["role"] in ("out", "inout")][0]
        _check_golden(case, ins, name, got_all[name])
        attention_all_heads(case, ins, got_all[name])
        return
    for name, want in run_oracle_all(case, ins).items():
        _check_golden(case, ins, name, got_all[name])
        _check_oracle(case, ins, name, got_all[name], want)


def _check_golden(case, ins, name, got):
    """The reference kernel's own output (Triton interpreter), where recorded: the whole output's hash for
    exact programs, else the recorded sample under the output's parity bar."""
    if not case["golden"]:
        return
    dt = next(a["dtype"] for a in case["args"] if a["name"] == name)
    gold = np.load(os.path.join(HERE, "golden", case["golden"]))
    stride = int(gold[f"{name}__stride"][0])
    gb = as_bits(got.reshape(-1))
    bar = bar_of(case, name)
    if bar == T.EXACT:
        assert hashlib.sha256(gb.tobytes()).digest() == bytes(gold[f"{name}__sha256"]), "differs from the reference kernel"
        return
    g, w = as_float(gb[::stride], dt), as_float(gold[name], dt)
    if dt == "bfloat16":
        g, w = g.to(torch.bfloat16), w.to(torch.bfloat16)
    T.check(g, w, bar, row=row_of(case) if stride == 1 else None,
            magnitude=magnitude_of(case, ins, w) if bar == T.FP32_SUM else None, name=f"{case['name']} vs reference kernel")


def _check_oracle(case, ins, name, got, want):
    bar = bar_of(case, name)
    if bar == T.EXACT:
        assert torch.equal(got.reshape(-1).view(torch.uint8) if got.dtype != torch.bool else got,
                           want.reshape(-1).to(got.dtype).view(torch.uint8)), "differs from the oracle"
        return
    T.check(got, want.to(got.dtype) if got.dtype != want.dtype and bar != T.FP32_SUM else want, bar,
            row=row_of(case), magnitude=magnitude_of(case, ins, want) if bar == T.FP32_SUM else None,
            name=f"{case['name']} vs oracle")
