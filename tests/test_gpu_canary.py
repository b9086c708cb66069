"""Out-of-bounds writes caught on the GPU: every committed kernel object launched with each argument inside a
larger device buffer whose guard bands before and after it hold a poison pattern, and, after the launch,

  - every guard band still holds the poison (no kernel wrote past either end of a tensor it was given), and
  - every read-only argument is unchanged (no kernel wrote into an input).

The GPU analogue of the reference's scratchpad poisoning before every run (codegen/wrapper.py:64-79
poison_spad): there the poison word exposes reads of memory no DMA filled; here the poison exposes writes
outside the tensors.  The guards are 4 KiB on each side (a multiple of 256 bytes, so every argument keeps
the 16-byte alignment the TMA descriptors need), filled with 0xA5 bytes, a pattern no zero-filled output
or seeded input produces in a whole band.  Objects whose arguments pass 1.5 GB in total are left to the
object tests (the MoE expert weights)."""
import json
import os

import pytest
import torch

from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.runtime import cuda as RC
from tests.test_oracle_golden import make_inputs

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
OBJ = os.path.join(HERE, "golden", "objects")
GUARD = 4096
POISON = 0xA5
LIMIT = 1500 << 20


def cases():
    with open(os.path.join(HERE, "golden", "index.json")) as fh:
        names = json.load(fh)
    out = []
    for n in names:
        c = json.load(open(os.path.join(OBJ, n, "case.json")))
        size = sum(a["numel"] * torch.empty(0, dtype=getattr(torch, a["dtype"])).element_size() for a in c["args"])
        if size <= LIMIT:
            out.append(c)
    return out


def guarded(t, dev):
    """`t` copied into the middle of a poisoned byte buffer on `dev`: (the buffer, the tensor view)."""
    nbytes = t.numel() * t.element_size()
    buf = torch.full((GUARD + nbytes + GUARD,), POISON, dtype=torch.uint8, device=dev)
    view = buf[GUARD:GUARD + nbytes].view(t.dtype)
    view.copy_(t.reshape(-1))
    return buf, view


@pytest.mark.parametrize("case", cases(), ids=lambda c: c["name"])
def test_no_write_outside_the_tensors(case):
    dev = torch.device("cuda", 0)
    d = os.path.join(OBJ, case["name"])
    m = ko.read(d)
    blob = ko.read_desc(d, m)
    ins = make_inputs(case)
    bufs, views = [], []
    for a in m["args"]:
        b, v = guarded(ins[a["name"]], dev)
        bufs.append(b)
        views.append(v)
    before = [b.clone() for b in bufs]
    RC.launch_tensors(blob, views, 0, D.from_bytes(blob).units)
    torch.cuda.synchronize()
    for a, b, b0 in zip(m["args"], bufs, before):
        lo, hi = b[:GUARD], b[-GUARD:]
        assert bool((lo == POISON).all()), f"{case['name']}: a write landed in the guard before {a['name']}"
        assert bool((hi == POISON).all()), f"{case['name']}: a write landed in the guard after {a['name']}"
        if a["role"] == "in":
            assert torch.equal(b, b0), f"{case['name']}: the read-only argument {a['name']} changed"
