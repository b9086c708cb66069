"""Out-of-bounds writes caught on the GPU: every committed kernel object launched with each argument inside a
larger device buffer whose guard bands before and after it hold a poison pattern, and, after the launch,

  - every guard band still holds the poison (no kernel wrote past either end of a tensor it was given), and
  - every read-only argument is unchanged (no kernel wrote into an input).

The GPU analogue of the reference's scratchpad poisoning before every run (codegen/wrapper.py:64-79
poison_spad): there the poison word exposes reads of memory no DMA filled; here the poison exposes writes
outside the tensors.  The guards are 4 KiB on each side (a multiple of 256 bytes, so every argument keeps
the 16-byte alignment the TMA descriptors need), filled with 0xA5 bytes, a pattern no zero-filled output
or seeded input produces in a whole band.  Objects whose arguments pass 1.5 GB in total are left to the
object tests (the MoE expert weights).

The same poisoning checks the DMA-access trace (runtime/dma_access.py): run twice with outputs filled with two
different byte patterns, the elements that differ from the pattern in either run are the ones the kernel
wrote, and they must be exactly the elements the trace's write streams name."""
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


def written_elements(case, m, blob, ins, poison, dev):
    """Per written argument, a bool tensor of the elements a launch changed from the poison `poison`."""
    views, bufs = [], []
    for a in m["args"]:
        t = ins[a["name"]]
        if a["role"] in ("out", "inout"):
            t = torch.full((t.numel() * t.element_size(),), poison, dtype=torch.uint8).view(t.dtype)
        b, v = guarded(t, dev)
        bufs.append(b)
        views.append(v)
    RC.launch_tensors(blob, views, 0, D.from_bytes(blob).units)
    torch.cuda.synchronize()
    out = {}
    for a, v in zip(m["args"], views):
        if a["role"] in ("out", "inout"):
            by = v.reshape(-1).view(torch.uint8).view(v.numel(), v.element_size())
            out[a["name"]] = (by != poison).any(dim=1)
    return out


@pytest.mark.parametrize("case", [c for c in cases() if sum(a["numel"] for a in c["args"]
                                                            if a["role"] in ("out", "inout")) <= (32 << 20)],
                         ids=lambda c: c["name"])
def test_trace_write_footprint_is_what_the_kernel_writes(case):
    """The DMA-access trace's write streams (runtime/dma_access.py) name exactly the elements the kernel
    changes: outputs poisoned with two different byte patterns, an element written in either run counts."""
    import numpy as np
    from pytorchsim_triton_compiler.runtime import dma_access as DA
    dev = torch.device("cuda", 0)
    d = os.path.join(OBJ, case["name"])
    m = ko.read(d)
    blob = ko.read_desc(d, m)
    desc = D.from_bytes(blob)
    ins = make_inputs(case)
    wa = written_elements(case, m, blob, ins, 0xA5, dev)
    wb = written_elements(case, m, blob, ins, 0x5A, dev)
    host = {k: v.numpy() if v.dtype != torch.bfloat16 else v.view(torch.int16).numpy() for k, v in ins.items()}
    names = [a["name"] for a in m["args"]]
    want = {n: torch.zeros_like(wa[n]) for n in wa}
    for s in DA.streams(desc, 0, desc.units, names, host=host):
        if s["dir"] != "write":
            continue
        acc = s["access"]
        if "map" in acc:
            e = torch.from_numpy(DA.elements(acc)).to(dev)
        else:
            rows = acc["indirect"]["resolved_rows"]
            c = acc["indirect"]["row_elems"]
            if not rows:
                continue
            e = torch.from_numpy(np.concatenate([np.arange(lo * c, hi * c) for lo, hi in rows])).to(dev)
        want[s["arg"]][e] = True
    for n in wa:
        got = wa[n] | wb[n]
        assert torch.equal(got, want[n]), (f"{case['name']}: {n}: the trace names {int(want[n].sum())} written "
                                           f"elements, the kernel wrote {int(got.sum())} "
                                           f"({int((got & ~want[n]).sum())} outside the trace)")
