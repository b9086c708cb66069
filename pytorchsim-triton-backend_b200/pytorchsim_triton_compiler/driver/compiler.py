"""The stage machine of the B200 build (the reference's driver/compiler.py:35-104 stage table and
register_stage, :56-68): a kernel file goes through

    lower   trace the Triton source and lower it into a launch descriptor: kernel.json + desc.bin
    cuda    materialise the spec's inputs as .raw files and run the object on the CUDA device
    verify  compare the written .raw files with the spec's torch reference (rtol/atol of the spec)

Each stage is a function of a Ctx; stages run in table order between --from and --to.  A Refused lowering
leaves failure.json (kind "refuse", its Reason) and stops; so does a device failure (kind "device")."""
import dataclasses
import os
import sys
import time

from ..contract import failure, kernel_object
from ..contract.stop import Refused


@dataclasses.dataclass
class Stage:
    name: str
    fn: object
    help: str


STAGES = []


def register_stage(name, fn, help_text="", after=None):
    """Add (or replace) a stage; `after` places a new one right behind an existing stage.  Idempotent."""
    for i, s in enumerate(STAGES):
        if s.name == name:
            STAGES[i] = Stage(name, fn, help_text)
            return STAGES
    st = Stage(name, fn, help_text)
    if after is not None:
        at = next(i for i, s in enumerate(STAGES) if s.name == after)
        STAGES.insert(at + 1, st)
    else:
        STAGES.append(st)
    return STAGES


class StageError(RuntimeError):
    def __init__(self, stage, message, **facts):
        super().__init__(message)
        self.stage, self.facts = stage, facts


class Ctx:
    def __init__(self, spec, workdir, log):
        self.spec, self.workdir, self.log = spec, workdir, log
        self.runtime_dir = os.path.join(workdir, "runtime")
        self.inputs = None
        self.raw_paths = {}
        self.timings = {}


def stage_lower(ctx):
    from ..targets.b200 import lower as L
    lowered = L.lower(ctx.spec)
    path = kernel_object.write(ctx.workdir, ctx.spec, lowered.summary, lowered.blob)
    ctx.log(f"[lower] {ctx.spec.name}: {lowered.kind} -> {path}")
    return path


def _np_dtype(name):
    import numpy as np
    return np.dtype(kernel_object.NP_DTYPE[name])


def materialise_inputs(ctx):
    """The spec's inputs from make_inputs(torch, seed=0) as .raw files (bf16 as uint16 bits), written
    arguments zero-filled: the reference suite's _materialise_inputs (tests/runtime/stages.py:72-93)."""
    import numpy as np
    import torch
    os.makedirs(ctx.runtime_dir, exist_ok=True)
    if ctx.inputs is None:
        ctx.inputs = ctx.spec.make_inputs(torch, seed=0)
    for a in ctx.spec.args:
        p = os.path.join(ctx.runtime_dir, f"{a.name}.raw")
        ctx.raw_paths[a.name] = p
        if a.role in ("in", "inout"):
            t = ctx.inputs[a.name].contiguous().cpu()
            if a.dtype == "bfloat16":
                t = t.view(torch.uint16)
            elif a.dtype in ("float8_e5m2", "float8_e4m3fn"):
                t = t.view(torch.uint8)
            t.numpy().astype(_np_dtype(a.dtype)).tofile(p)
        else:
            np.zeros(a.numel, dtype=_np_dtype(a.dtype)).tofile(p)


def stage_cuda(ctx):
    from ..runtime import device
    materialise_inputs(ctx)
    manifest = kernel_object.read(ctx.workdir)
    kernel_object.refuse_if_it_disagrees(manifest, ctx.spec)
    req = device.Launch(ctx.workdir, manifest, ctx.runtime_dir, ctx.raw_paths, ctx.log,
                        error=lambda message, **kw: StageError("cuda", message, **kw))
    device.get("cuda").launch(req)
    return ctx.runtime_dir


def stage_verify(ctx):
    """Compare each written argument with spec.reference(inputs): PASS/FAIL with max abs/rel error (the
    reference suite's verify.compare, tests/runtime/verify.py:28-69)."""
    import numpy as np
    import torch
    if ctx.inputs is None:
        ctx.inputs = ctx.spec.make_inputs(torch, seed=0)
    want_all = ctx.spec.reference(ctx.inputs) if ctx.spec.reference else {}
    ok_all, lines = True, []
    for a in ctx.spec.outputs():
        if a.name not in want_all:
            lines.append(f"  {a.name:<10} SKIP  (the spec's reference gives no value)")
            continue
        p = ctx.raw_paths.get(a.name) or os.path.join(ctx.runtime_dir, f"{a.name}.raw")
        got = np.fromfile(p, dtype=_np_dtype(a.dtype), count=a.numel)
        g = torch.from_numpy(got.copy())
        if a.dtype == "bfloat16":
            g = g.view(torch.bfloat16)
        g = g.float().reshape(a.shape)
        w = want_all[a.name].detach().cpu().float().reshape(a.shape)
        ok = torch.allclose(g, w, rtol=ctx.spec.rtol, atol=ctx.spec.atol, equal_nan=True)
        d = (g - w).abs()
        ok_all &= bool(ok)
        lines.append(f"  {a.name:<10} {'PASS' if ok else 'FAIL'}  shape={tuple(a.shape)} dtype={a.dtype}")
        lines.append(f"    max_abs_err = {float(d.max()) if d.numel() else 0:.6g}   (rtol={ctx.spec.rtol}, atol={ctx.spec.atol})")
    for line in lines:
        ctx.log(line)
        print(line)
    if not ok_all:
        raise StageError("verify", "outputs differ from the reference")
    return ok_all


register_stage("lower", stage_lower, "trace the Triton kernel and lower it into a B200 launch descriptor")
register_stage("cuda", stage_cuda, "run the kernel object on the CUDA device over .raw tensors")
register_stage("verify", stage_verify, "compare the outputs with the spec's torch reference")


def run(spec, workdir, frm=None, to=None, log=None):
    """Run the stages from `frm` to `to` (inclusive) for `spec` in `workdir`; returns the last result."""
    os.makedirs(workdir, exist_ok=True)
    logfile = open(os.path.join(workdir, "stage.log"), "a")

    def _log(msg):
        logfile.write(msg + "\n")
        logfile.flush()
        if log:
            log(msg)

    names = [s.name for s in STAGES]
    lo = names.index(frm) if frm else 0
    hi = names.index(to) if to else len(names) - 1
    ctx = Ctx(spec, workdir, _log)
    failure.forget(workdir)
    result = None
    try:
        for st in STAGES[lo:hi + 1]:
            t0 = time.perf_counter()
            try:
                result = st.fn(ctx)
            except Refused as e:
                failure.leave(workdir, st.name, failure.REFUSED, str(e), reason=e.reason.value)
                raise
            except StageError as e:
                failure.leave(workdir, st.name, failure.DEVICE if st.name == "cuda" else failure.ERROR, str(e),
                              **{k: v for k, v in e.facts.items() if isinstance(v, (int, str, float))})
                raise
            except Exception as e:  # noqa: BLE001 -- recorded, then re-raised
                failure.leave(workdir, st.name, failure.ERROR, f"{type(e).__name__}: {e}")
                raise
            ctx.timings[st.name] = time.perf_counter() - t0
            _log(f"[{st.name}] done in {ctx.timings[st.name]:.3f} s")
    finally:
        logfile.close()
    return result
