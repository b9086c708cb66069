"""Time the reference's own kernels executed by the Triton interpreter (TRITON_INTERPRET=1, numpy, one
core) -- the closest runnable analogue of the reference's CPU functional simulation of the same programs,
whose simulator (Spike + the Coprocessor model) is not installable here.  Run in the build container, where
the read-only reference tree exists (the GPU box has no copy of it); the result is committed as
tests/golden/interpreter_baseline.json and bench.py reports it beside its own CPU baseline.

The kernels run with make_golden.py's interpreter shims, on the reference's input convention (one generator
seeded 0, randn per read argument):
  - vector add, fp32 x, y of 1,048,576 (tests/cases/smoke/add.py at BLOCK 1024);
  - row softmax, bf16 [4096, 4096] (configs[1]; validation/pytorchsim/vector_softmax_4096x4096_bf16/00_*);
  - GEMM bf16 128 x 768 x 768 (validation/pytorchsim/gemm_128x768x768_bf16/00_*; the configs[2] kernel
    template at a shape the interpreter finishes);
  - causal attention bf16 16 x 8 heads, S 128 (validation/pytorchsim/attention_prefill_16x8x128_bf16/00_*;
    the configs[3] kernel at a shape the interpreter finishes).

    PTSIM_REFERENCE=<reference checkout> python tests/golden/interpreter_baseline.py [case ...]"""
import os

for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
    os.environ[_v] = "1"

import json  # noqa: E402
import platform  # noqa: E402
import sys  # noqa: E402
import time  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import make_golden as MG  # noqa: E402  (sets TRITON_INTERPRET=1 and checks PTSIM_REFERENCE)


def cpu_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def main():
    import torch
    from pytorchsim_triton_compiler.contract.kernel_spec import load_spec
    torch.set_num_threads(1)
    MG.install_interpreter_shims()
    cases = [
        ("vector_add_1m", os.path.join(MG.REF, "tests", "cases", "smoke", "add.py"), MG.add_config,
         "GB/s", lambda s: 3 * 4 * 1_048_576),
        ("softmax_4096x4096", MG.spec_file("vector_softmax_4096x4096_bf16", 0), None,
         "GB/s", lambda s: 2 * 2 * 4096 * 4096),
        ("gemm_128x768x768", MG.spec_file("gemm_128x768x768_bf16", 0), None,
         "GFLOP/s", lambda s: 2 * 128 * 768 * 768),
        ("attention_16x8x128", MG.spec_file("attention_prefill_16x8x128_bf16", 0), None,
         "GFLOP/s", lambda s: 4 * 16 * 128 * 128 * 128 // 2),
    ]
    out = {"what": "the reference's Triton kernels executed by the Triton 3.6 interpreter (numpy), one thread",
           "measured_in": "the build container (the reference tree is not on the GPU box)",
           "cpu": cpu_name(), "cores": 1, "torch": torch.__version__, "results": {}}
    only = sys.argv[1:]
    for name, path, modify, unit, work in cases:
        if only and name not in only:
            continue
        spec = load_spec(path)
        if modify is not None:
            spec = modify(spec)
        inputs = spec.make_inputs(torch, seed=0) if spec.make_inputs is not None else MG.convention_inputs(spec, set(), {})
        runs, t0 = 0, time.perf_counter()
        while True:                               # whole runs, at least one, until about 10 s have passed
            MG.interpret(spec, inputs)
            runs += 1
            dt = time.perf_counter() - t0
            if dt > 10.0 or runs >= 20:
                break
        sec = dt / runs
        val = work(spec) / sec / 1e9
        out["results"][name] = {"seconds_per_run": round(sec, 4), "value": round(val, 4), "unit": unit,
                                "runs": runs, "source": os.path.relpath(path, MG.REF)}
        print(name, out["results"][name], flush=True)
    path = os.path.join(HERE, "interpreter_baseline.json")
    if only and os.path.exists(path):              # a partial run updates the committed record
        prev = json.load(open(path))
        prev["results"].update(out["results"])
        out["results"] = prev["results"]
    with open(path, "w") as fh:
        json.dump(out, fh, indent=1)
        fh.write("\n")


if __name__ == "__main__":
    main()
