"""Lower every program of the reference's validation bundle (validation/pytorchsim/<workload>/<NN_kernel>/
*_spec.py, read from the reference tree in the build container) with the B200 lowering and record what
each became: tests/golden/lowering_coverage.json maps workload -> program -> descriptor kind, or
"refused: <reason>".  The record is committed; rerun after a lowering change:

    python tests/golden/lowering_coverage.py"""
import glob
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("PTSIM_REFERENCE", "")
if not REF or not os.path.isdir(REF):
    raise SystemExit("set PTSIM_REFERENCE to the reference checkout (the PyTorchSim-Triton-Backend source tree)")
sys.path.insert(0, os.path.join(ROOT, "pytorchsim-triton-backend_b200"))


def main():
    from pytorchsim_triton_compiler.contract.kernel_spec import load_spec
    from pytorchsim_triton_compiler.contract.stop import Refused
    from pytorchsim_triton_compiler.targets.b200 import lower as L
    out, lowered, total = {}, 0, 0
    for path in sorted(glob.glob(os.path.join(REF, "validation", "pytorchsim", "*", "*", "*_spec.py"))):
        prog = os.path.basename(os.path.dirname(path))
        wl = os.path.basename(os.path.dirname(os.path.dirname(path)))
        total += 1
        try:
            kind = L.lower(load_spec(path)).kind
            lowered += 1
        except Refused as e:
            kind = f"refused: {e}"
        out.setdefault(wl, {})[prog] = kind
    with open(os.path.join(HERE, "lowering_coverage.json"), "w") as fh:
        json.dump({"lowered": lowered, "programs": total, "workloads": out}, fh, indent=1, sort_keys=True)
        fh.write("\n")
    print(f"{lowered} of {total} programs lowered")


if __name__ == "__main__":
    main()
