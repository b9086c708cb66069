"""pytorchsim-triton-compiler, B200 edition (the reference's cli.py:21-127 entry point):

    pytorchsim-triton-compiler <kernel.py|spec.json> [--workdir W] [--from STAGE] [--to STAGE] [--list-stages]
    pytorchsim-triton-compiler doctor      what this machine can run (nvcc, GPU, library, NCCL)
    pytorchsim-triton-compiler target      the execution target this build lowers for

A kernel file is lowered (stage `lower`), run on the CUDA device (`cuda`) and checked against its spec's
torch reference (`verify`).  Exit code 0 on success, 1 on a failure, 2 on a refusal."""
import argparse
import json
import os
import shutil
import sys


def parser():
    ap = argparse.ArgumentParser(prog="pytorchsim-triton-compiler")
    ap.add_argument("kernel", help="a kernel file defining SPEC, a JSON spec, or doctor / target")
    ap.add_argument("--workdir", default=None)
    ap.add_argument("--from", dest="frm", default=None)
    ap.add_argument("--to", default=None)
    ap.add_argument("--list-stages", action="store_true")
    ap.add_argument("--quiet", action="store_true")
    return ap


def doctor():
    from .runtime import native
    out = {"nvcc": shutil.which("nvcc") or ("/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else None),
           "library": native.library_path(), "library_built": os.path.exists(native.library_path())}
    try:
        native.load()
        out["library_loads"] = True
    except native.NativeUnavailable as e:
        out["library_loads"] = str(e)
    try:
        import torch
        out["torch"] = torch.__version__
        out["gpus"] = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())] \
            if torch.cuda.is_available() else []
        import torch.distributed as dist
        out["nccl"] = dist.is_nccl_available()
    except Exception as e:  # noqa: BLE001
        out["torch"] = f"unavailable: {e}"
    print(json.dumps(out, indent=1))
    return 0


def target():
    """The target this build lowers for and every descriptor kind its executor runs (codegen/descriptors.py
    KIND_NAME, the PTSIM_KIND_* values of include/ptsim_b200.h)."""
    from .codegen import descriptors as D
    print(json.dumps({"name": "b200", "arch": "sm_100a", "executor": "libptsim_b200.so",
                      "kinds": [D.KIND_NAME[k] for k in sorted(D.KIND_NAME)]}, indent=1))
    return 0


def run(opts):
    from .contract.kernel_spec import load_spec
    from .contract.stop import Refused
    from .driver import compiler
    if opts.list_stages:
        for s in compiler.STAGES:
            print(f"{s.name:8s} {s.help}")
        return 0
    spec = load_spec(opts.kernel)
    workdir = opts.workdir or os.path.join(os.getcwd(), "pytorchsim-work", spec.name)
    log = None if opts.quiet else (lambda m: print(m, file=sys.stderr))
    try:
        compiler.run(spec, workdir, opts.frm, opts.to, log=log)
    except Refused as e:
        print(f"refused ({e.reason.value}): {e}", file=sys.stderr)
        return 2
    except Exception as e:  # noqa: BLE001
        print(f"failed: {type(e).__name__}: {e}", file=sys.stderr)
        return 1
    return 0


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if argv[:1] == ["doctor"]:
        return doctor()
    if argv[:1] == ["target"]:
        return target()
    return run(parser().parse_args(argv))


if __name__ == "__main__":
    sys.exit(main())
