"""Build libptsim_b200.so, the sm_100a executor, in-tree (next to the package that loads it).

    python build.py            # or: from csrc.build import build; build()

The library is one translation unit (ptsim_b200.cu includes the kernel headers) compiled for sm_100a
only, with the CUDA runtime linked statically and the driver's cuTensorMapEncodeTiled fetched at run
time, so it loads beside any PyTorch build without a libcuda link.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "pytorchsim_triton_compiler", "_lib")
OUT = os.path.join(PKG, "libptsim_b200.so")
SOURCES = ["ptsim_b200.cu"]
# Every kernel header of this directory (the translation unit includes them) and the ABI header.
DEPS = sorted(f for f in os.listdir(HERE) if f.endswith(".cuh")) + [os.path.join("..", "..", "include", "ptsim_b200.h")]


def nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the sm_100a executor cannot be built")


def stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(os.path.join(HERE, f)) > t for f in SOURCES + DEPS)


def build(force=False, verbose=False, extra=()):
    """Compile the library if a source is newer than it; returns its path."""
    if not force and not stale():
        return OUT
    os.makedirs(PKG, exist_ok=True)
    cmd = [nvcc(), "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
           "-Xcompiler", "-fPIC,-O2", "-shared", "--expt-relaxed-constexpr", "-Xptxas", "-v" if verbose else "-O3",
           "-o", OUT + ".tmp", *[os.path.join(HERE, s) for s in SOURCES], *extra]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + done.stdout[-6000:] + done.stderr[-6000:])
    os.replace(OUT + ".tmp", OUT)
    if verbose:
        sys.stderr.write(done.stderr)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
