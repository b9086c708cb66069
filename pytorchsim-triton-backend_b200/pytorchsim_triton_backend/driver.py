"""The Triton backend's launch side, kept call-compatible with the reference
(pytorchsim_triton_compiler/triton_extension/python/pytorchsim_triton_backend/driver.py:14-149):

  set_launcher(fn)   registers the function that runs a compiled kernel,
                     fn(binary, kernel_object, grid, args, artifacts=); None unregisters;
  _Launcher          Triton's per-kernel launcher: drops constexpr arguments, passes constexpr values in
                     the kernel object's "constexprs", and hands (binary, kernel_object, grid, args) to the
                     registered function; a launch with none registered raises RuntimeError;
  PYTORCHSIM_COLLECT_FAILURES makes a launch a no-op, as in the reference.

B200 edition: `binary` is the kernel object's launch descriptor (desc.bin) instead of the ELF, and
`cuda_launcher` is the launcher this package offers the device owner: it runs the descriptor on the CUDA
device holding the tensor arguments (runtime/cuda.py launch_tensors), in place, on torch's current stream."""
import json
import os

from triton.backends.compiler import GPUTarget
from triton.backends.driver import DriverBase

_LAUNCHER = None


def set_launcher(fn):
    """Register the function that runs a compiled kernel (None unregisters)."""
    global _LAUNCHER
    _LAUNCHER = fn


def _launcher():
    if _LAUNCHER is None:
        raise RuntimeError("no launcher is registered with the pytorchsim triton backend: the owner of the device "
                           "registers one with pytorchsim_triton_backend.driver.set_launcher")
    return _LAUNCHER


class _Launcher:
    """Triton's launcher for one compiled kernel.  `signature` is the kernel's {name: type} (constexpr
    parameters typed "constexpr"), `constants` the constexpr values by parameter position."""

    def __init__(self, src, metadata):
        self.metadata = metadata
        sig = getattr(src, "signature", {}) or {}
        self.width = len(sig)
        consts = getattr(src, "constants", {}) or {}
        self.constexpr = {i for i, ty in enumerate(sig.values()) if ty == "constexpr"} | \
                         {k[0] for k in consts if isinstance(k, tuple)}
        names = list(sig)
        self.constexprs = {names[k[0]]: v for k, v in consts.items()
                           if isinstance(k, tuple) and len(k) == 1 and k[0] < len(names)
                           and isinstance(v, (int, float, bool))}
        _launcher()

    def __call__(self, grid_x, grid_y, grid_z, stream, function, packed_metadata, launch_metadata,
                 enter_hook, exit_hook, *args):
        if os.environ.get("PYTORCHSIM_COLLECT_FAILURES"):
            return
        kobj = getattr(self.metadata, "kernel_object", "")
        if not kobj:
            raise RuntimeError("this kernel was compiled without pytorchsim_spec, which stops at the Triton IR: it "
                               "has no binary to launch")
        if len(args) == self.width:
            args = tuple(a for i, a in enumerate(args) if i not in self.constexpr)
        if self.constexprs:
            kobj = json.dumps({**json.loads(kobj), "constexprs": self.constexprs})
        _launcher()(function, kobj, (grid_x, grid_y, grid_z), args,
                    artifacts=getattr(self.metadata, "artifacts", None))


class _Utils:
    """What Triton's CompiledKernel asks of a driver before a launch: the device's limits and the binary
    loaded.  The descriptor is its own handle: the registered launcher runs it."""

    def get_device_properties(self, device):
        _launcher()
        return {"max_shared_mem": 2 ** 62}

    def load_binary(self, name, kernel, shared, device):
        _launcher()
        return kernel, kernel, 0, 0, 1

    def unload_module(self, module):
        pass


class CPUDriver(DriverBase):
    """Triton's driver for kernels compiled by this backend (the reference's class name; the launches it
    makes go to the registered launcher, cuda_launcher for the B200).  Never selected automatically: the
    device owner makes it active with triton.runtime.driver.set_active(CPUDriver())."""

    def __init__(self):
        self.utils = _Utils()
        self.launcher_cls = _Launcher

    def get_current_device(self):
        return 0

    def get_current_stream(self, device):
        return 0

    def set_current_device(self, device):
        pass

    @staticmethod
    def is_active():
        return False

    def map_python_to_cpp_type(self, ty: str) -> str:
        raise NotImplementedError("the pytorchsim backend maps no C types: it launches through set_launcher")

    def get_current_target(self):
        return GPUTarget("b200", 100, 32)

    def get_active_torch_device(self):
        import torch
        return torch.device("cuda", 0)

    def get_device_interface(self):
        import torch
        return torch.cuda

    def get_benchmarker(self):
        raise NotImplementedError("the pytorchsim backend benchmarks nothing itself")

    def get_empty_cache_for_benchmark(self):
        raise NotImplementedError("the pytorchsim backend benchmarks nothing itself")

    def clear_cache(self, cache):
        pass


class activated:
    """`with activated(): ...` makes a CPUDriver Triton's active driver for the block and then restores the one
    that was active before (also when none was: Triton then creates its default again on first use)."""

    def __enter__(self):
        from triton.runtime import driver
        self._saved = driver._active
        driver.set_active(CPUDriver())
        return driver.active

    def __exit__(self, *exc):
        from triton.runtime import driver
        driver._active = self._saved
        return False


def cuda_launcher(binary, kernel_object, grid, args, artifacts=None):
    """A launcher for set_launcher: run descriptor `binary` over the tensor arguments `args` on their CUDA
    device, in place, on torch's current stream.

    Scalars: the lowering folded the kernel's scalar parameters into the descriptor, so each scalar the
    launch passes (positionally, or specialised by Triton into the kernel object's "constexprs") must equal
    the value the descriptor holds; another value is refused, never run with the old one.
    Tensors: a non-contiguous argument runs on a contiguous copy, and a written one (out / inout) is copied
    back into the caller's tensor after the launch."""
    from pytorchsim_triton_compiler.contract import kernel_object as ko
    from pytorchsim_triton_compiler.runtime import cuda as RC
    manifest = json.loads(kernel_object) if isinstance(kernel_object, (str, bytes)) else kernel_object
    ko.refuse_grid_past_bound(manifest, grid)
    if tuple(ko.grid3(grid)) != tuple(ko.grid3(manifest["grid"])):
        raise RuntimeError(f"{manifest.get('name')}: lowered for grid {tuple(ko.grid3(manifest['grid']))}, launched "
                           f"with {tuple(ko.grid3(grid))}; relower for the new grid")
    tensors = [a for a in args if hasattr(a, "data_ptr")]
    if len(tensors) != len(manifest["args"]):
        raise RuntimeError(f"{manifest.get('name')}: {len(tensors)} tensors for {len(manifest['args'])} arguments")
    specialised = manifest.get("constexprs", {}) or {}
    table = [s["name"] for s in manifest.get("scalars", [])]
    positional = [n for n in table if n not in specialised]
    values = [a for a in args if not hasattr(a, "data_ptr")]
    if len(values) != len(positional):
        raise RuntimeError(f"{manifest.get('name')}: {len(values)} scalar arguments for the scalar parameters "
                           f"{positional}")
    given = dict(zip(positional, values))
    given.update({n: v for n, v in specialised.items() if n in table})
    ko.check_launch_scalars(manifest, given)
    run = [t if t.is_contiguous() else t.contiguous() for t in tensors]
    RC.launch_tensors(bytes(binary), run)
    for arg, mine, ran in zip(manifest["args"], tensors, run):
        if ran is not mine and arg["role"] != "in":
            mine.copy_(ran)
    return tensors
