"""What a device is: something that runs a kernel object over tensors on disk (the reference's
tests/runtime/device/base.py:25-59 and __init__.py:12-21).  A device reads the object's manifest and its
descriptor, never the compiler's source or the kernel's Python spec.  This build has one: "cuda"."""
import contextlib

from ..contract import kernel_object


class DeviceError(RuntimeError):
    pass


@contextlib.contextmanager
def _no_step(_name):
    yield


def _plain_error(message, **kw):
    return DeviceError(message)


class Launch:
    """One launch: a compiled object, where its tensors are, and how to run."""

    def __init__(self, obj_dir, manifest, runtime_dir, raw_paths, log, run=None, step=None, error=None, grid=None,
                 devices=None):
        self.grid = grid
        self.obj_dir = obj_dir
        self.manifest = manifest
        self.runtime_dir = runtime_dir
        self.raw_paths = raw_paths
        self.log = log
        self.run = run
        self.step = step or _no_step
        self.error = error or _plain_error
        self.devices = devices

    def artifact(self, kind):
        try:
            return kernel_object.artifact(self.obj_dir, kind, manifest=self.manifest)
        except kernel_object.ObjectError as e:
            raise DeviceError(f"{e}. This device needs it.") from None


class Device:
    name = None

    def launch(self, req):
        raise NotImplementedError


class CudaDevice(Device):
    """Runs the whole launch on the visible B200s, cutting the units over GPUs when the object allows."""

    name = "cuda"

    def launch(self, req):
        import os
        from . import cuda
        with open(req.artifact("desc"), "rb") as fh:
            blob = fh.read()
        want = os.environ.get("PYTORCHSIM_COMPILE_CUDA_DEVICES", "").strip()
        with req.step("run the grid"):
            cuda.launch(blob, req.manifest, req.runtime_dir, req.raw_paths, log=req.log, error=req.error,
                        grid=req.grid, devices=req.devices, want_jobs=want or None)
        req.log("[cuda] finished")
        return req.runtime_dir


REGISTRY = {d.name: d for d in (CudaDevice(),)}


def get(name):
    try:
        return REGISTRY[name]
    except KeyError:
        raise DeviceError(f"no device named {name!r}. Have: {', '.join(sorted(REGISTRY))}.") from None
