"""The Triton backend plugin's Python side, B200 edition, kept call-compatible with the reference's
pytorchsim_triton_backend package:
  compiler  the backend triton.compile selects for GPUTarget("cpu" | "npu" | "b200"): Triton's front end to
            TTIR, then the B200 lowering to a launch descriptor plus its kernel object (register() installs it);
  driver    the launcher registry (set_launcher) a device owner hooks, Triton's driver for these kernels
            (CPUDriver) and cuda_launcher, the launcher that runs a descriptor on the GPU holding the tensors."""


def register():
    """Install the backend into this process's Triton; importable afterwards as triton.backends.pytorchsim."""
    from .compiler import register as _register
    return _register()
