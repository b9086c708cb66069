"""pytorchsim_triton_compiler, B200 edition: the launch API of PyTorchSim-Triton-Backend (kernel specs,
kernel.json manifests, .raw tensors, the runtime launcher, the Triton backend's set_launcher and the CLI)
over a functional executor made of hand-written sm_100a CUDA kernels instead of Spike + the Coprocessor
model.  The package name is the reference's, so callers import it unchanged."""
__version__ = "0.1.0+b200"
