"""A vector add written for this suite (o = x + y over n fp32 values, one BLOCK per program): the kernel the
Triton-plugin tests compile through triton.compile and launch through set_launcher."""
from pytorchsim_triton_compiler.contract.kernel_spec import KernelSpec, Arg, IN, OUT

N = 1 << 16
BLOCK = 1024


def kernel():
    import triton
    import triton.language as tl

    @triton.jit
    def add_kernel(x_ptr, y_ptr, o_ptr, n, BLOCK: tl.constexpr):
        offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
        keep = offs < n
        tl.store(o_ptr + offs, tl.load(x_ptr + offs, mask=keep) + tl.load(y_ptr + offs, mask=keep), mask=keep)

    return add_kernel


SPEC = KernelSpec(name="add_kernel", kernel=kernel,
                  signature={"x_ptr": "*fp32", "y_ptr": "*fp32", "o_ptr": "*fp32", "n": "i32", "BLOCK": "constexpr"},
                  constexprs={"BLOCK": BLOCK},
                  args=[Arg("x_ptr", IN, "float32", (N,)), Arg("y_ptr", IN, "float32", (N,)),
                        Arg("o_ptr", OUT, "float32", (N,))],
                  grid=(N // BLOCK,), reference=None, make_inputs=None, extra={"scalar_values": {"n": N}})
