"""A kernel the executor must refuse: an atomic accumulation (the reference refuses atomics too,
contract/stop.py Reason.ATOMICS)."""
from pytorchsim_triton_compiler.contract.kernel_spec import KernelSpec, Arg, IN, INOUT
from pytorchsim_triton_compiler.contract.stop import Reason, Stop

N = 1024


def kernel():
    import triton
    import triton.language as tl

    @triton.jit
    def atomic_accumulate(x_ptr, o_ptr, XBLOCK: tl.constexpr):
        xindex = tl.program_id(0) * XBLOCK + tl.arange(0, XBLOCK)
        tl.atomic_add(o_ptr + xindex % 8, tl.load(x_ptr + xindex))

    return atomic_accumulate


SPEC = KernelSpec(name="atomic_accumulate", kernel=kernel,
                  signature={"x_ptr": "*fp32", "o_ptr": "*fp32", "XBLOCK": "constexpr"}, constexprs={"XBLOCK": 128},
                  args=[Arg("x", IN, "float32", (N,)), Arg("o", INOUT, "float32", (8,))], grid=(N // 128,),
                  reference=None, make_inputs=None, expect="refuse", expect_why="atomics have no tile program",
                  expect_stop=Stop("lower", Reason.ATOMICS))
