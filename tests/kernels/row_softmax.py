"""Row softmax over fp32 rows written for this suite (a textbook Triton softmax: one block of rows per
program, the whole row in one block): the lowering must recognise it as the softmax row program."""
from pytorchsim_triton_compiler.contract.kernel_spec import KernelSpec, Arg, IN, OUT

ROWS, COLS, XB = 256, 512, 16


def kernel():
    import triton
    import triton.language as tl

    @triton.jit
    def softmax_rows(x_ptr, o_ptr, XBLOCK: tl.constexpr, R0_BLOCK: tl.constexpr):
        xnumel = 256
        r0_numel = 512
        xindex = tl.program_id(0) * XBLOCK + tl.arange(0, XBLOCK)[:, None]
        r0_index = tl.arange(0, R0_BLOCK)[None, :]
        x = tl.load(x_ptr + (r0_index + 512 * xindex)).to(tl.float32)
        m = tl.max(x, 1)[:, None]
        e = tl.exp(x - m)
        s = tl.sum(e, 1)[:, None]
        tl.store(o_ptr + (r0_index + 512 * xindex), e / s)

    return softmax_rows


def make_inputs(torch, seed=0):
    g = torch.Generator().manual_seed(seed)
    return {"x": torch.randn(ROWS * COLS, generator=g)}


def reference(inputs):
    return {"o": inputs["x"].view(ROWS, COLS).softmax(dim=1).reshape(-1)}


SPEC = KernelSpec(name="softmax_rows", kernel=kernel,
                  signature={"x_ptr": "*fp32", "o_ptr": "*fp32", "XBLOCK": "constexpr", "R0_BLOCK": "constexpr"},
                  constexprs={"XBLOCK": XB, "R0_BLOCK": COLS},
                  args=[Arg("x", IN, "float32", (ROWS * COLS,)), Arg("o", OUT, "float32", (ROWS * COLS,))],
                  grid=(ROWS // XB,), reference=reference, make_inputs=make_inputs, rtol=1e-5, atol=1e-6)
