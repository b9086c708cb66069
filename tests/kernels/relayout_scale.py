"""A pointwise program with a non-trivial DMA box: out[t, h, d] = 2 * x[h, t, d] + y[t, h, d] (heads-major to
token-major relayout fused with a scale and an add), written for this suite in the style of an Inductor
pointwise kernel (xindex digits by // and %)."""
from pytorchsim_triton_compiler.contract.kernel_spec import KernelSpec, Arg, IN, OUT

T, H, D = 64, 4, 32
N = T * H * D
BLOCK = 2048


def kernel():
    import triton
    import triton.language as tl

    @triton.jit
    def relayout_scale(x_ptr, y_ptr, o_ptr, XBLOCK: tl.constexpr):
        xindex = tl.program_id(0) * XBLOCK + tl.arange(0, XBLOCK)
        d = xindex % 32
        h = (xindex // 32) % 4
        t = xindex // 128
        a = tl.load(x_ptr + (d + 32 * t + 2048 * h)).to(tl.float32)
        b = tl.load(y_ptr + xindex).to(tl.float32)
        tl.store(o_ptr + xindex, a * 2.0 + b)

    return relayout_scale


def make_inputs(torch, seed=0):
    g = torch.Generator().manual_seed(seed)
    return {"x": torch.randn(N, generator=g).to(torch.bfloat16), "y": torch.randn(N, generator=g).to(torch.bfloat16)}


def reference(inputs):
    x = inputs["x"].float().view(H, T, D).transpose(0, 1).reshape(-1)
    return {"o": (x * 2.0 + inputs["y"].float()).to(inputs["x"].dtype)}


SPEC = KernelSpec(name="relayout_scale", kernel=kernel,
                  signature={"x_ptr": "*bf16", "y_ptr": "*bf16", "o_ptr": "*bf16", "XBLOCK": "constexpr"},
                  constexprs={"XBLOCK": BLOCK},
                  args=[Arg("x", IN, "bfloat16", (N,)), Arg("y", IN, "bfloat16", (N,)), Arg("o", OUT, "bfloat16", (N,))],
                  grid=(N // BLOCK,), reference=reference, make_inputs=make_inputs, rtol=1e-2, atol=1e-2)
