"""Generate the committed parity fixtures from the reference (run in the build container, where the read-only
reference tree exists; the GPU box only reads what this writes):

  tests/golden/objects/<case>/kernel.json + desc.bin
      the B200 lowering of the reference's own kernel (its KernelSpec and Triton source, loaded from the
      reference tree), i.e. the kernel object the CUDA device runs; plus case.json: the input convention
      (the reference spec's make_inputs: one generator seeded 0, randn per read argument in order) and the
      oracle program with its parameters, read off the kernel source by hand (cited below);
  tests/golden/vectors/<case>.npz
      for the small cases, the outputs of the reference's kernel executed by the Triton interpreter
      (TRITON_INTERPRET=1, numpy) on make_inputs(torch, seed=0): the functional result of the reference's
      program.  Outputs over 8192 elements are stored as an evenly strided sample plus the SHA-256 of the
      whole output.

Three shims make the interpreter run these kernels as the NPU defines them:
  - Triton 3.6's interpreter multiplies bf16 tl.dot operands as their raw uint16 bits; the shim widens
    them to fp32 first (the value tl.dot(bf16, bf16, out_dtype=fp32) is defined to use);
  - Inductor's `libdevice.exp / rsqrt` resolve to the CUDA libdevice module, which the interpreter does not
    patch; the shim routes them to tl.exp / tl.rsqrt;
  - the interpreter narrows fp32 to bf16 by truncation; the NPU packs bf16 rounding to nearest, ties to
    even (misc.pack, targets/tpu/include/Dialect/PyTorchSimTpu/IR/PyTorchSimTpuOps.td:46-50), and so does
    Triton's own default cast; the shim rounds to nearest even.
The interpreter's and Triton's block limit (2**20 elements) is lifted so the bundle's large blocks run.

    python tests/golden/make_golden.py [--only <case>]"""
import argparse
import contextlib
import copy
import dataclasses
import hashlib
import json
import math
import os
import shutil
import sys

os.environ["TRITON_INTERPRET"] = "1"
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("PTSIM_REFERENCE", "")
if not REF or not os.path.isdir(REF):
    raise SystemExit("set PTSIM_REFERENCE to the reference checkout (the PyTorchSim-Triton-Backend source tree)")
sys.path.insert(0, os.path.join(ROOT, "pytorchsim-triton-backend_b200"))
sys.path.insert(0, ROOT)

V = os.path.join(REF, "validation", "pytorchsim")
Q2048 = "qwen3_8b_layer_prefill_2048x2048_bf16"
Q128 = "qwen3_8b_layer_prefill_128x128_bf16"
Q4096 = "qwen3_8b_layer_prefill_4096x4096_bf16"
EPS = 1e-6


def kdir(workload, idx):
    """The kernel directory `idx` (two digits) of a bundle workload."""
    base = os.path.join(V, workload)
    d = next(n for n in sorted(os.listdir(base)) if n.startswith(f"{idx:02d}_"))
    return os.path.join(base, d)


def spec_file(workload, idx):
    d = kdir(workload, idx)
    return os.path.join(d, next(f for f in os.listdir(d) if f.endswith("_spec.py")))


def qwen_cases(wl, T, tag, golden):
    """The 12 kernels of a Qwen3-8B prefill layer workload (manifest.json launches), with the oracle program
    each restates (parameters from the kernel sources: hidden 4096, 32 q / 8 kv heads of 128, SiLU
    intermediate 12288, eps 1e-6 -- e.g. qwen3_8b_layer_prefill_2048x2048_bf16/00_*_triton.py xnumel/r0_numel,
    09_*: N = 24576)."""
    H, HQ, HKV, D, I = 4096, 32, 8, 128, 12288
    return [
        (f"{tag}_00_rmsnorm", spec_file(wl, 0), {"family": "rmsnorm_rows", "rows": T, "cols": H, "eps": EPS}, golden),
        (f"{tag}_01_q_mm", spec_file(wl, 1), {"family": "gemm", "M": T, "N": HQ * D, "K": H, "residual": False}, golden),
        (f"{tag}_02_qnorm_rope", spec_file(wl, 2), {"family": "qknorm_rope", "tokens": T, "heads": HQ, "eps": EPS}, golden),
        (f"{tag}_03_kv_mm", spec_file(wl, 3), {"family": "gemm", "M": T, "N": HKV * D, "K": H, "residual": False}, golden),
        (f"{tag}_04_knorm_rope", spec_file(wl, 4), {"family": "qknorm_rope", "tokens": T, "heads": HKV, "eps": EPS}, golden),
        (f"{tag}_05_v_relayout", spec_file(wl, 5), {"family": "token_to_head_major", "tokens": T, "heads": HKV, "dim": D}, golden),
        (f"{tag}_06_attention", spec_file(wl, 6), {"family": "attention_prefill", "batch": 1, "hq": HQ, "g": HQ // HKV,
                                                   "seq": T, "dim": D, "causal": True, "scale": 1 / math.sqrt(D)}, golden),
        (f"{tag}_07_o_relayout", spec_file(wl, 7), {"family": "heads_to_token_major", "tokens": T, "heads": HQ, "dim": D}, golden),
        (f"{tag}_08_o_mm_residual", spec_file(wl, 8), {"family": "gemm", "M": T, "N": H, "K": HQ * D, "residual": True}, golden),
        (f"{tag}_09_gate_up_mm", spec_file(wl, 9), {"family": "gemm", "M": T, "N": 2 * I, "K": H, "residual": False}, golden),
        (f"{tag}_10_silu_mul", spec_file(wl, 10), {"family": "silu_mul", "tokens": T, "inter": I}, golden),
        (f"{tag}_11_down_mm_residual", spec_file(wl, 11), {"family": "gemm", "M": T, "N": H, "K": I, "residual": True}, golden),
    ]


def add_config(spec):
    """tests/cases/smoke/add.py at BASELINE.json configs[0]: x, y fp32 of 1,048,576, BLOCK_SIZE 1024."""
    from pytorchsim_triton_compiler.contract.kernel_spec import Arg
    n, blk = 1_048_576, 1024
    s = copy.copy(spec)
    s.constexprs = {"n": n, "BLOCK": blk}
    s.args = [Arg(a.name, a.role, a.dtype, (n,)) for a in spec.args]
    s.grid = (n // blk,)
    return s


def attention_batch4(spec):
    """The bundle's attention_prefill_32x8x4096_bf16 kernel at BASELINE.json's batch 4 (its program index
    decodes b = pid // HQ, _prefill_kernel_triton.py:7-11): q/o of 4x the elements, grid 4 x 32."""
    from pytorchsim_triton_compiler.contract.kernel_spec import Arg
    s = copy.copy(spec)
    s.args = [Arg(a.name, a.role, a.dtype, (a.numel * 4,)) for a in spec.args]
    s.grid = (4 * spec.grid[0], 1, 1)
    return s


def cases():
    out = [
        ("smoke_add_1024", os.path.join(REF, "tests", "cases", "smoke", "add.py"), {"family": "vector_add"}, True),
        ("vector_add_1m", os.path.join(REF, "tests", "cases", "smoke", "add.py"), {"family": "vector_add", "modify": "add_config"}, False),
        ("vector_add1_8x128", spec_file("vector_add1_8x128_bf16", 0), {"family": "add_one"}, True),
        ("vector_add1_4096x4096", spec_file("vector_add1_4096x4096_bf16", 0), {"family": "add_one"}, False),
        ("vector_slice_8x128", spec_file("vector_slice_8x128_bf16", 0), {"family": "slice_add_one"}, True),
        ("vector_sum_8x128", spec_file("vector_sum_8x128_bf16", 0), {"family": "reduce_all", "op": "sum"}, True),
        ("vector_max_8x128", spec_file("vector_max_8x128_bf16", 0), {"family": "reduce_all", "op": "max"}, True),
        ("vector_sum_4096x4096", spec_file("vector_sum_4096x4096_bf16", 0), {"family": "reduce_all", "op": "sum"}, False),
        ("vector_max_4096x4096", spec_file("vector_max_4096x4096_bf16", 0), {"family": "reduce_all", "op": "max"}, False),
        ("softmax_32x128", spec_file("vector_softmax_32x128_bf16", 0), {"family": "softmax_rows", "rows": 32, "cols": 128}, True),
        ("softmax_128x1536", spec_file("vector_softmax_128x1536_bf16", 0), {"family": "softmax_rows", "rows": 128, "cols": 1536}, True),
        ("softmax_4096x4096", spec_file("vector_softmax_4096x4096_bf16", 0), {"family": "softmax_rows", "rows": 4096, "cols": 4096}, False),
        ("rmsnorm_4096x4096", spec_file(Q4096, 0), {"family": "rmsnorm_rows", "rows": 4096, "cols": 4096, "eps": EPS}, False),
        ("gemm_32x768x768", spec_file("gemm_32x768x768_bf16", 0), {"family": "gemm", "M": 32, "N": 768, "K": 768, "residual": False}, True),
        ("gemm_128x768x768", spec_file("gemm_128x768x768_bf16", 0), {"family": "gemm", "M": 128, "N": 768, "K": 768, "residual": False}, True),
        ("attention_16x8x128", spec_file("attention_prefill_16x8x128_bf16", 0),
         {"family": "attention_prefill", "batch": 1, "hq": 16, "g": 2, "seq": 128, "dim": 128, "causal": True,
          "scale": 1 / math.sqrt(128)}, True),
        ("attention_32x8x4096_b4", spec_file("attention_prefill_32x8x4096_bf16", 0),
         {"family": "attention_prefill", "batch": 4, "hq": 32, "g": 4, "seq": 4096, "dim": 128, "causal": True,
          "scale": 1 / math.sqrt(128), "modify": "attention_batch4"}, False),
    ]
    # Decode attention (SCALE 1/sqrt(128), GP 16, BKV = S in every bundle workload) and the M = 1 matmul
    # (gemm_1xKxN: a multiply-reduce program, out[x] = sum_r in0[r] * in1[x + N r]).
    for hq, s, gold in ((16, 128, True), (64, 512, True), (32, 4096, True), (32, 8192, False)):
        g = hq // 8
        out.append((f"attention_decode_{hq}x8x{s}", spec_file(f"attention_decode_{hq}x8x{s}_bf16", 0),
                    {"family": "attention_decode", "hkv": 8, "g": g, "gp": 16, "seq": s, "dim": 128, "bkv": s,
                     "scale": 1 / math.sqrt(128)}, gold))
    for k, n, gold in ((384, 1152, True), (768, 768, True), (2048, 2048, True), (4096, 4096, False), (4096, 2048, False)):
        out.append((f"gemm_1x{k}x{n}", spec_file(f"gemm_1x{k}x{n}_bf16", 0),
                    {"family": "gemm", "M": 1, "N": n, "K": k, "residual": False}, gold))
    # MoE routing ops (Qwen3-30B-A3B layer ops: 128 experts, top-8, hidden 2048).
    for T, gold in ((1, True), (128, True), (4096, False)):
        rp, dp = f"layer_op_router_post_{T}x0_bf16", f"layer_op_dispatch_{T}x0_bf16"
        out += [
            (f"moe_router_t{T}_00_softmax", spec_file(rp, 0),
             {"family": "softmax_rows", "rows": T, "cols": 128, "out_dtype": "float32"}, gold),
            (f"moe_router_t{T}_01_topk", spec_file(rp, 1),
             {"family": "topk", "rows": T, "cols": 128, "cols_padded": 128, "k": 8, "largest": True}, gold),
            (f"moe_router_t{T}_02_normalise", spec_file(rp, 2), {"family": "row_divsum", "rows": T, "cols": 8}, gold),
            (f"moe_dispatch_t{T}_00_sort", spec_file(dp, 0),
             {"family": "sort", "rows": 1, "cols": 8 * T, "descending": False, "float_keys": False}, gold),
            (f"moe_dispatch_t{T}_01_gather", spec_file(dp, 1),
             {"family": "dispatch_gather", "tokens": T, "hidden": 2048, "topk": 8}, gold),
            (f"moe_combine_t{T}_03_weighted", spec_file(f"layer_op_combine_{T}x0_bf16", 3),
             {"family": "combine_weighted", "tokens": T, "hidden": 2048, "topk": 8, "experts": 128}, gold),
            # the combine's routing tables: per-expert counts and running counts over the 8T routed ids
            # (00), their running sum (01), each routed row's slot within its expert (02)
            (f"moe_combine_t{T}_00_counts", spec_file(f"layer_op_combine_{T}x0_bf16", 0),
             {"family": "expert_counts", "experts": 128, "n": 8 * T}, gold),
            (f"moe_combine_t{T}_02_slot", spec_file(f"layer_op_combine_{T}x0_bf16", 2),
             {"family": "slot_of", "experts": 128, "n": 8 * T}, gold),
        ]
    # the grouped matmul's group tables over the 128 experts (the same three programs at every T):
    # running offsets (01), previous offset / count / running non-empty groups (02), groups at or below each
    # expert (03); and the combine's int64 running sum of the expert counts (01)
    gu = "layer_op_gmm_gate_up_128x0_bf16"
    out += [
        ("moe_gmm_01_offsets", spec_file(gu, 1), {"family": "cumsum_int", "n": 128}, True),
        ("moe_gmm_02_group_tables", spec_file(gu, 2), {"family": "group_tables", "n": 128}, True),
        ("moe_gmm_03_count_le", spec_file(gu, 3), {"family": "count_le", "n": 128, "rows": 128}, True),
        ("moe_combine_01_offsets", spec_file("layer_op_combine_128x0_bf16", 1), {"family": "cumsum_int", "n": 128}, True),
    ]
    # The MoE expert matmul: the reference kernel at an interpreter-sized configuration (golden), and the
    # bundle's T = 1 and 128 objects (gate_up K 2048 -> N 1536, down K 768 -> N 2048; 128 experts; the group
    # tables of the recorded routing are kept as input fixtures).
    out.append(("moe_gmm_small", spec_file("layer_op_gmm_gate_up_1x0_bf16", 5),
                {"family": "grouped_gemm", "M": 210, "N": 96, "K": 64, "groups": 6, "modify": "gmm_small"}, True))
    for T in (1, 128):
        out.append((f"moe_gmm_gate_up_t{T}", spec_file(f"layer_op_gmm_gate_up_{T}x0_bf16", 5),
                    {"family": "grouped_gemm", "M": 8 * T, "N": 1536, "K": 2048, "groups": 128}, False))
        out.append((f"moe_gmm_down_t{T}", spec_file(f"layer_op_gmm_down_{T}x0_bf16", 5),
                    {"family": "grouped_gemm", "M": 8 * T, "N": 2048, "K": 768, "groups": 128}, False))
    # The Qwen3-8B decode layer's fused programs (T = 1, context 128; hidden 4096): the sums of squares of the
    # two RMSNorms (00; 05 over the residual sum) and the matrix-vector products with the RMSNorm'd vector
    # (01: q 4096 -> 4096; 06: residual sum, gate_up 4096 -> 24576) or the SiLU'd vector and two residual rows
    # (07: down 12288 -> 4096).
    dw = "qwen3_8b_layer_decode_1x128_bf16"
    out += [
        ("qwen3_decode_00_sumsq", spec_file(dw, 0), {"family": "sumsq", "n": 4096}, True),
        ("qwen3_decode_01_rmsnorm_q_mm", spec_file(dw, 1),
         {"family": "rmsnorm_gemv", "K": 4096, "N": 4096, "eps": EPS}, True),
        ("qwen3_decode_05_sumsq_residual", spec_file(dw, 5), {"family": "sumsq", "n": 4096}, True),
        ("qwen3_decode_06_rmsnorm_gate_up_mm", spec_file(dw, 6),
         {"family": "rmsnorm_gemv", "K": 4096, "N": 24576, "eps": EPS, "residual": True}, True),
        ("qwen3_decode_07_silu_down_mm", spec_file(dw, 7), {"family": "silu_gemv", "K": 12288, "N": 4096}, True),
        ("qwen3_decode_02_qnorm_rope", spec_file(dw, 2),
         {"family": "qknorm_rope", "tokens": 1, "heads": 32, "eps": EPS, "inout_first": True}, True),
    ]
    # The whole Qwen3-8B decode layer at a 4096-token context (objects for the GPU parity run and the bench's
    # decode-layer step; the oracle checks them, the weights are too large for committed vectors).
    d4 = "qwen3_8b_layer_decode_1x4096_bf16"
    out += [
        ("qwen3_decode_s4096_00_sumsq", spec_file(d4, 0), {"family": "sumsq", "n": 4096}, False),
        ("qwen3_decode_s4096_01_rmsnorm_q_mm", spec_file(d4, 1),
         {"family": "rmsnorm_gemv", "K": 4096, "N": 4096, "eps": EPS}, False),
        ("qwen3_decode_s4096_02_qnorm_rope", spec_file(d4, 2),
         {"family": "qknorm_rope", "tokens": 1, "heads": 32, "eps": EPS, "inout_first": True}, False),
        ("qwen3_decode_s4096_03_attention", spec_file(d4, 3),
         {"family": "attention_decode", "hkv": 8, "g": 4, "gp": 16, "seq": 4096, "dim": 128, "bkv": 4096,
          "scale": 1 / math.sqrt(128)}, False),
        ("qwen3_decode_s4096_04_o_mm", spec_file(d4, 4), {"family": "gemm", "M": 1, "N": 4096, "K": 4096, "residual": False},
         False),
        ("qwen3_decode_s4096_05_sumsq_residual", spec_file(d4, 5), {"family": "sumsq", "n": 4096}, False),
        ("qwen3_decode_s4096_06_rmsnorm_gate_up_mm", spec_file(d4, 6),
         {"family": "rmsnorm_gemv", "K": 4096, "N": 24576, "eps": EPS, "residual": True}, False),
        ("qwen3_decode_s4096_07_silu_down_mm", spec_file(d4, 7), {"family": "silu_gemv", "K": 12288, "N": 4096}, False),
    ]
    # The Qwen3-30B-A3B MoE layer's own fused programs (hidden 2048, 128 experts, top-8): the combine with
    # renormalised weights and the residual stream (decode 23 at T = 1, prefill 27 at T = 128), the RMSNorm
    # of the residual sum (prefill 18), the per-token weight sums (prefill 22), the rotary embedding layer ops
    # (32 q / 4 k heads of 128) and the one-token RMSNorm layer op.
    ld, lp = "layer_layer_decode_1x128_bf16", "layer_layer_prefill_128x128_bf16"
    out += [
        ("moe_layer_decode_23_combine", spec_file(ld, 23),
         {"family": "combine_weighted_fused", "tokens": 1, "hidden": 2048, "topk": 8, "experts": 128}, True),
        ("moe_layer_prefill_27_combine", spec_file(lp, 27),
         {"family": "combine_weighted_fused", "tokens": 128, "hidden": 2048, "topk": 8, "experts": 128}, True),
        ("moe_layer_prefill_18_rmsnorm_residual", spec_file(lp, 18),
         {"family": "rmsnorm_rows", "rows": 128, "cols": 2048, "eps": EPS, "residual": True}, True),
        ("moe_layer_prefill_22_weight_sum", spec_file(lp, 22), {"family": "row_sum", "rows": 128, "cols": 8}, True),
        ("moe_rope_q_t128", spec_file("layer_op_rope_q_128x0_bf16", 0), {"family": "rope_rows", "tokens": 128, "heads": 32}, True),
        ("moe_rope_k_t128", spec_file("layer_op_rope_k_128x0_bf16", 0), {"family": "rope_rows", "tokens": 128, "heads": 4}, True),
        ("moe_rope_q_t1", spec_file("layer_op_rope_q_1x0_bf16", 0), {"family": "rope_rows", "tokens": 1, "heads": 32}, True),
        ("moe_rmsnorm_t1", spec_file("layer_op_rmsnorm_1x0_bf16", 0),
         {"family": "rmsnorm_rows", "rows": 1, "cols": 2048, "eps": EPS}, True),
    ]
    for m in (128, 512, 2048, 4096, 8192):
        out.append((f"gemm_{m}x4096x4096", spec_file(f"gemm_{m}x4096x4096_bf16", 0),
                    {"family": "gemm", "M": m, "N": 4096, "K": 4096, "residual": False}, False))
    out += qwen_cases(Q128, 128, "qwen3_t128", True)
    out += qwen_cases(Q2048, 2048, "qwen3_t2048", False)
    return out


def gmm_small(spec):
    """The bundle's _grouped_mm_kernel source (layer_op_gmm_gate_up_*/05__grouped_mm_kernel) at a size the
    interpreter runs: 6 groups of K = 64 x N = 96 weights plus the empty entry, 210 rows of which group 4's 10
    are listed by no program (their output rows must keep their values), one group of 130 rows (two 128-row
    tiles), empty groups; the tile constants of the bundle (BM 128, BN 2048 masked to N, BK = KP = K)."""
    from pytorchsim_triton_compiler.contract.kernel_spec import Arg
    G, M, K, N = 6, 210, 64, 96
    rows = [0, 37, 130, 1, 10, 32, 0]
    start = [sum(rows[:i]) for i in range(G + 1)]
    group = [1, 2, 3, 5, 6, 6]          # the groups with rows, then the empty entry; group 4 is not listed
    s = copy.copy(spec)
    s.constexprs = dict(spec.constexprs, sbg=K * N, sbk=N, sbn=1, K=K, KP=K, N=N, BK=K)
    s.args = [Arg("a_ptr", "in", "bfloat16", (M * K,)), Arg("b_ptr", "in", "bfloat16", (G * K * N,)),
              Arg("group_ptr", "in", "int32", (len(group),)), Arg("start_ptr", "in", "int32", (G + 1,)),
              Arg("rows_ptr", "in", "int32", (G + 1,)), Arg("c_ptr", "inout", "bfloat16", (M * N,))]
    s.grid = (len(group), 1, 1)

    def make_inputs(torch, seed=0):
        g = torch.Generator().manual_seed(seed)
        return {"a_ptr": torch.randn(M * K, generator=g).to(torch.bfloat16),
                "b_ptr": torch.randn(G * K * N, generator=g).to(torch.bfloat16),
                "group_ptr": torch.tensor(group, dtype=torch.int32), "start_ptr": torch.tensor(start, dtype=torch.int32),
                "rows_ptr": torch.tensor(rows, dtype=torch.int32),
                "c_ptr": torch.randn(M * N, generator=g).to(torch.bfloat16)}
    s.make_inputs = make_inputs
    return s


MODIFY = {"add_config": add_config, "attention_batch4": attention_batch4, "gmm_small": gmm_small}

# ---------------------------------------------------------------------------------------------------
# Triton interpreter shims
# ---------------------------------------------------------------------------------------------------


def install_interpreter_shims():
    import numpy as np
    import triton._utils as tu
    import triton.language.core as tc
    from triton.runtime import interpreter as I
    tu.TRITON_MAX_TENSOR_NUMEL = 1 << 40
    tc.TRITON_MAX_TENSOR_NUMEL = 1 << 40
    orig = I.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        def widen(h):
            if str(h.dtype.scalar) == "bf16":
                return I.TensorHandle((h.data.astype(np.uint32) << 16).view(np.float32), I.tl.float32)
            return h
        return orig(self, widen(a), widen(b), d, input_precision, max_num_imprecise_acc)

    I.InterpreterBuilder.create_dot = create_dot

    def to_bf16_rne(data):
        b = np.ascontiguousarray(data, dtype=np.float32).view(np.uint32).astype(np.uint64)
        r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
        nan = np.isnan(np.ascontiguousarray(data, dtype=np.float32))
        return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)

    orig_cast = I.InterpreterBuilder.cast_impl

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == I.tl.float32 and dst_type.scalar == I.tl.bfloat16:
            return I.TensorHandle(to_bf16_rne(src.data), dst_type.scalar)
        return orig_cast(self, src, dst_type)

    I.InterpreterBuilder.cast_impl = cast_impl
    for name in ("create_fp_ext", "create_fp_trunc"):
        setattr(I.InterpreterBuilder, name, lambda self, src, dst_type: self.cast_impl(src, dst_type))
    orig_fp_to_fp = I.InterpreterBuilder.create_fp_to_fp

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar == I.tl.float32 and dst_type.scalar == I.tl.bfloat16:
            return I.TensorHandle(to_bf16_rne(src.data), dst_type.scalar)
        return orig_fp_to_fp(self, src, dst_type, rounding_mode)

    I.InterpreterBuilder.create_fp_to_fp = create_fp_to_fp


class _Libdevice:
    """libdevice.<fn> of Inductor kernels routed to the interpreter's tl.<fn>."""

    def __getattr__(self, name):
        import triton.language as tl
        return getattr(tl, name)


def interpret(spec, inputs):
    """Run `spec`'s kernel under the Triton interpreter over copies of `inputs`; return every written arg."""
    import torch
    import triton
    from pytorchsim_triton_compiler.targets.b200.frontend import load_kernel
    fn = load_kernel(spec)
    while hasattr(fn, "fn") and not isinstance(fn, triton.runtime.interpreter.InterpretedFunction):
        fn = fn.fn
    inner = getattr(fn, "fn", fn)
    if "libdevice" in getattr(inner, "__globals__", {}):
        inner.__globals__["libdevice"] = _Libdevice()
    tens = []
    for a in spec.args:
        if a.name in inputs:
            tens.append(inputs[a.name].clone())
        else:
            tens.append(torch.zeros(a.shape, dtype=getattr(torch, a.dtype)))
    scal = spec.extra.get("scalar_values", {})
    kw = {}
    ti = 0
    for n, s in spec.signature.items():
        if n in spec.constexprs:
            kw[n] = spec.constexprs[n]
        elif s == "constexpr":
            continue
        elif s.startswith("*"):
            kw[n] = tens[ti]
            ti += 1
        else:
            kw[n] = scal.get(n, 0)
    fn[tuple(spec.grid)](**kw)
    return {a.name: t for a, t in zip(spec.args, tens) if a.role in ("out", "inout")}


def convention_inputs(spec, skip, given):
    """The input convention (one generator seeded 0, randn per read argument in order, cast to its dtype),
    with the arguments in `skip` taken from `given` and drawing nothing."""
    import torch
    g = torch.Generator().manual_seed(0)
    out = {}
    for a in spec.args:
        if a.role not in ("in", "inout"):
            continue
        out[a.name] = given[a.name] if a.name in skip else torch.randn(a.numel, generator=g).to(getattr(torch, a.dtype))
    return out


def recorded_args(spec, inputs):
    """The read arguments the spec's make_inputs does not draw (loaded from a recording): grown one at a time
    until every other argument matches the convention exactly."""
    import torch
    skip = []
    while True:
        conv = convention_inputs(spec, set(skip), inputs)
        diff = [n for n in inputs if not torch.equal(conv[n].reshape(-1), inputs[n].reshape(-1))]
        new = [n for n in diff if n not in skip]
        if not new:
            return skip
        skip.append(new[0])


def bits(t):
    import torch
    t = t.contiguous()
    return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def main():
    import numpy as np
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--no-golden", action="store_true")
    opts = ap.parse_args()
    from pytorchsim_triton_compiler.contract import kernel_object as ko
    from pytorchsim_triton_compiler.contract.kernel_spec import load_spec
    from pytorchsim_triton_compiler.targets.b200 import lower as L
    install_interpreter_shims()
    objdir, vecdir = os.path.join(HERE, "objects"), os.path.join(HERE, "vectors")
    os.makedirs(objdir, exist_ok=True)
    os.makedirs(vecdir, exist_ok=True)
    index = []
    for name, path, oracle, golden in cases():
        if opts.only and opts.only != name:
            continue
        spec = load_spec(path)
        modified = oracle.pop("modify", None)
        if modified:
            spec = MODIFY[modified](spec)
        lowered = L.lower(spec)
        d = os.path.join(objdir, name)
        shutil.rmtree(d, ignore_errors=True)
        ko.write(d, spec, lowered.summary, lowered.blob)
        gen = [{"name": a.name, "role": a.role, "dtype": a.dtype, "numel": a.numel} for a in spec.args]
        reads = [a.name for a in spec.args if a.role in ("in", "inout")]
        case = {"name": name, "source": os.path.relpath(path, REF), "kind": lowered.kind, "args": gen,
                "inputs": reads, "oracle": oracle, "golden": None}
        if modified:
            case["modified"] = modified   # the spec was resized from the reference's (MODIFY[modified])
        if not golden and spec.make_inputs is not None and any(a.dtype.startswith("int") for a in spec.args
                                                                  if a.role in ("in", "inout")):
            # integer inputs (routing tables) of a case without output vectors: keep the recorded ones
            inputs = spec.make_inputs(torch, seed=0)
            recorded = recorded_args(spec, inputs)
            if recorded:
                np.savez_compressed(os.path.join(vecdir, f"{name}__inputs.npz"),
                                    **{a: inputs[a].contiguous().numpy() for a in recorded})
                case["recorded"] = {"file": f"vectors/{name}__inputs.npz", "args": recorded}
            del inputs
        if golden and not opts.no_golden:
            g = torch.Generator().manual_seed(0)
            if spec.make_inputs is None:
                raise SystemExit(f"{name}: no make_inputs")
            inputs = spec.make_inputs(torch, seed=0)
            if list(inputs) != reads:
                raise SystemExit(f"{name}: make_inputs builds {list(inputs)}, the read arguments are {reads}")
            recorded = recorded_args(spec, inputs)
            if recorded:
                # Arguments the spec loads from a recording beside it (routing indices of a model run): kept as
                # a fixture; they consume no random draw, so the other arguments still follow the convention.
                np.savez_compressed(os.path.join(vecdir, f"{name}__inputs.npz"),
                                    **{a: inputs[a].contiguous().numpy() for a in recorded})
                case["recorded"] = {"file": f"vectors/{name}__inputs.npz", "args": recorded}
            outs = interpret(spec, inputs)
            payload = {}
            for k, t in outs.items():
                flat = t.reshape(-1)
                full = bits(flat)
                payload[f"{k}__sha256"] = np.frombuffer(hashlib.sha256(full.tobytes()).digest(), dtype=np.uint8)
                if flat.numel() > 8192:
                    stride = -(-flat.numel() // 8192)
                    payload[f"{k}__stride"] = np.array([stride], dtype=np.int64)
                    payload[k] = full[::stride].copy()
                else:
                    payload[f"{k}__stride"] = np.array([1], dtype=np.int64)
                    payload[k] = full
            np.savez_compressed(os.path.join(vecdir, f"{name}.npz"), **payload)
            case["golden"] = f"vectors/{name}.npz"
        with open(os.path.join(d, "case.json"), "w") as fh:
            json.dump(case, fh, indent=1)
            fh.write("\n")
        index.append(name)
        print(f"{name:32s} {lowered.kind:12s} golden={'yes' if case['golden'] else 'no'}", flush=True)
    if not opts.only:
        with open(os.path.join(HERE, "index.json"), "w") as fh:
            json.dump(index, fh, indent=1)
            fh.write("\n")


if __name__ == "__main__":
    main()
