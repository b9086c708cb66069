"""The bounded-wait (timeout) path of every pipelined kernel family, on the GPU, without a GPU fault.

A launch whose descriptor carries PTSIM_FLAG_TEST_STALL has its first CTA (or cluster) arm one pipeline
stage and issue none of that stage's copies, and gives every mbarrier wait a 1 ms limit: the waits on that
stage give up, the kernel records PTSIM_E_TIMEOUT and every CTA unwinds (copies in flight land, issued MMAs
drain, TMEM is freed, cluster barriers are all met).  Each test checks that

  - the stalled launch returns within seconds and ptsim_sync reports PTSIM_E_TIMEOUT (202), the GPU
    analogue of a program ending in one of Spike's named traps (runtime/spike.py:12,36-41 in the
    reference);
  - the status word is cleared by that report (the next sync reports nothing);
  - the same descriptor launched again without the flag, on the same device and buffers, still meets its
    parity bar against the CPU oracle.

Families: the one-CTA tcgen05 GEMM, its split-K cluster form (the exchange is skipped by every CTA of a
cluster in which one gave up), the 2-CTA pair GEMM, both attention kernels, decode attention and the
bulk-copy GEMV."""
import math
import time

import pytest
import torch

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.runtime import cuda as RC
from pytorchsim_triton_compiler.runtime import native
from oracle import programs as O
from oracle.tolerance import ATTENTION, CONTRACTION
from tests._helpers import parity

pytestmark = pytest.mark.gpu

TIMEOUT = 202   # PTSIM_E_TIMEOUT


def _gemm_inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    std = 1.0 / math.sqrt(K)
    a = (torch.randn(M * K, generator=g) * std).to(torch.bfloat16)
    b = (torch.randn(K * N, generator=g) * std).to(torch.bfloat16)
    return [a, b, torch.zeros(M * N, dtype=torch.bfloat16)]


def _attn_inputs(batch, hq, hkv, seq, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch * hq * seq * 128, generator=g).to(torch.bfloat16)
    k = torch.randn(batch * hkv * seq * 128, generator=g).to(torch.bfloat16)
    v = torch.randn(batch * hkv * seq * 128, generator=g).to(torch.bfloat16)
    return [q, k, v, torch.zeros_like(q)]


def _decode_inputs(hkv, group, seq, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(hkv * group * 128, generator=g).to(torch.bfloat16)
    k = torch.randn(hkv * seq * 128, generator=g).to(torch.bfloat16)
    v = torch.randn(hkv * seq * 128, generator=g).to(torch.bfloat16)
    return [q, k, v, torch.zeros_like(q)]


def _check_gemm(M, N, K):
    def check(ins, out):
        parity(out, O.gemm(ins[0], ins[1], M, N, K), CONTRACTION, row=N, name=f"gemm {M}x{N}x{K} after a timeout")
    return check


def _check_attention(batch, hq, hkv, seq):
    def check(ins, out):
        want = O.attention_prefill(ins[0], ins[1], ins[2], batch, hq, hq // hkv, seq, 128, min(1024, seq),
                                   min(1024, seq), True, 1 / math.sqrt(128))
        parity(out, want, ATTENTION, row=128, name=f"attention S={seq} after a timeout")
    return check


def _check_decode(hkv, group, seq):
    def check(ins, out):
        want = O.attention_decode(ins[0], ins[1], ins[2], torch.zeros_like(ins[3]), hkv, group, 16, seq, 128, seq,
                                  1 / math.sqrt(128))
        parity(out, want, ATTENTION, row=128, name=f"decode attention S={seq} after a timeout")
    return check


# (family, descriptor, inputs, the output's argument index, the parity check of a normal launch)
CASES = {
    # 2 x 8 tiles of 128 x 64 on one CTA each: no split, no pair
    "gemm": lambda: (B.gemm(256, 512, 256), _gemm_inputs(256, 512, 256, 1), 2, _check_gemm(256, 512, 256)),
    # one 128-row tile band over 4096 columns: split-K over thread-block clusters
    "gemm_splitk": lambda: (B.gemm(128, 4096, 4096), _gemm_inputs(128, 4096, 4096, 2), 2, _check_gemm(128, 4096, 4096)),
    # 9 x 16 tiles of 256 x 256: the 2-CTA pair kernel
    "gemm_pair": lambda: (B.gemm(2304, 4096, 512), _gemm_inputs(2304, 4096, 512, 3), 2, _check_gemm(2304, 4096, 512)),
    # sequence a multiple of 256: two query tiles per CTA (register-split warpgroups)
    "attention": lambda: (B.attention(1, 4, 1, 512), _attn_inputs(1, 4, 1, 512, 4), 3, _check_attention(1, 4, 1, 512)),
    # sequence 384: one query tile per CTA
    "attention_one_tile": lambda: (B.attention(1, 2, 1, 384), _attn_inputs(1, 2, 1, 384, 5), 3,
                                   _check_attention(1, 2, 1, 384)),
    "decode": lambda: (B.attention_decode(2, 4, 4096), _decode_inputs(2, 4, 4096, 6), 3, _check_decode(2, 4, 4096)),
    # 8192 x 4096 matrix (32 Mi elements): the bulk-copy ring and its reduce
    "gemv_bulk": lambda: (B.gemv(4096, 8192), _gemm_inputs(1, 4096, 8192, 7), 2, _check_gemm(1, 4096, 8192)),
}


@pytest.mark.parametrize("family", list(CASES))
def test_stalled_stage_times_out_and_device_stays_usable(family):
    desc, ins, out_arg, check = CASES[family]()
    dev = torch.device("cuda", 0)
    ts = [t.to(dev) for t in ins]
    stream = torch.cuda.current_stream(dev)
    ws_n = native.workspace_size(D.to_bytes(desc), 0)
    ws = torch.empty(max(1, ws_n), dtype=torch.uint8, device=dev)
    native.init(0)
    native.sync(stream.cuda_stream)             # nothing pending before the test

    stalled = D.from_bytes(D.to_bytes(desc))
    stalled.flags |= D.FLAG_TEST_STALL
    blob = D.to_bytes(stalled)
    t0 = time.perf_counter()
    native.launch(blob, [t.data_ptr() for t in ts], 0, stalled.units, ws.data_ptr(), ws_n, stream.cuda_stream)
    with pytest.raises(native.ExecutorError) as err:
        native.sync(stream.cuda_stream)
    took = time.perf_counter() - t0
    assert err.value.code == TIMEOUT, f"{family}: the stalled launch reported {err.value.code}, not PTSIM_E_TIMEOUT"
    # 1 ms limits: a few serial waits, far below one 2 s default limit
    assert took < 1.5, f"{family}: the stalled launch took {took:.2f} s; the test limit was not in effect"
    native.sync(stream.cuda_stream)             # the report cleared the status word

    # The same launch without the flag, on the same device and buffers, meets its bar.
    ts[out_arg].zero_()
    blob = D.to_bytes(desc)
    native.launch(blob, [t.data_ptr() for t in ts], 0, desc.units, ws.data_ptr(), ws_n, stream.cuda_stream)
    native.sync(stream.cuda_stream)
    check(ins, ts[out_arg].cpu())
