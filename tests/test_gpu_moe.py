"""The MoE routing programs on the B200 against the CPU oracle (the Qwen3-30B-A3B layer ops of the bundle):
top-k selection and row sorts are bit exact (values are copies, indices integers); the row normalisation is
element-wise bf16 (1e-2 relative, no absolute floor, at most 2 ulps); the grouped GEMM and the combine's
weighted sums are bf16 sums of products (1e-2 relative plus 2^-10 of the row's RMS); the dispatch gather is a
bit-exact copy (bars: oracle/tolerance.py).  Edge cases follow the reference's
own rules: tied values go to the lowest column, -inf inputs make the top-k repeat an index, fp32 sort keys
order NaN last and -0 with +0, a gather row outside the table records PTSIM_E_OOB (the reference asserts)."""
import math

import pytest
import torch

from pytorchsim_triton_compiler.codegen import build as B
from pytorchsim_triton_compiler.codegen import descriptors as D
from pytorchsim_triton_compiler.runtime import cuda as RC
from pytorchsim_triton_compiler.runtime import native
from oracle import programs as O
from oracle.tolerance import CONTRACTION, FP32, POINTWISE
from tests._helpers import bits_equal, parity

pytestmark = pytest.mark.gpu


def run(desc, tensors):
    ts = [t.cuda() for t in tensors]
    RC.launch_tensors(D.to_bytes(desc), ts)
    return [t.cpu() for t in ts]


@pytest.mark.parametrize("rows,cols,padded,k,largest,dtype", [
    (4096, 128, 128, 8, True, "float32"), (1, 128, 128, 8, True, "float32"), (37, 100, 128, 5, False, "float32"),
    (64, 8, 8, 8, True, "float32"), (10, 1000, 1024, 3, True, "float32"), (300, 64, 64, 4, True, "bfloat16")])
def test_topk(rows, cols, padded, k, largest, dtype):
    g = torch.Generator().manual_seed(rows + cols)
    x = torch.randn(rows * cols, generator=g).to(getattr(torch, dtype))
    v, i = run(B.topk(rows, cols, k, largest, padded, dtype), [x, torch.zeros(rows * k, dtype=x.dtype),
                                                                torch.zeros(rows * k, dtype=torch.int64)])[1:]
    wv, wi = O.topk_rows(x, rows, cols, padded, k, largest)
    assert bits_equal(v, wv) and torch.equal(i, wi)


def test_topk_ties_and_spent_columns():
    """Equal values go to the lowest column; a row with fewer than k finite values takes the lowest spent
    column again (the reference keeps spent columns as candidates)."""
    rows, cols, k = 3, 16, 6
    x = torch.zeros(rows, cols)
    x[0] = torch.tensor([3.0, 1, 3, 2, 3, 0, 1, 2, 3, 3, 0, 0, 1, 2, 3, 3])
    x[1] = -math.inf
    x[1, 5], x[1, 9] = 1.0, 2.0
    x[2] = torch.arange(cols, dtype=torch.float32).flip(0)
    x = x.reshape(-1)
    v, i = run(B.topk(rows, cols, k), [x, torch.zeros(rows * k), torch.zeros(rows * k, dtype=torch.int64)])[1:]
    wv, wi = O.topk_rows(x, rows, cols, cols, k, True)
    assert bits_equal(v, wv) and torch.equal(i, wi)
    assert i.view(rows, k)[1].tolist() == [9, 5, 0, 0, 0, 0]


@pytest.mark.parametrize("rows,cols,lo,hi,desc", [
    (1, 32768, 0, 128, False), (1, 1024, -4, 5, False), (3, 5000, 0, 256, True), (2, 8192, -10**12, 10**12, False),
    (4, 777, -(1 << 62), 1 << 62, True), (1, 8, 0, 8, False), (5, 1, 0, 3, False)])
def test_sort_int_keys(rows, cols, lo, hi, desc):
    g = torch.Generator().manual_seed(cols)
    x = torch.randint(lo, hi, (rows * cols,), generator=g, dtype=torch.int64)
    v, i = run(B.sort(rows, cols, desc), [x, torch.zeros_like(x), torch.zeros_like(x)])[1:]
    wv, wi = O.sort_rows(x, rows, cols, desc)
    assert torch.equal(v, wv) and torch.equal(i, wi)


@pytest.mark.parametrize("desc", [False, True])
def test_sort_float_keys(desc):
    rows, cols = 2, 4000
    g = torch.Generator().manual_seed(3)
    x = torch.randn(rows * cols, generator=g)
    x[::97] = float("nan")
    x[5::101] = -0.0
    x[7::103] = 0.0
    x[11::107] = math.inf
    x[13::109] = -math.inf
    x[17::53] = 1.5      # ties
    v, i = run(B.sort(rows, cols, desc, float_keys=True, dtype="float32"), [x, torch.zeros_like(x),
                                                                             torch.zeros(rows * cols, dtype=torch.int64)])[1:]
    wv, wi = O.sort_rows(x, rows, cols, desc, float_keys=True)
    assert bits_equal(v, wv) and torch.equal(i, wi)


@pytest.mark.parametrize("rows,cols,lo,hi,desc", [(1, 32768, 0, 128, False), (3, 20000, -5, 200, True),
                                                  (2, 100000, 0, 256, False), (1, 8193, 7, 9, False),
                                                  (4, 65536, 0, 1, True)])
def test_sort_long_rows_over_ctas(rows, cols, lo, hi, desc):
    """Rows past the shared-memory sort: the stable counting sort over 1024-key chunks (ragged last chunks,
    several rows per launch, descending order, a span of exactly 256 values, one repeated key)."""
    g = torch.Generator().manual_seed(cols + rows)
    x = torch.randint(lo, hi, (rows * cols,), generator=g, dtype=torch.int64)
    v, i = run(B.sort(rows, cols, desc), [x, torch.zeros_like(x), torch.zeros_like(x)])[1:]
    wv, wi = O.sort_rows(x, rows, cols, desc)
    assert torch.equal(v, wv) and torch.equal(i, wi)


def test_sort_long_row_paths_agree():
    """Given no scratch, a long row runs the one-CTA counting sort; both paths give the same bits."""
    cols = 32768
    x = torch.randint(0, 128, (cols,), generator=torch.Generator().manual_seed(9), dtype=torch.int64).cuda()
    multi = [x, torch.zeros_like(x), torch.zeros_like(x)]
    RC.launch_tensors(D.to_bytes(B.sort(1, cols)), multi)
    single = [x, torch.zeros_like(x), torch.zeros_like(x)]
    stream = torch.cuda.current_stream()
    native.launch(D.to_bytes(B.sort(1, cols)), [t.data_ptr() for t in single], 0, 1, 0, 0, stream.cuda_stream)
    native.sync(stream.cuda_stream)
    assert torch.equal(multi[1], single[1]) and torch.equal(multi[2], single[2])


def test_sort_wide_long_row_is_reported():
    """A row longer than the shared-memory sort whose keys span more than the counting sort's 256 values is
    not run: the kernel records PTSIM_E_UNSUPPORTED, reported at synchronisation."""
    x = torch.arange(9000, dtype=torch.int64).flip(0) * 1000
    ts = [x.cuda(), torch.zeros_like(x).cuda(), torch.zeros_like(x).cuda()]
    with pytest.raises(native.ExecutorError) as e:
        RC.launch_tensors(D.to_bytes(B.sort(1, 9000)), ts)
    assert e.value.code == D.E_UNSUPPORTED


@pytest.mark.parametrize("rows,cols", [(4096, 8), (1, 8), (100, 33), (7, 1000)])
def test_row_divsum(rows, cols):
    g = torch.Generator().manual_seed(rows)
    x = torch.rand(rows * cols, generator=g) + 0.1
    out = run(B.row_divsum(rows, cols), [x, torch.zeros(rows * cols, dtype=torch.bfloat16)])[1]
    parity(out, O.row_divsum(x, rows, cols), POINTWISE, name=f"row_divsum {rows}x{cols}")


@pytest.mark.parametrize("rows,cols", [(4096, 8), (1, 8), (300, 33)])
def test_row_sum(rows, cols):
    """The MoE layer's per-token weight sums: fp32 row sums under the fp32 bar."""
    g = torch.Generator().manual_seed(rows + cols)
    x = torch.rand(rows * cols, generator=g)
    out = run(B.row_sum(rows, cols), [x, torch.zeros(rows)])[1]
    parity(out, O.row_sum(x, rows, cols), FP32, name=f"row_sum {rows}x{cols}")


@pytest.mark.parametrize("tokens,hidden,topk", [(4096, 2048, 8), (128, 2048, 8), (5, 64, 2), (300, 40, 3)])
def test_dispatch_gather(tokens, hidden, topk):
    rows = tokens * topk
    g = torch.Generator().manual_seed(tokens)
    pos = torch.randperm(rows, generator=g).to(torch.int64)
    pos[:: 7] -= rows          # negative positions: floor division then the wrap by + tokens
    table = torch.randn(tokens * hidden, generator=g).to(torch.bfloat16)
    d = B.gather_rows_floordiv(rows, hidden, tokens, topk)
    out = run(d, [pos, table, torch.zeros(rows * hidden, dtype=torch.bfloat16)])[2]
    assert bits_equal(out, O.dispatch_gather(pos, table, tokens, hidden, topk))


def test_dispatch_gather_out_of_range_is_recorded():
    tokens, hidden, topk = 16, 64, 2
    pos = torch.arange(tokens * topk, dtype=torch.int64)
    pos[3] = 10 * tokens * topk        # floor(pos / topk) >= tokens: outside the table
    table = torch.randn(tokens * hidden).to(torch.bfloat16)
    ts = [pos.cuda(), table.cuda(), torch.zeros(tokens * topk * hidden, dtype=torch.bfloat16).cuda()]
    with pytest.raises(native.ExecutorError) as e:
        RC.launch_tensors(D.to_bytes(B.gather_rows_floordiv(tokens * topk, hidden, tokens, topk)), ts)
    assert e.value.code == D.E_OOB


def _gmm_tables(sizes, listed, gen):
    """int32 group / start / rows tables for groups of the given row counts (plus the empty entry at the end);
    `listed`: the groups the programs take, padded to the table length with the empty entry."""
    G = len(sizes)
    rows = torch.tensor(list(sizes) + [0], dtype=torch.int32)
    start = torch.zeros(G + 1, dtype=torch.int32)
    start[1:] = torch.cumsum(rows[:-1], 0)
    start[G] = int(rows[:-1].sum())
    group = torch.tensor(list(listed) + [G] * (G - len(listed)), dtype=torch.int32)
    return group, start, rows


@pytest.mark.parametrize("T,K,N", [(512, 2048, 1536), (512, 768, 2048), (64, 64, 96), (300, 256, 200)])
def test_grouped_gemm(T, K, N):
    """Routing-shaped groups: 128 experts of 8 * T rows with uneven sizes (empty experts, experts longer than
    one 128-row tile); experts listed in order, one expert with rows left unlisted (its output rows keep
    their values)."""
    G, M = 128, 8 * T
    gen = torch.Generator().manual_seed(T + K)
    w = torch.rand(G, generator=gen) ** 3
    w[::9] = 0
    sizes = (w / w.sum() * M).floor().to(torch.int64)
    sizes[0] += M - int(sizes.sum())
    skip = int(torch.nonzero(sizes).flatten()[3])
    listed = [g for g in range(G) if sizes[g] > 0 and g != skip]
    group, start, rows = _gmm_tables(sizes.tolist(), listed, gen)
    std = 1.0 / math.sqrt(K)
    a = (torch.randn(M * K, generator=gen) * std).to(torch.bfloat16)
    b = (torch.randn(G * K * N, generator=gen) * std).to(torch.bfloat16)
    c = torch.randn(M * N, generator=gen).to(torch.bfloat16)
    out = run(B.grouped_gemm(M, N, K, G, G), [a, b, group, start, rows, c])[5]
    want = O.grouped_gemm(a, b, group, start, rows, c, M, N, K, G)
    s0, n0 = int(start[skip]), int(rows[skip])
    assert bits_equal(out.view(M, N)[s0:s0 + n0], c.view(M, N)[s0:s0 + n0])
    parity(out, want, CONTRACTION, row=N, name=f"grouped_gemm T={T} K={K} N={N}")


def test_grouped_gemm_bad_table_is_recorded():
    """A group id past the table records PTSIM_E_OOB; the program's rows are not touched."""
    G, M, K, N = 4, 64, 64, 64
    group, start, rows = _gmm_tables([16, 16, 16, 16], [0, 1, 2, 3], None)
    group[2] = 99
    ts = [torch.randn(M * K).to(torch.bfloat16), torch.randn(G * K * N).to(torch.bfloat16), group, start, rows,
          torch.zeros(M * N, dtype=torch.bfloat16)]
    ts = [t.cuda() for t in ts]
    with pytest.raises(native.ExecutorError) as e:
        RC.launch_tensors(D.to_bytes(B.grouped_gemm(M, N, K, G, G)), ts)
    assert e.value.code == D.E_OOB


def test_grouped_gemm_after_split_k_gemm():
    """A grouped launch after a split-K launch of the same GEMM kernel (whose occupancy query sets the kernel's
    shared-memory limit first) still gets room for its program table."""
    gemm = B.gemm(128, 4096, 4096)
    ts = [t.cuda() for t in (torch.zeros(128 * 4096, dtype=torch.bfloat16), torch.zeros(4096 * 4096, dtype=torch.bfloat16),
                             torch.zeros(128 * 4096, dtype=torch.bfloat16))]
    RC.launch_tensors(D.to_bytes(gemm), ts)
    test_grouped_gemm(64, 2048, 1536)


def moe_routing(tokens, topk, experts, seed):
    """A consistent routing: each (token, k) slot's expert id, the experts' counts and inclusive cumulative
    counts, and each slot's 1-based rank among the slots of its expert (so cum - cnt + pos - 1 is the slot's row
    in expert order)."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, experts, (tokens * topk,), generator=g)
    cnt = torch.bincount(ids, minlength=experts)
    cum = torch.cumsum(cnt, 0)
    order = torch.argsort(ids, stable=True)
    rank = torch.empty_like(ids)
    rank[order] = torch.arange(tokens * topk) - (cum - cnt)[ids[order]]
    return ids, cum, cnt, rank + 1


@pytest.mark.parametrize("tokens,hidden,topk,experts", [(4096, 2048, 8, 128), (128, 2048, 8, 128), (3, 64, 2, 4),
                                                        (100, 200, 4, 16)])
def test_combine_weighted(tokens, hidden, topk, experts):
    ids, cum, cnt, pos = moe_routing(tokens, topk, experts, tokens)
    ids[::5] -= experts                      # negative ids: wrapped by + experts
    g = torch.Generator().manual_seed(1)
    expert_out = torch.randn(tokens * topk * hidden, generator=g).to(torch.bfloat16)
    w = torch.rand(tokens * topk, generator=g).to(torch.bfloat16)
    ins = [ids, cum, cnt, pos, expert_out, w, torch.zeros(tokens * hidden, dtype=torch.bfloat16)]
    out = run(B.combine_gather_sum(tokens, hidden, topk, experts), ins)[6]
    want = O.combine_weighted(ids, cum, cnt, pos, expert_out, w, tokens, hidden, topk, experts)
    parity(out, want, CONTRACTION, row=hidden, name=f"combine T={tokens} hidden={hidden} topk={topk}")


@pytest.mark.parametrize("tokens,hidden", [(4096, 2048), (1, 2048), (37, 200)])
def test_combine_weighted_fused(tokens, hidden):
    """The MoE layer's combine: weights renormalised by each token's sum, the residual stream added."""
    topk, experts = 8, 128
    ids, cum, cnt, pos = moe_routing(tokens, topk, experts, tokens + 5)
    g = torch.Generator().manual_seed(2)
    expert_out = torch.randn(tokens * topk * hidden, generator=g).to(torch.bfloat16)
    w = torch.rand(tokens * topk, generator=g)
    wsum = w.view(tokens, topk).sum(dim=1)
    res = torch.randn(tokens * hidden, generator=g).to(torch.bfloat16)
    out0 = torch.randn(tokens * hidden, generator=g).to(torch.bfloat16)
    ins = [ids, cum, cnt, pos, expert_out, w, wsum, res, out0.clone()]
    got = run(B.combine_gather_sum(tokens, hidden, topk, experts, fused=True), ins)[8]
    want = O.combine_weighted_fused(ids, cum, cnt, pos, expert_out, w, wsum, res, out0, tokens, hidden, topk, experts)
    parity(got, want, CONTRACTION, row=hidden, name=f"combine fused T={tokens} hidden={hidden}")


def test_combine_out_of_range_is_recorded():
    tokens, hidden, topk, experts = 8, 64, 2, 4
    ids, cum, cnt, pos = moe_routing(tokens, topk, experts, 3)
    pos[5] += 1000                           # a slot past the expert-ordered rows
    ts = [ids, cum, cnt, pos, torch.randn(tokens * topk * hidden).to(torch.bfloat16),
          torch.rand(tokens * topk).to(torch.bfloat16), torch.zeros(tokens * hidden, dtype=torch.bfloat16)]
    ts = [t.cuda() for t in ts]
    with pytest.raises(native.ExecutorError) as e:
        RC.launch_tensors(D.to_bytes(B.combine_gather_sum(tokens, hidden, topk, experts)), ts)
    assert e.value.code == D.E_OOB


# ---- the routing tables (INT_TABLE): exact integer results ------------------------------------------------

def routed_ids(n, experts, seed, wild=False):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, experts, (n,), generator=g)
    if wild:                                  # ids no expert matches: negative and past the last expert
        ids[::7] = -1 - ids[::7]
        ids[3::11] += experts
    return ids


def interpreted(desc, on):
    """`desc` with PTSIM_FLAG_INTERPRET set when `on` (the element interpreter instead of a direct kernel)."""
    if on:
        desc.flags |= D.FLAG_INTERPRET
    return desc


@pytest.mark.parametrize("interp", [False, True], ids=["direct", "interpreter"])
@pytest.mark.parametrize("n,experts,wild", [(32768, 128, False), (1024, 128, True), (8, 128, False),
                                            (5000, 16, True), (100000, 3, False), (1, 1, False), (3000, 1000, True),
                                            (700, 45, True)])
def test_expert_counts(n, experts, wild, interp):
    """Counts and running counts: the direct one-hot kernels, and the interpreter's unsplit path (short
    routed range) and split one (a long range over few experts: chunk totals through the workspace)."""
    ids = routed_ids(n, experts, n, wild)
    cnt, run_ = run(interpreted(B.expert_counts(n, experts), interp),
                    [ids, torch.zeros(experts, dtype=torch.int64), torch.zeros(n * experts, dtype=torch.int64)])[1:]
    wc, wr = O.expert_counts(ids, experts, n)
    assert torch.equal(cnt, wc) and torch.equal(run_, wr)


@pytest.mark.parametrize("n,in_dtype,out_dtype", [(128, "int32", "int32"), (128, "int64", "int64"),
                                                  (100000, "int64", "int64"), (3, "int32", "int64"),
                                                  (70000, "int32", "int32")])
def test_cumsum_int(n, in_dtype, out_dtype):
    g = torch.Generator().manual_seed(n)
    x = torch.randint(-1000, 100000, (n,), generator=g).to(getattr(torch, in_dtype))
    if in_dtype == "int32" and n > 1000:
        x[::3] = 2**31 - 5                    # the int32 running sum wraps, as the reference's int32 scan does
    got = run(B.cumsum_int(n, in_dtype, out_dtype), [x, torch.zeros(n, dtype=getattr(torch, out_dtype))])[1]
    assert torch.equal(got, O.cumsum_int(x, n, getattr(torch, out_dtype)))


@pytest.mark.parametrize("interp", [False, True], ids=["direct", "interpreter"])
@pytest.mark.parametrize("n,experts", [(32768, 128), (8, 128), (3000, 7)])
def test_slot_of(n, experts, interp):
    ids = routed_ids(n, experts, 7, wild=True)
    g = torch.Generator().manual_seed(8)
    running = torch.randint(-50, 50, (n * experts,), generator=g)
    got = run(interpreted(B.slot_of(n, experts), interp), [running, ids, torch.zeros(n, dtype=torch.int64)])[2]
    assert torch.equal(got, O.slot_of(running, ids, n, experts))


@pytest.mark.parametrize("n", [128, 5, 1, 4096])
def test_group_tables(n):
    g = torch.Generator().manual_seed(n)
    counts = torch.randint(0, 4, (n,), generator=g) * (torch.rand(n, generator=g) < 0.6)   # empty groups
    offs = torch.cumsum(counts, 0).to(torch.int32)
    got = run(B.group_tables(n), [offs] + [torch.zeros(n, dtype=torch.int64) for _ in range(3)])[1:]
    for a, b in zip(got, O.group_tables(offs, n)):
        assert torch.equal(a, b)


@pytest.mark.parametrize("n,rows", [(128, 128), (129, 7), (4096, 300)])
def test_count_le(n, rows):
    g = torch.Generator().manual_seed(rows)
    v = torch.sort(torch.randint(-2, rows + 3, (n,), generator=g)).values
    got = run(B.count_le(n, rows), [v, torch.zeros(rows, dtype=torch.int32)])[1]
    assert torch.equal(got, O.count_le(v, n, rows, torch.int32))


def test_routing_chain_reproduces_the_routing():
    """counts (00) -> their running sum (01) -> each routed row's slot (02) rebuild the (cum, cnt, pos) tables a
    consistent routing has, which the weighted combine (03) reads."""
    tokens, topk, experts = 4096, 8, 128
    n = tokens * topk
    ids, cum, cnt, pos = moe_routing(tokens, topk, experts, 11)
    c0, r0 = run(B.expert_counts(n, experts), [ids, torch.zeros(experts, dtype=torch.int64),
                                               torch.zeros(n * experts, dtype=torch.int64)])[1:]
    c1 = run(B.cumsum_int(experts), [c0, torch.zeros(experts, dtype=torch.int64)])[1]
    s2 = run(B.slot_of(n, experts), [r0, ids, torch.zeros(n, dtype=torch.int64)])[2]
    assert torch.equal(c0, cnt) and torch.equal(c1, cum) and torch.equal(s2, pos)


@pytest.mark.parametrize("interp", [False, True], ids=["direct", "interpreter"])
def test_int_table_unit_ranges(interp):
    """Rows launched in parts (the runtime's split of a launch over GPUs) give the whole launch's tables."""
    n, experts = 20000, 64
    ids = routed_ids(n, experts, 5)
    d = D.to_bytes(interpreted(B.expert_counts(n, experts), interp))
    ts = [t.cuda() for t in (ids, torch.zeros(experts, dtype=torch.int64), torch.zeros(n * experts, dtype=torch.int64))]
    for lo, hi in ((0, 5), (5, 40), (40, 64)):
        RC.launch_tensors(d, ts, lo, hi)
    wc, wr = O.expert_counts(ids, experts, n)
    assert torch.equal(ts[1].cpu(), wc) and torch.equal(ts[2].cpu(), wr)


def test_int_table_out_of_range_is_recorded():
    """A load past its tensor records PTSIM_E_OOB (the reference's bounds assertion) and reads 0."""
    n = 64
    desc = B.cumsum_int(n)
    desc.arg_numel[0] = n - 1                 # the tensor holds one element fewer than the program reads
    ts = [torch.arange(n - 1, dtype=torch.int64).cuda(), torch.zeros(n, dtype=torch.int64).cuda()]
    with pytest.raises(native.ExecutorError) as e:
        RC.launch_tensors(D.to_bytes(desc), ts)
    assert e.value.code == D.E_OOB


def test_select_out_of_range_ids_report_like_the_interpreter():
    """An id read past its tensor records PTSIM_E_OOB on both paths."""
    n, experts = 16, 8
    for interp in (False, True):
        desc = interpreted(B.slot_of(n, experts), interp)
        desc.arg_numel[1] = n - 1
        ts = [torch.zeros(n * experts, dtype=torch.int64).cuda(), torch.zeros(n - 1, dtype=torch.int64).cuda(),
              torch.zeros(n, dtype=torch.int64).cuda()]
        with pytest.raises(native.ExecutorError) as e:
            RC.launch_tensors(D.to_bytes(desc), ts)
        assert e.value.code == D.E_OOB
