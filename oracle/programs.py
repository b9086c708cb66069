"""CPU oracle of the validation-class tile programs -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this module,
and only as the checker or the timed CPU baseline; the B200 product path never calls it.

Each function restates one program of the reference (the Triton source the reference compiles, cited per
function) in torch CPU arithmetic: fp32 compute, bf16 storage rounded to nearest-even, casts exactly where
the source casts, and the NPU's own op rules where the source leaves a choice to the target:
  - exp is 2^(x * log2 e), as the EUP computes it (targets/tpu/lower_vector_functions.py:310-329);
  - max/min propagate NaN (PyTorchSimTpuOps.td:64-74; tl.PropagateNan.ALL);
  - bf16 results are packed round-to-nearest-even (PyTorchSimTpuOps.td:46-50, lower_matmul.py:585-591).
torch CPU runs every op on all host threads (torch.set_num_threads), which is how the CPU baseline uses the
box's cores.  Tensors are flat, as kernel.json states them; bf16 arguments are torch.bfloat16."""
import math

import torch

LOG2E = 1.4426950408889634


def f32(t):
    return t.to(torch.float32)


def bf16(t):
    """Round an fp32 tensor to bf16 (RNE), as a store to a bf16 pointer does."""
    return t.to(torch.bfloat16)


def npu_exp(x):
    return torch.exp2(x * torch.tensor(LOG2E, dtype=torch.float32))


def nan_max(a, dim=None):
    """max that returns NaN whenever a NaN takes part (torch.max / amax already propagate NaN)."""
    return torch.amax(a, dim=dim, keepdim=True) if dim is not None else torch.amax(a)


# ---------------------------------------------------------------------------------------------------
# Pointwise programs
# ---------------------------------------------------------------------------------------------------

def vector_add(x, y):
    """tests/cases/smoke/add.py:20-25: o = x + y (fp32, bit exact)."""
    return x + y


def add_one(x):
    """validation/pytorchsim/vector_add1_*/00_*_triton.py: out = bf16(float(x) + 1.0)."""
    return bf16(f32(x) + 1.0)


def slice_add_one(x):
    """validation/pytorchsim/vector_slice_*/00_*_triton.py: out[0] = float(x[0]) + 1.0 (fp32 output)."""
    return (f32(x[:1]) + 1.0).to(torch.float32)


def heads_to_token_major(x, tokens, heads, dim):
    """qwen3_8b_layer_prefill_*/07_*: out[t, h, d] = in[h, t, d] (bit exact)."""
    return x.view(heads, tokens, dim).transpose(0, 1).contiguous().view(-1)


def token_to_head_major(x, tokens, heads, dim):
    """qwen3_8b_layer_prefill_*/05_*: out[h, t, d] = in[t, h, d] (bit exact)."""
    return x.view(tokens, heads, dim).transpose(0, 1).contiguous().view(-1)


def silu_mul(x, tokens, inter):
    """qwen3_8b_layer_prefill_*/10_*: x = [gate | up] per token; out = bf16(gate / (1 + exp(-gate)) * up)."""
    v = f32(x).view(tokens, 2 * inter)
    g, u = v[:, :inter], v[:, inter:]
    return bf16(g / (npu_exp(-g) + 1.0) * u).reshape(-1)


# ---------------------------------------------------------------------------------------------------
# Row programs
# ---------------------------------------------------------------------------------------------------

def softmax_rows(x, rows, cols, out_dtype=torch.bfloat16):
    """validation/pytorchsim/vector_softmax_*/00_*_triton.py:17-68: per row m = max (NaN-propagating),
    s = sum exp(x - m), out = bf16(exp(x - m) / s).  The MoE router's softmax
    (layer_op_router_post_*/00_*) stores the same quotient as fp32."""
    v = f32(x).view(rows, cols)
    m = nan_max(v, 1)
    e = npu_exp(v - m)
    return (e / e.sum(dim=1, keepdim=True)).to(out_dtype).reshape(-1)


def rmsnorm_rows(x, w, rows, cols, eps, res=None):
    """qwen3_8b_layer_prefill_*/00_*_triton.py: r = rsqrt(sum(x^2) / cols + eps); out = bf16((x * r) * w); with
    `res` (layer_layer_prefill_*/18_*) the row is x + res in fp32, unrounded."""
    v = f32(x).view(rows, cols)
    if res is not None:
        v = v + f32(res).view(rows, cols)
    ss = (v * v).sum(dim=1, keepdim=True)
    r = torch.rsqrt(ss / float(cols) + torch.tensor(eps, dtype=torch.float32))
    return bf16((v * r) * f32(w).view(1, cols)).reshape(-1)


def qknorm_rope(x, w, cos, sin, tokens, heads, eps, dim=128):
    """qwen3_8b_layer_prefill_*/02_*, 04_*: each (token, head) row of `dim`: r = rsqrt(mean(x^2) + eps),
    n = (x * r) * w, rot = cat(-n[half:], n[:half]), out[h, t] = bf16(n * cos[t] + rot * sin[t]), stored
    head-major (out index d + dim * t + tokens * dim * h)."""
    v = f32(x).view(tokens, heads, dim)
    r = torch.rsqrt((v * v).sum(dim=2, keepdim=True) / float(dim) + torch.tensor(eps, dtype=torch.float32))
    n = (v * r) * f32(w).view(1, 1, dim)
    half = dim // 2
    rot = torch.cat([-n[..., half:], n[..., :half]], dim=2)
    c = f32(cos).view(tokens, 1, dim)
    s = f32(sin).view(tokens, 1, dim)
    out = n * c + rot * s
    return bf16(out).transpose(0, 1).contiguous().reshape(-1)


def row_sum(x, rows, cols):
    """layer_layer_prefill_*/22_*_triton.py: out[r] = the fp32 sum of row r (the top-k weights of a token)."""
    return f32(x).view(rows, cols).sum(dim=1)


def rope_rows(x, cos, sin, tokens, heads, dim=128):
    """layer_op_rope_{q,k}_*/00_*_triton.py: each (token, head) row of `dim`: rot = cat(-x[half:], x[:half]),
    out = bf16(x * cos[t] + rot * sin[t]) in fp32, token-major like the input (one token: the tables are that
    position's)."""
    v = f32(x).view(tokens, heads, dim)
    half = dim // 2
    rot = torch.cat([-v[..., half:], v[..., :half]], dim=2)
    c = f32(cos).view(tokens, 1, dim)
    s = f32(sin).view(tokens, 1, dim)
    return bf16(v * c + rot * s).reshape(-1)


def reduce_all(x, op):
    """vector_sum_* / vector_max_*: one fp32 value over the whole tensor."""
    v = f32(x).reshape(-1)
    return (v.sum() if op == "sum" else torch.amax(v)).reshape(1)


# ---------------------------------------------------------------------------------------------------
# Matrix-unit programs
# ---------------------------------------------------------------------------------------------------

def gemm(a, b, M, N, K, residual=None, b_kn=True, out_dtype=torch.bfloat16):
    """gemm_*/00_*_triton.py and Qwen3 01/03/08/09/11: acc = A . B in fp32 from bf16 inputs (the MXU's f32
    pop, lower_matmul.py:421-506); + float(residual) when the epilogue adds one; stored as bf16."""
    A = f32(a).view(M, K)
    B = f32(b).view(K, N) if b_kn else f32(b).view(N, K).t()
    acc = A @ B
    if residual is not None:
        acc = acc + f32(residual).view(M, N)
    return acc.to(out_dtype).reshape(-1)


def attention_prefill(q, k, v, batch, hq, g, seq, dim, bq, bkv, causal, scale):
    """validation/pytorchsim/attention_prefill_*/00__prefill_kernel/_prefill_kernel_triton.py:3-44, block for
    block: per query block of bq rows m = -1e30, l = 0, acc = 0; per key block of bkv below the diagonal and
    then the diagonal block (masked to -1e30 where key > query): qk = (q . k^T) * SCALE in fp32,
    m' = max(m, rowmax), alpha = exp(m - m'), p = exp(qk - m'), l = l*alpha + rowsum p,
    acc = acc*alpha + bf16(p) . v; out = bf16(acc / l)."""
    hkv = hq // g
    Q = f32(q).view(batch, hq, seq, dim)
    Kt = f32(k).view(batch, hkv, seq, dim)
    V = f32(v).view(batch, hkv, seq, dim)
    out = torch.empty(batch, hq, seq, dim, dtype=torch.bfloat16)
    sc = torch.tensor(scale, dtype=torch.float32)
    for qb in range(seq // bq):
        rm = torch.arange(qb * bq, (qb + 1) * bq)
        qt = Q[:, :, qb * bq:(qb + 1) * bq, :]                      # [B, HQ, bq, D]
        m = torch.full((batch, hq, bq, 1), -1.0e30)
        l = torch.zeros((batch, hq, bq, 1))
        acc = torch.zeros((batch, hq, bq, dim))
        starts = list(range(0, qb * bq if causal else seq, bkv))
        blocks = [(s, False) for s in starts] + ([(qb * bq, True)] if causal else [])
        for start, diag in blocks:
            kb = Kt[:, :, start:start + bkv, :].repeat_interleave(g, dim=1)
            vb = V[:, :, start:start + bkv, :].repeat_interleave(g, dim=1)
            qk = (qt @ kb.transpose(2, 3)) * sc
            if diag:
                n = torch.arange(start, start + bkv)
                qk = torch.where(rm[:, None] >= n[None, :], qk, torch.tensor(-1.0e30))
            m_new = torch.maximum(m, torch.amax(qk, dim=3, keepdim=True))
            alpha = npu_exp(m - m_new)
            p = npu_exp(qk - m_new)
            l = l * alpha + p.sum(dim=3, keepdim=True)
            acc = acc * alpha + f32(p.to(torch.bfloat16)) @ vb
            m = m_new
        out[:, :, qb * bq:(qb + 1) * bq, :] = (acc / l).to(torch.bfloat16)
    return out.reshape(-1)


def attention_decode(q, k, v, o_init, hkv, g, gp, seq, dim, bkv, scale):
    """validation/pytorchsim/attention_decode_32x8x4096_bf16/00__decode_kernel/_decode_kernel_triton.py:4-31, block
    for block: program p (one KV head) loads its GP query rows (rows >= G masked to 0); m = -1e30, l = 0,
    acc = 0; per key block of BKV: qk = (q . k^T) * SCALE in fp32, m' = max(m, rowmax qk), alpha = exp(m - m'),
    p = exp(qk - m'), l = l*alpha + rowsum p, acc = acc*alpha + bf16(p) . v; the G real rows of
    bf16(acc / l) are stored (o is inout: nothing else of it changes)."""
    Q = torch.zeros(hkv, gp, dim)
    Q[:, :g] = f32(q).view(hkv, g, dim)
    Kt = f32(k).view(hkv, seq, dim)
    V = f32(v).view(hkv, seq, dim)
    sc = torch.tensor(scale, dtype=torch.float32)
    m = torch.full((hkv, gp, 1), -1.0e30)
    l = torch.zeros((hkv, gp, 1))
    acc = torch.zeros((hkv, gp, dim))
    for start in range(0, seq, bkv):
        kb, vb = Kt[:, start:start + bkv], V[:, start:start + bkv]
        qk = (Q @ kb.transpose(1, 2)) * sc
        m_new = torch.maximum(m, torch.amax(qk, dim=2, keepdim=True))
        alpha = npu_exp(m - m_new)
        p = npu_exp(qk - m_new)
        l = l * alpha + p.sum(dim=2, keepdim=True)
        acc = acc * alpha + f32(p.to(torch.bfloat16)) @ vb
        m = m_new
    out = o_init.clone().view(hkv, g, dim)
    out[:] = (acc / l)[:, :g].to(torch.bfloat16)
    return out.reshape(-1)


# ---------------------------------------------------------------------------------------------------
# Mixture-of-experts routing programs (the Qwen3-30B-A3B layer ops of the validation bundle)
# ---------------------------------------------------------------------------------------------------

def topk_rows(x, rows, cols, cols_padded, k, largest=True):
    """layer_op_router_post_*/01__topk_kernel/_topk_kernel_triton.py:3-26: per row, columns past `cols` (up to
    the program's EP = cols_padded) hold the spent value (-inf for largest); k passes each take the best value,
    then the smallest column holding it, and overwrite that column with the spent value.  Returns (values,
    int64 column indices), k per row."""
    spent = float("-inf") if largest else float("inf")
    X = torch.full((rows, cols_padded), spent, dtype=torch.float32)
    X[:, :cols] = f32(x).view(rows, cols)
    c = torch.arange(cols_padded)
    vals = torch.zeros(rows, k, dtype=torch.float32)
    idxs = torch.zeros(rows, k, dtype=torch.int64)
    r = torch.arange(rows)
    for n in range(k):
        best = X.max(dim=1).values if largest else X.min(dim=1).values
        at = torch.where(X == best[:, None], c, cols_padded).min(dim=1).values
        vals[:, n], idxs[:, n] = best, at
        X[r, at.clamp(max=cols_padded - 1)] = spent
    return vals.to(x.dtype).reshape(-1), idxs.reshape(-1)


def sort_rows(x, rows, cols, descending=False, float_keys=False):
    """layer_op_dispatch_*/00__sort_kernel/_sort_kernel_triton.py:3-53: each row sorted by the key k = x (int64)
    or, for fp32, bits b = (NaN -> 0x7FC00000, +-0 -> 0) mapped to the order-preserving b ^ ((b >> 31) &
    0x7FFFFFFF); descending sorts ~k; ties by source position (the network compares (k, position)).  The
    stored values are the sorted keys mapped back, positions as int64."""
    if float_keys:
        f = f32(x).view(rows, cols)
        b = f.view(torch.int32).clone()
        b = torch.where(torch.isnan(f), torch.full_like(b, 0x7FC00000), b)
        b = torch.where(f == 0, torch.zeros_like(b), b)
        k = (b ^ ((b >> 31) & 0x7FFFFFFF)).to(torch.int64)
    else:
        k = x.view(rows, cols).to(torch.int64)
    if descending:
        k = ~k
    order = torch.sort(k, dim=1, stable=True).indices
    ks = torch.gather(k, 1, order)
    if descending:
        ks = ~ks
    if float_keys:
        b = ks.to(torch.int32)
        vals = (b ^ ((b >> 31) & 0x7FFFFFFF)).view(torch.float32)
    else:
        vals = ks
    return vals.to(x.dtype).reshape(-1), order.reshape(-1)


def row_divsum(x, rows, cols, out_dtype=torch.bfloat16):
    """layer_op_router_post_*/02_*_triton.py: out = (x / sum(x)) per row in fp32, cast on the store."""
    v = f32(x).view(rows, cols)
    return (v / v.sum(dim=1, keepdim=True)).to(out_dtype).reshape(-1)


def dispatch_gather(idx, table, tokens, hidden, topk):
    """layer_op_dispatch_*/01_*_triton.py: output row r (of `hidden` values) is token t of the table, t =
    Python floor division of the sorted position idx[r] by top-k (the kernel's ~ / // / ~ sequence), negative t
    wrapped by + tokens; the kernel asserts 0 <= t < tokens.  bf16 -> fp32 -> bf16 is a copy."""
    q = torch.div(idx.to(torch.int64), topk, rounding_mode="floor")
    q = torch.where(q < 0, q + tokens, q)
    if not bool(((q >= 0) & (q < tokens)).all()):
        raise IndexError("dispatch gather index out of range (the reference asserts)")
    return table.view(tokens, hidden)[q].reshape(-1)


def combine_weighted(idx, cum, cnt, pos, expert_out, w, tokens, hidden, topk, experts):
    """layer_op_combine_*/03_*_triton.py: token t's k-th choice e = idx[t, k] (negative e wrapped by + experts)
    sits in expert order at row p = cum[e] - cnt[e] + (pos[t, k] - 1) (negative p wrapped by + tokens * topk; the
    kernel asserts both ranges); out[t, :] = bf16(sum over k of float(expert_out[p, :]) * float(w[t, k]))."""
    e = idx.to(torch.int64).view(tokens, topk)
    e = torch.where(e < 0, e + experts, e)
    rows = tokens * topk
    p = cum.to(torch.int64)[e] - cnt.to(torch.int64)[e] + (pos.to(torch.int64).view(tokens, topk) - 1)
    p = torch.where(p < 0, p + rows, p)
    if not bool(((e >= 0) & (e < experts)).all() and ((p >= 0) & (p < rows)).all()):
        raise IndexError("combine index out of range (the reference asserts)")
    g = f32(expert_out).view(rows, hidden)[p]                  # [tokens, topk, hidden]
    acc = (g * f32(w).view(tokens, topk, 1)).sum(dim=1)
    return acc.to(torch.bfloat16).reshape(-1)


def expert_counts(ids, experts, n):
    """layer_op_combine_*/00_*_triton.py: over the n routed expert ids (int64), for each expert x < experts
    count[x] = the number of ids equal to x (out_ptr0), and running[x + experts * r] = the number of
    ids[0..r] equal to x, inclusive (out_ptr1: the kernel's block scan plus the carried total of the blocks
    before, rows of `experts`)."""
    onehot = (ids.reshape(-1)[:n].to(torch.int64)[:, None] == torch.arange(experts)[None, :]).to(torch.int64)
    return onehot.sum(dim=0), onehot.cumsum(dim=0).reshape(-1)


def cumsum_int(x, n, out_dtype):
    """layer_op_gmm_*/01_*_triton.py (int32) and layer_op_combine_*/01_*_triton.py (int64): the inclusive
    running sum of n integers, stored as out_dtype (integer sums wrap; an int32 scan's low 32 bits equal the
    int64 sum's)."""
    return torch.cumsum(x.reshape(-1)[:n].to(torch.int64), dim=0).to(out_dtype)


def slot_of(running, ids, n, experts):
    """layer_op_combine_*/02_*_triton.py: out[x] = sum over r < experts of running[r + experts * x] *
    (ids[x] == r), i.e. running[x, ids[x]] for ids in [0, experts), else 0 (int64)."""
    run = running.reshape(-1)[:n * experts].to(torch.int64).view(n, experts)
    hit = (ids.reshape(-1)[:n].to(torch.int64)[:, None] == torch.arange(experts)[None, :]).to(torch.int64)
    return (run * hit).sum(dim=1)


def group_tables(offsets, n):
    """layer_op_gmm_*/02_*_triton.py over the n running offsets o (int32 in, int64 out): prev[r] = o[r - 1]
    (0 at r = 0; out_ptr1), count[r] = o[r] - prev[r] (out_ptr2), and the inclusive running number of
    non-empty groups, cumsum(count > 0) (out_ptr0)."""
    o = offsets.reshape(-1)[:n].to(torch.int64)
    prev = torch.cat([torch.zeros(1, dtype=torch.int64), o[:-1]])
    count = o - prev
    return torch.cumsum((count > 0).to(torch.int64), dim=0), prev, count


def count_le(x, n, rows, out_dtype):
    """layer_op_gmm_*/03_*_triton.py: out[e] = the number of r < n with x[r] <= e, for e < rows (cast on the
    store)."""
    v = x.reshape(-1)[:n].to(torch.int64)
    return (v[None, :] <= torch.arange(rows)[:, None]).to(torch.int64).sum(dim=1).to(out_dtype)


def combine_weighted_fused(idx, cum, cnt, pos, expert_out, w, wsum, res_a, res_b, tokens, hidden, topk, experts):
    """layer_layer_{decode,prefill}_*/23_*, 27_*: the combine with each token's weights divided by their sum
    (fp32 w[t, k] / wsum[t]) and the residual stream added: out = bf16((res_a + res_b) + sum over k of
    float(expert_out[p, :]) * (w / wsum)), p as combine_weighted's."""
    e = idx.to(torch.int64).view(tokens, topk)
    e = torch.where(e < 0, e + experts, e)
    rows = tokens * topk
    p = cum.to(torch.int64)[e] - cnt.to(torch.int64)[e] + (pos.to(torch.int64).view(tokens, topk) - 1)
    p = torch.where(p < 0, p + rows, p)
    if not bool(((e >= 0) & (e < experts)).all() and ((p >= 0) & (p < rows)).all()):
        raise IndexError("combine index out of range (the reference asserts)")
    g = f32(expert_out).view(rows, hidden)[p]
    wk = f32(w).view(tokens, topk) / f32(wsum).view(-1)[:tokens].view(tokens, 1)
    acc = (g * wk.view(tokens, topk, 1)).sum(dim=1)
    resid = f32(res_a).view(tokens, hidden) + f32(res_b).view(tokens, hidden)
    return (resid + acc).to(torch.bfloat16).reshape(-1)


def grouped_gemm(a, b, group, start, rows, c_init, M, N, K, groups):
    """layer_op_gmm_*/05__grouped_mm_kernel/_grouped_mm_kernel_triton.py:4-44: program p takes group
    g = group[p] and its rows [start[g], start[g] + rows[g]); those rows of c become bf16(a_rows . b[g]) with
    fp32 accumulation; rows no program lists keep c's values."""
    A = f32(a).view(M, K)
    B = f32(b).view(groups, K, N)
    out = c_init.clone().view(M, N)
    for g in group.tolist():
        n = int(rows[g])
        if n <= 0:
            continue
        s = int(start[g])
        out[s:s + n] = (A[s:s + n] @ B[g]).to(out.dtype)
    return out.reshape(-1)


def sumsq(x, n, res=None):
    """qwen3_8b_layer_decode_*/00_*_triton.py (and 05_*, with a residual row added first, unrounded): one fp32
    value, the sum over the n elements of (x (+ res))^2."""
    v = f32(x).reshape(-1)[:n]
    if res is not None:
        v = v + f32(res).reshape(-1)[:n]
    return (v * v).sum().reshape(1)


def rmsnorm_gemv(x, ss, w, mat, K, N, eps, res=None, out_dtype=torch.bfloat16):
    """qwen3_8b_layer_decode_*/01_*_triton.py (and 06_*, with a residual row added first): the RMSNorm'd vector
    v = (x (+ res)) * rsqrt(ss / K + eps) * w in fp32, never rounded to bf16, times the [K, N] matrix (fp32
    accumulation), cast on the store; ss is the fp32 sum of squares the previous program stored."""
    v = f32(x).reshape(-1)[:K]
    if res is not None:
        v = v + f32(res).reshape(-1)[:K]
    v = (v * torch.rsqrt(f32(ss).reshape(-1)[0] / K + eps)) * f32(w).reshape(-1)[:K]
    return (v @ f32(mat).view(K, N)).to(out_dtype)


def silu_gemv(gate_up, mat, res1, res2, K, N, out_dtype=torch.bfloat16):
    """qwen3_8b_layer_decode_*/07_*_triton.py: v = silu(gate) * up over the [gate | up] row (gate / (1 + exp(-gate))
    in fp32, unrounded), out = v . [K, N] matrix + (res1 + res2), cast on the store."""
    gu = f32(gate_up).reshape(-1)
    g, u = gu[:K], gu[K:2 * K]
    v = (g / (npu_exp(-g) + 1.0)) * u
    acc = v @ f32(mat).view(K, N)
    return (acc + (f32(res1).reshape(-1)[:N] + f32(res2).reshape(-1)[:N])).to(out_dtype)


def rope_tables(tokens, dim=128, theta=1.0e6):
    """cos/sin tables [tokens, dim] in fp32 for RoPE with base `theta` (the Qwen3 layer feeds them as the
    fp32 inputs in_ptr2/in_ptr3 of 02/04)."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    t = torch.arange(tokens, dtype=torch.float64)
    f = torch.outer(t, inv)
    emb = torch.cat([f, f], dim=1)
    return emb.cos().to(torch.float32).reshape(-1), emb.sin().to(torch.float32).reshape(-1)


def layer_attention_half(x, p, T, hq, hkv, residual, hidden=4096, dim=128, eps=1e-6, cos=None, sin=None,
                         bq=1024, bkv=1024):
    """Launches 00-08 of the layer for `hq` query / `hkv` KV heads (a tensor-parallel rank's share when
    they are fewer than 32 / 8): bf16 o-projection output, plus `x` when `residual`."""
    h = rmsnorm_rows(x, p["ln1"], T, hidden, eps)
    q = gemm(h, p["wq"], T, hq * dim, hidden)
    k = gemm(h, p["wk"], T, hkv * dim, hidden)
    v = gemm(h, p["wv"], T, hkv * dim, hidden)
    qh = qknorm_rope(q, p["qn"], cos, sin, T, hq, eps, dim)
    kh = qknorm_rope(k, p["kn"], cos, sin, T, hkv, eps, dim)
    vh = token_to_head_major(v, T, hkv, dim)
    o = attention_prefill(qh, kh, vh, 1, hq, hq // hkv, T, dim, min(bq, T), min(bkv, T), True, 1.0 / math.sqrt(dim))
    ot = heads_to_token_major(o, T, hq, dim)
    return gemm(ot, p["wo"], T, hidden, hq * dim, residual=x if residual else None)


def layer_mlp_half(x1, p, T, inter, residual, hidden=4096, eps=1e-6):
    """Launches 00, 09-11 of the layer for `inter` intermediate columns: bf16 down-projection output,
    plus `x1` when `residual`."""
    h2 = rmsnorm_rows(x1, p["ln2"], T, hidden, eps)
    gu = gemm(h2, p["wgu"], T, 2 * inter, hidden)
    a = silu_mul(gu, T, inter)
    return gemm(a, p["wd"], T, hidden, inter, residual=x1 if residual else None)


def decoder_layer(x, p, T, hidden=4096, hq=32, hkv=8, dim=128, inter=12288, eps=1e-6, cos=None, sin=None,
                  bq=1024, bkv=1024):
    """The Qwen3-8B-shaped prefill layer as the 14 launches of validation/pytorchsim/
    qwen3_8b_layer_prefill_2048x2048_bf16/manifest.json run it: RMSNorm, q/k/v projections, QK-RMSNorm +
    RoPE into head-major q/k, v relayout, causal GQA attention, head -> token relayout, o projection +
    residual, RMSNorm, gate_up projection, SiLU * mul, down projection + residual.  `p` holds the weights
    (bf16, [in, out] row-major as the bundle feeds them)."""
    h = rmsnorm_rows(x, p["ln1"], T, hidden, eps)
    q = gemm(h, p["wq"], T, hq * dim, hidden)
    k = gemm(h, p["wk"], T, hkv * dim, hidden)
    v = gemm(h, p["wv"], T, hkv * dim, hidden)
    qh = qknorm_rope(q, p["qn"], cos, sin, T, hq, eps, dim)
    kh = qknorm_rope(k, p["kn"], cos, sin, T, hkv, eps, dim)
    vh = token_to_head_major(v, T, hkv, dim)
    bq_, bkv_ = min(bq, T), min(bkv, T)
    o = attention_prefill(qh, kh, vh, 1, hq, hq // hkv, T, dim, bq_, bkv_, True, 1.0 / math.sqrt(dim))
    ot = heads_to_token_major(o, T, hq, dim)
    x1 = gemm(ot, p["wo"], T, hidden, hq * dim, residual=x)
    h2 = rmsnorm_rows(x1, p["ln2"], T, hidden, eps)
    gu = gemm(h2, p["wgu"], T, 2 * inter, hidden)
    a = silu_mul(gu, T, inter)
    return gemm(a, p["wd"], T, hidden, inter, residual=x1)
