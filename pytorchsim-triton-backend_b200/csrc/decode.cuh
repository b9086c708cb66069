// One-token GQA attention (decode): the attention_decode_* program of the validation bundle and launch 03
// of the Qwen3 decode layer (validation/pytorchsim/attention_decode_32x8x4096_bf16/00__decode_kernel/
// _decode_kernel_triton.py:4-31).  Program p is one KV head: q [G, D] at p*G*D (G real rows of GP = 16),
// keys and values [S, D] at p*S*D.  Per query row: m = -1e30, l = 0, acc = 0; per key block
// qk = (q . k^T) * SCALE in fp32, m' = max(m, rowmax qk), alpha = exp(m - m'), p = exp(qk - m'),
// l = l * alpha + rowsum p, acc = acc * alpha + bf16(p) . v; o = bf16(acc / l).  exp is 2^(x * log2 e)
// as the NPU's EUP computes it.
//
// The bundle has 8 programs of up to 8192 keys each -- far fewer than 148 SMs -- so the keys of every
// program are split into chunks (flash decoding) and the per-chunk states merged afterwards:
//   decode_part_kernel     one CTA per (KV head, chunk of L keys).  Warp 4 streams the chunk's K and V
//                          tiles (64 keys x 128 d as two 128B-swizzled 8 KB TMA boxes each) into a
//                          3-deep ring; warps 0-3 each take 16 keys of every tile: S = Q . K^T and
//                          O += bf16(P) . V on mma.sync m16n8k16, whose M = 16 is exactly the program's
//                          padded query rows (tcgen05.mma's smallest M is 64: three quarters of every
//                          tile would be padding, plus a TMEM round trip per 16-key softmax, in a kernel
//                          whose bound is streaming K and V from HBM at <= 16 FLOP per byte).  The
//                          online softmax stays in registers; the four warps' states meet in shared
//                          memory and the CTA writes its chunk's (m, l, O) to the workspace.
//   decode_combine_kernel  per (head, row): m = max_c m_c, l = sum_c l_c 2^((m_c - m) log2 e),
//                          o = bf16(sum_c O_c 2^((m_c - m) log2 e) / l), chunks in ascending order (a
//                          fixed summation order).  Launched as a programmatic dependent of the first
//                          kernel (griddepcontrol), which releases it as soon as its CTAs start, so the
//                          merge's launch overlaps the streaming instead of following it.
// Every wait is bounded; a wait that gives up records PTSIM_E_TIMEOUT, the loader drains the copies it
// issued, and the CTA exits normally.
#pragma once
#include "sm100.cuh"
#include "gemm.cuh"

namespace ptsim {

constexpr int kDecTile = 64;                          // keys per ring tile
constexpr int kDecD = 128;                            // head dim
constexpr int kDecRows = 16;                          // query rows of a program, padded (its GP)
constexpr int kDecStages = 3;
constexpr int kDecBox = kDecTile * 64 * 2;            // 8 KB: 64 keys x 64 d
constexpr int kDecStage = 4 * kDecBox;                // K d 0-63, K d 64-127, V d 0-63, V d 64-127
constexpr int kDecThreads = 160;                      // warps 0-3 compute, warp 4 loads
constexpr int kDecSmem = kDecStages * kDecStage + 1024 + 128;
constexpr float kDecLog2e = 1.4426950408889634f;

struct DecodeArgs {
  CUtensorMap tk, tv;      // [hkv * S, 128] bf16, box {64, 64}, 128-byte swizzle
  const uint16_t *q;
  uint16_t *o;
  float *part_o;           // [units of the launch][chunks][G][128]
  float *part_ml;          // [units of the launch][chunks][G][2]: (m, l)
  int64_t unit_begin;      // first KV head of the launch
  int32_t G, S, chunks, chunk_keys;
  float scale;
  // PTSIM_FLAG_TEST_STALL: the first chunk of the first KV head arms its first stage but issues none of
  // its copies, and every wait gives up after kTestWaitUs -- the timeout path under test.
  int32_t stall;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D (16 x 8, fp32) += A (16 x 16, bf16, row) . B (16 x 8, bf16, col).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld_bf16x2(const uint16_t *p) {
  return uint32_t(__ldg(p)) | (uint32_t(__ldg(p + 1)) << 16);
}

__global__ void __launch_bounds__(kDecThreads, 2) decode_part_kernel(const __grid_constant__ DecodeArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kDecStages * kDecStage);
  uint64_t *empty = full + kDecStages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kDecStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunk = blockIdx.x;
  const int64_t ul = blockIdx.y;                   // unit (KV head) within the launch
  const int64_t unit = g.unit_begin + ul;
  const int key0 = chunk * g.chunk_keys;
  const int nkeys = g.S - key0 < g.chunk_keys ? g.S - key0 : g.chunk_keys;
  const int ntiles = nkeys / kDecTile;
  const int row0 = int(unit * g.S) + key0;         // TMA row of the chunk's first key
  const uint32_t wl = g.stall ? kTestWaitUs : kWaitUs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kDecStages; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 4);                // one arrival per compute warp
    }
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  __syncthreads();
  // The merge kernel may be scheduled now: it waits (griddepcontrol.wait) for this whole grid to finish
  // and flush, so starting it early only hides its launch.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int gq = lane >> 2, qd = lane & 3;         // fragment row (and row + 8) and column pair
  float o[16][4];                                  // O rows gq / gq+8, d = 8 i + 2 qd (+1)
  float m0 = -1.0e30f, m1 = -1.0e30f, l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  if (warp == 4) {
    if (lane == 0) {
      sm100::tma_prefetch_desc(&g.tk);
      sm100::tma_prefetch_desc(&g.tv);
      int j = 0;
      for (; j < ntiles; ++j) {
        const int st = j % kDecStages;
        if (j >= kDecStages && !sm100::mbar_wait(&empty[st], ((j / kDecStages) - 1) & 1, wl)) {
          *abort_flag = 1;
          break;
        }
        uint8_t *b = smem + st * kDecStage;
        const int y = row0 + j * kDecTile;
        sm100::mbar_arrive_expect_tx(&full[st], kDecStage);
        if (g.stall && chunk == 0 && ul == 0 && j == 0) continue;   // test hook: armed, no copy in flight
        sm100::tma_load_2d(b, &g.tk, &full[st], 0, y);
        sm100::tma_load_2d(b + kDecBox, &g.tk, &full[st], 64, y);
        sm100::tma_load_2d(b + 2 * kDecBox, &g.tv, &full[st], 0, y);
        sm100::tma_load_2d(b + 3 * kDecBox, &g.tv, &full[st], 64, y);
      }
      // The last fills of each stage have landed before the ring is reused by the epilogue.
      for (int i = j - kDecStages < 0 ? 0 : j - kDecStages; i < j; ++i)
        sm100::mbar_wait(&full[i % kDecStages], (i / kDecStages) & 1, wl);
    }
  } else {
    // Q fragments (A operand, rows gq and gq + 8, zero past G): d = 16 kk + 2 qd (+1) and + 8.
    uint32_t qa[8][4];
    const uint16_t *qp = g.q + unit * int64_t(g.G) * kDecD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = 16 * kk + 2 * qd;
      qa[kk][0] = gq < g.G ? ld_bf16x2(qp + gq * kDecD + d0) : 0u;
      qa[kk][1] = gq + 8 < g.G ? ld_bf16x2(qp + (gq + 8) * kDecD + d0) : 0u;
      qa[kk][2] = gq < g.G ? ld_bf16x2(qp + gq * kDecD + d0 + 8) : 0u;
      qa[kk][3] = gq + 8 < g.G ? ld_bf16x2(qp + (gq + 8) * kDecD + d0 + 8) : 0u;
    }
    const uint32_t base = sm100::smem_u32(smem);
    // ldmatrix row addresses.  K (x4): matrices (keys 0-7 | d +0), (keys 0-7 | d +8), (keys 8-15 | d +0),
    // (keys 8-15 | d +8) of the warp's 16 keys = B fragments of both 8-key score tiles.  V (x4, transposed):
    // (keys 0-7 | d +0), (keys 8-15 | d +0), (keys 0-7 | d +8), (keys 8-15 | d +8) = B fragments of two
    // 8-column output tiles.  Row r of a box holds 16-byte unit u at u ^ (r % 8) (128-byte swizzle).
    const int kr = 16 * warp + (lane & 7) + ((lane >> 4) << 3);
    const int kc = (lane >> 3) & 1;
    const int vr = 16 * warp + (lane & 7) + (((lane >> 3) & 1) << 3);
    const int vc = lane >> 4;
    const float scale = g.scale;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % kDecStages;
      if (!sm100::mbar_wait(&full[st], (j / kDecStages) & 1, wl)) {
        *abort_flag = 1;
        break;
      }
      const uint32_t kb = base + st * kDecStage, vb = kb + 2 * kDecBox;
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int u = 2 * (kk & 3) + kc;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + (kk >> 2) * kDecBox + kr * 128 + ((u ^ (kr & 7)) << 4), b0, b1, b2, b3);
        mma_16816(s0, qa[kk], b0, b1);
        mma_16816(s1, qa[kk], b2, b3);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s0[i] *= scale;
        s1[i] *= scale;
      }
      float x0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
      float x1 = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
      x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, 1));
      x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, 2));
      x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, 1));
      x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, 2));
      const float mn0 = fmaxf(m0, x0), mn1 = fmaxf(m1, x1);
      const float al0 = ex2_fast((m0 - mn0) * kDecLog2e), al1 = ex2_fast((m1 - mn1) * kDecLog2e);
      m0 = mn0;
      m1 = mn1;
      float p0[4], p1[4];
      p0[0] = ex2_fast((s0[0] - mn0) * kDecLog2e);
      p0[1] = ex2_fast((s0[1] - mn0) * kDecLog2e);
      p0[2] = ex2_fast((s0[2] - mn1) * kDecLog2e);
      p0[3] = ex2_fast((s0[3] - mn1) * kDecLog2e);
      p1[0] = ex2_fast((s1[0] - mn0) * kDecLog2e);
      p1[1] = ex2_fast((s1[1] - mn0) * kDecLog2e);
      p1[2] = ex2_fast((s1[2] - mn1) * kDecLog2e);
      p1[3] = ex2_fast((s1[3] - mn1) * kDecLog2e);
      l0 = l0 * al0 + ((p0[0] + p0[1]) + (p1[0] + p1[1]));
      l1 = l1 * al1 + ((p0[2] + p0[3]) + (p1[2] + p1[3]));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        o[i][0] *= al0;
        o[i][1] *= al0;
        o[i][2] *= al1;
        o[i][3] *= al1;
      }
      // P as the A operand of P . V: its accumulator layout is the A fragment layout of one k-step.
      const uint32_t pa[4] = {pack_bf16x2(p0[0], p0[1]), pack_bf16x2(p0[2], p0[3]), pack_bf16x2(p1[0], p1[1]),
                              pack_bf16x2(p1[2], p1[3])};
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int u = 2 * (dp & 3) + vc;
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vb + (dp >> 2) * kDecBox + vr * 128 + ((u ^ (vr & 7)) << 4), v0, v1, v2, v3);
        mma_16816(o[2 * dp], pa, v0, v1);
        mma_16816(o[2 * dp + 1], pa, v2, v3);
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty[st]);
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  }
  __syncthreads();  // every tile consumed and every copy landed: the ring is free for the merge

  // The four warps' (m, l, O) meet in shared memory; the CTA's chunk state goes to the workspace.
  float *cm = reinterpret_cast<float *>(smem);     // [4][16]
  float *cl = cm + 4 * kDecRows;                   // [4][16]
  float *co = cl + 4 * kDecRows;                   // [4][16][128]
  if (warp < 4) {
    if (qd == 0) {
      cm[warp * kDecRows + gq] = m0;
      cm[warp * kDecRows + gq + 8] = m1;
      cl[warp * kDecRows + gq] = l0;
      cl[warp * kDecRows + gq + 8] = l1;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int d = 8 * i + 2 * qd;
      *reinterpret_cast<float2 *>(&co[(warp * kDecRows + gq) * kDecD + d]) = make_float2(o[i][0], o[i][1]);
      *reinterpret_cast<float2 *>(&co[(warp * kDecRows + gq + 8) * kDecD + d]) = make_float2(o[i][2], o[i][3]);
    }
  }
  __syncthreads();
  if (threadIdx.x < kDecD && !*abort_flag) {
    const int t = threadIdx.x;
    const int64_t slot = (ul * g.chunks + chunk) * g.G;
    for (int r = 0; r < g.G; ++r) {
      float ms = cm[r];
#pragma unroll
      for (int w = 1; w < 4; ++w) ms = fmaxf(ms, cm[w * kDecRows + r]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float e = ex2_fast((cm[w * kDecRows + r] - ms) * kDecLog2e);
        L += cl[w * kDecRows + r] * e;
        O += co[(w * kDecRows + r) * kDecD + t] * e;
      }
      g.part_o[(slot + r) * kDecD + t] = O;
      if (t == 0) {
        g.part_ml[(slot + r) * 2] = ms;
        g.part_ml[(slot + r) * 2 + 1] = L;
      }
    }
  }
}

// grid (units of the launch, G), 128 threads: thread t = output column d.  Every load is issued before
// the one barrier (one L2 round trip): thread c < chunks fetches chunk c's (m, l), every thread its column
// of up to 32 chunks' O; then the weights 2^((m_c - m) log2 e) and the sums in ascending chunk order.
constexpr int kDecMaxChunks = 64;

__global__ void __launch_bounds__(kDecD) decode_combine_kernel(const __grid_constant__ DecodeArgs g) {
  __shared__ float wm[kDecMaxChunks], wl[kDecMaxChunks];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t ul = blockIdx.x;
  const int r = blockIdx.y, t = threadIdx.x, C = g.chunks;
  const int64_t first = ul * C * g.G + r;          // slot of chunk 0; chunk c at + c * G
  const int64_t ostep = int64_t(g.G) * kDecD;
  const float *po = g.part_o + first * kDecD + t;
  if (t < C) {
    wm[t] = g.part_ml[(first + int64_t(t) * g.G) * 2];
    wl[t] = g.part_ml[(first + int64_t(t) * g.G) * 2 + 1];
  }
  float ov[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) ov[i] = i < C ? po[i * ostep] : 0.f;
  __syncthreads();
  float ms = wm[0];
  for (int c = 1; c < C; ++c) ms = fmaxf(ms, wm[c]);
  float L = 0.f, O = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i < C) {
      const float e = ex2_fast((wm[i] - ms) * kDecLog2e);
      L += wl[i] * e;
      O += ov[i] * e;
    }
  for (int c = 32; c < C; c += 32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) ov[i] = c + i < C ? po[(c + i) * ostep] : 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (c + i < C) {
        const float e = ex2_fast((wm[c + i] - ms) * kDecLog2e);
        L += wl[c + i] * e;
        O += ov[i] * e;
      }
  }
  g.o[((g.unit_begin + ul) * g.G + r) * kDecD + t] = f32_to_bf16_bits(__fdiv_rn(O, L));
}

// The chunk plan: about one CTA per SM over the whole launch (measured: two per SM streams no faster and
// doubles the merge), at most 64 chunks per program, each a whole number of 64-key tiles.  It follows the
// descriptor's unit count, never the unit range, so every range of a launch merges its keys in the same
// chunks.
struct DecodePlan {
  int chunks, chunk_keys;
};

static DecodePlan plan_decode(int64_t units, int64_t seq, int sm_count) {
  int64_t per = int64_t(sm_count) / (units > 0 ? units : 1);
  if (per < 1) per = 1;
  if (per > kDecMaxChunks) per = kDecMaxChunks;
  const int64_t keys = ceil_div(ceil_div(seq, per), kDecTile) * kDecTile;
  return DecodePlan{int(ceil_div(seq, keys)), int(keys)};
}

int64_t decode_workspace(const ptsim_desc &d, int sm_count) {
  const ptsim_attn_params &a = d.p.attn;
  if (a.hkv < 1 || a.seq < 1) return 0;
  const DecodePlan pl = plan_decode(d.units, a.seq, sm_count);
  return d.units * pl.chunks * (a.hq / a.hkv) * int64_t(kDecD + 2) * int64_t(sizeof(float));
}

int launch_decode(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                  const LaunchCtx &c) {
  const ptsim_attn_params &a = d.p.attn;
  for (int arg : {a.q_arg, a.k_arg, a.v_arg, a.o_arg})
    if (d.arg_dtype[arg] != PTSIM_DT_BF16) return fail(PTSIM_E_UNSUPPORTED, "decode attention runs bf16 tensors");
  const int64_t G = a.hq / a.hkv;
  if (a.dim != kDecD) return fail(PTSIM_E_UNSUPPORTED, "decode attention with head dim %lld (runs 128)", (long long)a.dim);
  if (G < 1 || G > kDecRows) return fail(PTSIM_E_UNSUPPORTED, "decode attention with %lld query rows per KV head (runs 1-16)", (long long)G);
  if (a.seq < kDecTile || a.seq % kDecTile != 0)
    return fail(PTSIM_E_UNSUPPORTED, "decode attention over %lld keys (runs multiples of %d)", (long long)a.seq, kDecTile);
  if (a.hkv * a.seq >= (int64_t(1) << 31)) return fail(PTSIM_E_UNSUPPORTED, "decode attention over more than 2^31 key rows");
  const DecodePlan pl = plan_decode(d.units, a.seq, c.sm_count);
  const int64_t units = hi - lo;
  const int64_t need_o = units * pl.chunks * G * kDecD * int64_t(sizeof(float));
  const int64_t need = need_o + units * pl.chunks * G * 2 * int64_t(sizeof(float));
  if (ws == nullptr || int64_t(ws_bytes) < need)
    return fail(PTSIM_E_RESOURCE, "decode attention needs %lld bytes of workspace, got %zu", (long long)need, ws_bytes);
  if (reinterpret_cast<uintptr_t>(ws) % 16 != 0) return fail(PTSIM_E_ARGS, "workspace is not 16-byte aligned");
  DecodeArgs g;
  memset(&g, 0, sizeof(g));
  int rc = make_tmap_2d(&g.tk, ptrs[a.k_arg], kDecD, uint64_t(a.hkv * a.seq), kDecD, 64, kDecTile);
  if (rc) return rc;
  rc = make_tmap_2d(&g.tv, ptrs[a.v_arg], kDecD, uint64_t(a.hkv * a.seq), kDecD, 64, kDecTile);
  if (rc) return rc;
  g.q = reinterpret_cast<const uint16_t *>(ptrs[a.q_arg]);
  g.o = reinterpret_cast<uint16_t *>(ptrs[a.o_arg]);
  g.part_o = reinterpret_cast<float *>(ws);
  g.part_ml = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ws) + need_o);
  g.unit_begin = lo;
  g.G = int(G);
  g.S = int(a.seq);
  g.chunks = pl.chunks;
  g.chunk_keys = pl.chunk_keys;
  g.scale = a.scale;
  g.stall = (d.flags & PTSIM_FLAG_TEST_STALL) ? 1 : 0;
  PTSIM_CUDA((smem_limit_once<decode_part_kernel>(kDecSmem, c.device)));
  decode_part_kernel<<<dim3(unsigned(pl.chunks), unsigned(units), 1), kDecThreads, kDecSmem, c.stream>>>(g);
  PTSIM_CUDA(cudaGetLastError());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(units), unsigned(G), 1);
  cfg.blockDim = dim3(kDecD, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = c.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PTSIM_CUDA(cudaLaunchKernelEx(&cfg, decode_combine_kernel, g));
  return PTSIM_OK;
}

}  // namespace ptsim
