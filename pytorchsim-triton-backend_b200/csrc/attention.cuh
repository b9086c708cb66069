// Causal GQA flash-attention forward on the tensor core: the attention_prefill_* / Qwen3 06 program of
// the validation bundle (validation/pytorchsim/attention_prefill_32x8x4096_bf16/00__prefill_kernel/
// _prefill_kernel_triton.py:3-44).  Per query row: m = -1e30, l = 0, acc = 0; per key block
// qk = (q . k^T) * SCALE in fp32 (masked to -1e30 above the diagonal), m' = max(m, rowmax qk),
// alpha = exp(m - m'), p = exp(qk - m'), l = l * alpha + rowsum p, acc = acc * alpha + bf16(p) . v;
// out = bf16(acc / l).  exp is 2^(x * log2 e) as the NPU's EUP computes it.
//
// One CTA per (batch, query head, 128-row query tile), heaviest (most key tiles) first.  Roles:
//   warp 0      TMA: the Q tile once, then K and V tiles of 128 keys into a two-deep ring;
//   warp 1      TMEM owner + MMA issuer: S_j = Q . K_j^T (M=128 N=128 K=128) into one of two TMEM S
//               buffers, then O += P_j . V_j (M=128 N=128 K=128) into the TMEM O accumulator; S_{j+1}
//               is issued before PV_j so the softmax of tile j+1 overlaps PV_j;
//   warps 2..5  softmax/correction: one query row per thread -- tcgen05.ld of S, row max / exp / row sum
//               in fp32 registers, P rounded to bf16 into 128B-swizzled shared memory, O rescaled in
//               TMEM by alpha (skipped when a whole warp has alpha == 1), finally O / l stored as bf16.
#pragma once
#include "sm100.cuh"
#include "gemm.cuh"
#include <initializer_list>

namespace ptsim {

constexpr int kAttnBM = 128;   // query rows per CTA
constexpr int kAttnBN = 128;   // keys per tile
constexpr int kAttnD = 128;    // head dim
constexpr int kAttnThreads = 192;
constexpr int kAttnTile = kAttnBM * kAttnD * 2;  // 32 KB: a [128 x 128] bf16 tile as two 16 KB swizzled halves
constexpr int kAttnSmem = 6 * kAttnTile + 1024 + 256;  // Q, K x2, V x2, P

struct AttnArgs {
  CUtensorMap tq, tk, tv;  // [rows, 128] bf16, box {64, 128}
  uint16_t *o;
  int64_t hq, hkv, seq;
  int32_t q_tiles, causal;
  int64_t unit_begin, unit_end;  // (batch, head) units of this launch
  float scale;
  // PTSIM_FLAG_TEST_STALL: CTA 0 arms its first K tile but issues none of its copies, and every wait
  // gives up after kTestWaitUs -- the timeout path under test.
  int32_t stall;
};

// Store 128 bf16 values of row r of a [128 x 128] K-major operand tile (two 64-column halves, each
// 128 rows x 128 B with the 128-byte swizzle: 16-byte unit u of row r lands at unit u ^ (r % 8)).
__device__ __forceinline__ void store_sw128_row(uint8_t *tile, int r, const uint32_t (&packed)[64]) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint8_t *base = tile + c * 16384 + r * 128;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int w = c * 32 + u * 4;
      *reinterpret_cast<uint4 *>(base + ((u ^ (r & 7)) << 4)) = make_uint4(packed[w], packed[w + 1], packed[w + 2], packed[w + 3]);
    }
  }
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__global__ void __launch_bounds__(kAttnThreads, 1) attn_fwd_kernel(const __grid_constant__ AttnArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sQ = smem;
  uint8_t *sK = smem + kAttnTile;       // 2 stages
  uint8_t *sV = smem + 3 * kAttnTile;   // 2 stages
  uint8_t *sP = smem + 5 * kAttnTile;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 6 * kAttnTile);
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1;    // 2
  uint64_t *v_full = bars + 3;    // 2
  uint64_t *kv_empty = bars + 5;  // 2
  uint64_t *s_full = bars + 7;    // 2
  uint64_t *p_full = bars + 9;
  uint64_t *pv_done = bars + 10;
  uint64_t *drain = bars + 11;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 12);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work item: heaviest query tiles first.
  const int64_t units = g.unit_end - g.unit_begin;
  const int64_t item = blockIdx.x;
  const int qt = g.q_tiles - 1 - int(item / units);
  const int64_t unit = g.unit_begin + item % units;  // b * hq + h
  const int64_t b = unit / g.hq, h = unit % g.hq;
  const int64_t kvh = b * g.hkv + h / (g.hq / g.hkv);
  const int q_row0 = int(unit * g.seq + int64_t(qt) * kAttnBM);
  const int kv_row0 = int(kvh * g.seq);
  const int nkv = g.causal ? qt + 1 : int(g.seq / kAttnBN);
  const uint32_t wl = g.stall ? kTestWaitUs : kWaitUs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 12; ++i) sm100::mbar_init(&bars[i], i == 9 ? 4u : 1u);  // p_full: one per softmax warp
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, 512);
    sm100::tmem_relinquish();
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS0 = tmem, tO = tmem + 256;  // S buffers at columns [0,128) and [128,256); O at [256,384)

  int issued = 0;   // (producer) K/V tiles whose stages were armed
  if (warp == 0) {
    if (lane == 0) {
      sm100::mbar_arrive_expect_tx(q_full, kAttnTile);
      sm100::tma_load_2d(sQ, &g.tq, q_full, 0, q_row0);
      sm100::tma_load_2d(sQ + 16384, &g.tq, q_full, 64, q_row0);
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        if (!sm100::mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, wl)) { *abort_flag = 1; break; }
        const int kr = kv_row0 + j * kAttnBN;
        sm100::mbar_arrive_expect_tx(&k_full[st], kAttnTile);
        sm100::mbar_arrive_expect_tx(&v_full[st], kAttnTile);
        ++issued;
        if (g.stall && blockIdx.x == 0 && j == 0) continue;   // test hook: stage armed, no copy in flight
        sm100::tma_load_2d(sK + st * kAttnTile, &g.tk, &k_full[st], 0, kr);
        sm100::tma_load_2d(sK + st * kAttnTile + 16384, &g.tk, &k_full[st], 64, kr);
        sm100::tma_load_2d(sV + st * kAttnTile, &g.tv, &v_full[st], 0, kr);
        sm100::tma_load_2d(sV + st * kAttnTile + 16384, &g.tv, &v_full[st], 64, kr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = sm100::idesc_bf16_f32(kAttnBM, kAttnBN, false, false);
      constexpr uint32_t idesc_o = sm100::idesc_bf16_f32(kAttnBM, kAttnD, false, true);
      const uint32_t q_addr = sm100::smem_u32(sQ), p_addr = sm100::smem_u32(sP);
      bool ok = sm100::mbar_wait(q_full, 0, wl);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!sm100::mbar_wait(&k_full[st], (j >> 1) & 1, wl)) return false;
        sm100::tc_fence_after();
        const uint32_t k_addr = sm100::smem_u32(sK + st * kAttnTile);
#pragma unroll
        for (int k = 0; k < kAttnD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          sm100::mma_bf16_ss(tS0 + st * 128, sm100::sw128_desc(q_addr + off, 16, 1024),
                             sm100::sw128_desc(k_addr + off, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
        }
        sm100::mma_commit(&s_full[st]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j & 1;
        if (!sm100::mbar_wait(p_full, j & 1, wl)) return false;
        if (!sm100::mbar_wait(&v_full[st], (j >> 1) & 1, wl)) return false;
        sm100::tc_fence_after();
        const uint32_t v_addr = sm100::smem_u32(sV + st * kAttnTile);
#pragma unroll
        for (int k = 0; k < kAttnBN / 16; ++k) {
          const uint32_t aoff = (k >> 2) * 16384 + (k & 3) * 32;
          sm100::mma_bf16_ss(tO, sm100::sw128_desc(p_addr + aoff, 16, 1024),
                             sm100::sw128_desc(v_addr + k * 16 * 128, 16384, 1024), idesc_o,
                             (j > 0 || k > 0) ? 1u : 0u);
        }
        sm100::mma_commit(pv_done);
        sm100::mma_commit(&kv_empty[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 1; ok && j < nkv; ++j) {
        ok = issue_s(j);
        if (ok) ok = issue_pv(j - 1);
      }
      if (ok) ok = issue_pv(nkv - 1);
      if (!ok) *abort_flag = 1;
      sm100::mma_commit(drain);
      sm100::mbar_wait(drain, 0, wl);
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const float sl2 = g.scale;
    const float kLog2e = 1.4426950408889634f;
    float m = -1.0e30f, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      if (*abort_flag || !sm100::mbar_wait(&s_full[st], (j >> 1) & 1, wl)) { ok = false; break; }
      sm100::tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        sm100::tmem_ld32(tS0 + st * 128 + lane_off + c * 32, v);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 32; ++q) s[c * 32 + q] = __fmul_rn(__uint_as_float(v[q]), sl2);
      }
      const bool diag = g.causal && j == qt;
      float mx = -INFINITY;
#pragma unroll
      for (int q = 0; q < 128; ++q) {
        if (diag && q > r) s[q] = -1.0e30f;
        mx = fmaxf(mx, s[q]);
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = exp2f(__fmul_rn(__fsub_rn(m, m_new), kLog2e));
      float rs = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int q = 0; q < 64; ++q) {
        const float p0 = exp2f(__fmul_rn(__fsub_rn(s[2 * q], m_new), kLog2e));
        const float p1 = exp2f(__fmul_rn(__fsub_rn(s[2 * q + 1], m_new), kLog2e));
        rs = __fadd_rn(__fadd_rn(rs, p0), p1);
        pk[q] = pack_bf16x2(p0, p1);
      }
      l = __fadd_rn(__fmul_rn(l, alpha), rs);
      m = m_new;
      if (j > 0) {
        // PV_{j-1} has finished: the P buffer is free and O holds every earlier tile.
        if (!sm100::mbar_wait(pv_done, (j - 1) & 1, wl)) { ok = false; break; }
        sm100::tc_fence_after();
      }
      store_sw128_row(sP, r, pk);
      fence_proxy_async_smem();
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          sm100::tmem_ld32(tO + lane_off + c * 32, v);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = __float_as_uint(__fmul_rn(__uint_as_float(v[q]), alpha));
          uint32_t lo16[16], hi16[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) { lo16[q] = v[q]; hi16[q] = v[16 + q]; }
          sm100::tmem_st16(tO + lane_off + c * 32, lo16);
          sm100::tmem_st16(tO + lane_off + c * 32 + 16, hi16);
        }
        sm100::tmem_wait_st();
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(p_full);
    }
    if (ok && !*abort_flag && sm100::mbar_wait(pv_done, (nkv - 1) & 1, wl)) {
      sm100::tc_fence_after();
      const float inv_l = l;  // divide, as the program does (acc / l)
      uint16_t *orow = g.o + (int64_t(q_row0) + r) * kAttnD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        sm100::tmem_ld32(tO + lane_off + c * 32, v);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 0]), inv_l), __fdiv_rn(__uint_as_float(v[q * 8 + 1]), inv_l));
          w.y = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 2]), inv_l), __fdiv_rn(__uint_as_float(v[q * 8 + 3]), inv_l));
          w.z = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 4]), inv_l), __fdiv_rn(__uint_as_float(v[q * 8 + 5]), inv_l));
          w.w = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 6]), inv_l), __fdiv_rn(__uint_as_float(v[q * 8 + 7]), inv_l));
          reinterpret_cast<uint4 *>(orow + c * 32)[q] = w;
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  // After an abort (final at the barrier above) the producer waits, bounded, for Q and the last fill of
  // each K/V stage, so no copy still lands in shared memory once the CTA has exited.
  if (warp == 0 && lane == 0 && *abort_flag) {
    sm100::mbar_wait(q_full, 0, wl);
    for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
      sm100::mbar_wait(&k_full[j & 1], (j >> 1) & 1, wl);
      sm100::mbar_wait(&v_full[j & 1], (j >> 1) & 1, wl);
    }
  }
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------------
// Version 2 (sequence a multiple of 256): two 128-row query tiles A and B per CTA share each K/V tile.
//   warp 0      TMA: Q_A, Q_B once; K_j, V_j into a two-deep ring;
//   warp 1      MMA: S_A(j) = Q_A.K_j^T, S_B(j) = Q_B.K_j^T into TMEM; then O_A += P_A(j).V_j and
//               O_B += P_B(j).V_j with P read from TMEM (the A operand of a TMEM-sourced MMA);
//   warps 2, 3  idle (they complete the first warpgroup, whose registers go to the softmax);
//   warps 4..7  softmax of tile A, warps 8..11 softmax of tile B (one query row per thread): the row's
//               128 scores are read from TMEM once, P is written back as packed bf16 pairs over the
//               consumed S columns, O is rescaled in TMEM when the row max moved, and at the end O / l is
//               stored.
// The two softmax warpgroups alternate with the tensor core: the MMA warp issues PV_A(j) and S_A(j+1)
// as soon as P_A(j) is ready, then PV_B(j) and S_B(j+1), so while one tile's softmax computes exp the
// tensor core runs the other tile's products.  In-order MMA execution makes S_X(j)'s commit imply
// PV_X(j-1) has finished, so a softmax may rescale O_X and overwrite P_X as soon as S_X(j) is ready.
// TMEM: S_A [0,128)  S_B [128,256)  O_A [256,384)  O_B [384,512).
// ---------------------------------------------------------------------------------------------------
// Three warpgroups: TMA + MMA (+ two idle warps), the softmax of tile A, the softmax of tile B.  Launched
// at 168 registers a thread (12 warps, three on each SMSP), setmaxnreg then moves registers from the first
// warpgroup to the other two: 128 x 56 + 256 x 224 = 64,512, exactly the 384 x 168 the launch holds (a split
// above it would wait forever; the launcher checks the build's count), and 56 + 224 + 224 = 504 <= 512 per
// SMSP.  The softmax holds a row's 128 scores in registers with room to keep many exponentials in flight.
constexpr int kAttn2Threads = 384;
constexpr int kAttn2SoftmaxWarp0 = 4;
constexpr int kAttn2ProducerRegs = 56, kAttn2SoftmaxRegs = 224;
static_assert(128 * kAttn2ProducerRegs + 256 * kAttn2SoftmaxRegs <= kAttn2Threads * 168,
              "register split above the launch's registers");
constexpr int kAttn2Smem = 6 * kAttnTile + 1024 + 256;  // Q_A, Q_B, K x2, V x2

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  sm100::tmem_st16(taddr, *reinterpret_cast<const uint32_t(*)[16]>(&r[0]));
  sm100::tmem_st16(taddr + 16, *reinterpret_cast<const uint32_t(*)[16]>(&r[16]));
}

__global__ void __launch_bounds__(kAttn2Threads, 1) attn2_fwd_kernel(const __grid_constant__ AttnArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sQ = smem;                   // Q_A, Q_B
  uint8_t *sK = smem + 2 * kAttnTile;   // 2 stages
  uint8_t *sV = smem + 4 * kAttnTile;   // 2 stages
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 6 * kAttnTile);
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1;    // 2
  uint64_t *v_full = bars + 3;    // 2
  uint64_t *k_empty = bars + 5;   // 2: K_j read by S_A(j) and S_B(j)
  uint64_t *s_full = bars + 7;    // [A, B]
  uint64_t *p_full = bars + 9;    // [A, B], 4 arrivals each
  uint64_t *o_done = bars + 11;   // [A, B]
  uint64_t *drain = bars + 13;
  uint64_t *v_empty = bars + 14;  // 2: V_j read by PV_A(j) and PV_B(j)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 16);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t units = g.unit_end - g.unit_begin;
  const int pairs = g.q_tiles / 2;
  const int qp = pairs - 1 - int(int64_t(blockIdx.x) / units);   // heaviest query-tile pairs first
  const int64_t unit = g.unit_begin + int64_t(blockIdx.x) % units;
  const int64_t b = unit / g.hq, h = unit % g.hq;
  const int64_t kvh = b * g.hkv + h / (g.hq / g.hkv);
  const int q_row0 = int(unit * g.seq + int64_t(qp) * 2 * kAttnBM);
  const int kv_row0 = int(kvh * g.seq);
  const int nA = g.causal ? 2 * qp + 1 : int(g.seq / kAttnBN);   // key tiles of query tile A
  const int nB = g.causal ? 2 * qp + 2 : nA;                      // and of tile B
  const uint32_t wl = g.stall ? kTestWaitUs : kWaitUs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 16; ++i) sm100::mbar_init(&bars[i], (i == 9 || i == 10) ? 4u : 1u);
    *abort_flag = 0;
    sm100::fence_barrier_init();
  }
  if (warp == 1) {
    sm100::tmem_alloc(tmem_slot, 512);
    sm100::tmem_relinquish();
  }
  pdl_enter();   // set-up above overlaps the previous kernel's tail; global memory after
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int kj = 0, vj = 0;   // (producer) K and V tiles whose stages were armed
  if (warp < kAttn2SoftmaxWarp0) {
  // Producer warpgroup: every warp of it gives its registers back at this one instruction.
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAttn2ProducerRegs));
  if (warp == 0) {
    if (lane == 0) {
      sm100::mbar_arrive_expect_tx(q_full, 2 * kAttnTile);
      sm100::tma_load_2d(sQ, &g.tq, q_full, 0, q_row0);
      sm100::tma_load_2d(sQ + 16384, &g.tq, q_full, 64, q_row0);
      sm100::tma_load_2d(sQ + kAttnTile, &g.tq, q_full, 0, q_row0 + kAttnBM);
      sm100::tma_load_2d(sQ + kAttnTile + 16384, &g.tq, q_full, 64, q_row0 + kAttnBM);
      // K and V slots are released separately (K after the S products, V after the PV products), so
      // K_{j+2} starts loading about half an iteration before V_{j+2} may.
      for (int j = 0; j < nB; ++j) {
        const int st = j & 1;
        const int kr = kv_row0 + j * kAttnBN;
        if (!sm100::mbar_wait(&k_empty[st], ((j >> 1) & 1) ^ 1, wl)) { *abort_flag = 1; break; }
        sm100::mbar_arrive_expect_tx(&k_full[st], kAttnTile);
        if (!(g.stall && blockIdx.x == 0 && j == 0)) {   // test hook: K_0 armed, no copy in flight
          sm100::tma_load_2d(sK + st * kAttnTile, &g.tk, &k_full[st], 0, kr);
          sm100::tma_load_2d(sK + st * kAttnTile + 16384, &g.tk, &k_full[st], 64, kr);
        }
        ++kj;
        if (!sm100::mbar_wait(&v_empty[st], ((j >> 1) & 1) ^ 1, wl)) { *abort_flag = 1; break; }
        sm100::mbar_arrive_expect_tx(&v_full[st], kAttnTile);
        sm100::tma_load_2d(sV + st * kAttnTile, &g.tv, &v_full[st], 0, kr);
        sm100::tma_load_2d(sV + st * kAttnTile + 16384, &g.tv, &v_full[st], 64, kr);
        ++vj;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = sm100::idesc_bf16_f32(kAttnBM, kAttnBN, false, false);
      constexpr uint32_t idesc_o = sm100::idesc_bf16_f32(kAttnBM, kAttnD, false, true);
      // Issue order (tiles ping-pong): S_A(0) S_B(0) | PV_A(0) S_A(1) | PV_B(0) S_B(1) | PV_A(1) S_A(2) | ...
      // so the tensor core runs one tile's products while the other tile's softmax computes.  S_X(j+1)
      // overwrites P_X(j) in TMEM only after PV_X(j), issued before it, has read it (in-order execution).
      auto issue_s = [&](int t, int j) {
        const uint32_t k_addr = sm100::smem_u32(sK + (j & 1) * kAttnTile);
        const uint32_t q_addr = sm100::smem_u32(sQ + t * kAttnTile);
#pragma unroll
        for (int k = 0; k < kAttnD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          sm100::mma_bf16_ss(tmem + t * 128, sm100::sw128_desc(q_addr + off, 16, 1024),
                             sm100::sw128_desc(k_addr + off, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
        }
        sm100::mma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t v_addr = sm100::smem_u32(sV + (j & 1) * kAttnTile);
#pragma unroll
        for (int k = 0; k < kAttnBN / 16; ++k)
          sm100::mma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + k * 8,
                             sm100::sw128_desc(v_addr + k * 16 * 128, 16384, 1024), idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        if (j == (t == 0 ? nA : nB) - 1) sm100::mma_commit(&o_done[t]);
      };
      bool ok = sm100::mbar_wait(q_full, 0, wl) && sm100::mbar_wait(&k_full[0], 0, wl);
      if (ok) {
        sm100::tc_fence_after();
        if (nA > 0) issue_s(0, 0);
        issue_s(1, 0);
        sm100::mma_commit(&k_empty[0]);   // K_0 is read once S_A(0) and S_B(0) are done
      }
      for (int j = 0; ok && j < nB; ++j) {
        const int st = j & 1;
        const bool next = j + 1 < nB;
        if (!sm100::mbar_wait(&v_full[st], (j >> 1) & 1, wl)) { ok = false; break; }
        if (j < nA) {
          if (!sm100::mbar_wait(&p_full[0], j & 1, wl)) { ok = false; break; }
          sm100::tc_fence_after();
          issue_pv(0, j);
          if (j + 1 < nA) {
            if (!sm100::mbar_wait(&k_full[st ^ 1], ((j + 1) >> 1) & 1, wl)) { ok = false; break; }
            sm100::tc_fence_after();
            issue_s(0, j + 1);
          }
        }
        if (!sm100::mbar_wait(&p_full[1], j & 1, wl)) { ok = false; break; }
        sm100::tc_fence_after();
        issue_pv(1, j);
        sm100::mma_commit(&v_empty[st]);    // V_j is read once PV_B(j) is done
        if (next) {
          if (!sm100::mbar_wait(&k_full[st ^ 1], ((j + 1) >> 1) & 1, wl)) { ok = false; break; }
          sm100::tc_fence_after();
          issue_s(1, j + 1);
          sm100::mma_commit(&k_empty[st ^ 1]);   // K_{j+1} is read once S_B(j+1) is done
        }
      }
      if (!ok) *abort_flag = 1;
      sm100::mma_commit(drain);
      sm100::mbar_wait(drain, 0, wl);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kAttn2SoftmaxRegs));
    const int t = (warp - kAttn2SoftmaxWarp0) >> 2;   // 0: tile A, 1: tile B
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;       // query row within the tile = TMEM lane
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_off, tO = tmem + 256 + t * 128 + lane_off;
    const int ntiles = t == 0 ? nA : nB;
    const int diag = t == 0 ? 2 * qp : 2 * qp + 1;   // the key tile holding this query tile's diagonal
    const float kLog2e = 1.4426950408889634f;
    const float sc = g.scale, sl = g.scale * kLog2e;
    float m = -1.0e30f, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (*abort_flag || !sm100::mbar_wait(&s_full[t], j & 1, wl)) { ok = false; break; }
      sm100::tc_fence_after();
      // The row's 128 products, read from TMEM once.  On the diagonal tile, keys past the query row become
      // -inf: they never win the max and their exp is 0, as the reference's -1e30 fill gives.
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) sm100::tmem_ld32(tS + c * 32, v[c]);
      sm100::tmem_wait_ld();
      if (g.causal && j == diag) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int q = 0; q < 32; ++q)
            if (c * 32 + q > r) v[c][q] = 0xff800000u;
      }
      // Row max (scale > 0 keeps the arg max), eight independent chains.
      float mx8[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) mx8[q] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int q = 0; q < 32; ++q) mx8[q & 7] = fmaxf(mx8[q & 7], __uint_as_float(v[c][q]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // Lazy rescaling: the row keeps its reference max m until the tile's max exceeds it by more than
      // 2^8 (8 in log2 units), so p <= 256 and O is rescaled only when the reference moves.  O / l is
      // unchanged (numerator and denominator share the reference); only P's bf16 rounding point moves.
      const float m_cand = fmaxf(m, __fmul_rn(mx, sc));
      const bool grow = __fmul_rn(__fsub_rn(m_cand, m), kLog2e) > 8.0f;
      float alpha = 1.0f;
      if (grow) {
        alpha = ex2_fast(__fmul_rn(__fsub_rn(m, m_cand), kLog2e));
        m = m_cand;
      }
      const float2 a2 = make_float2(sl, sl), b2 = make_float2(-m * kLog2e, -m * kLog2e);
      // p = exp(qk - m'): row sum over four chains, bf16 P packed over the consumed S columns.
      float2 acc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float2 u = __ffma2_rn(make_float2(__uint_as_float(v[c][2 * q]), __uint_as_float(v[c][2 * q + 1])), a2, b2);
          const float p0 = ex2_fast(u.x), p1 = ex2_fast(u.y);
          acc[q & 3] = __fadd2_rn(acc[q & 3], make_float2(p0, p1));
          pk[q] = pack_bf16x2(p0, p1);
        }
        sm100::tmem_st16(tS + c * 16, pk);
      }
      const float2 s2 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
      l = __fadd_rn(__fmul_rn(l, alpha), __fadd_rn(s2.x, s2.y));
      // O rescale (O already holds PV_X(j-1): S_X(j) was issued after it); lanes that kept their
      // reference multiply by 1.
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        const float2 al2 = make_float2(alpha, alpha);
        uint32_t o[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) sm100::tmem_ld32(tO + c * 32, o[c]);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float2 x = __fmul2_rn(make_float2(__uint_as_float(o[c][2 * q]), __uint_as_float(o[c][2 * q + 1])), al2);
            o[c][2 * q] = __float_as_uint(x.x);
            o[c][2 * q + 1] = __float_as_uint(x.y);
          }
          tmem_st32(tO + c * 32, o[c]);
        }
      }
      sm100::tmem_wait_st();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&p_full[t]);
    }
    if (ok && !*abort_flag && sm100::mbar_wait(&o_done[t], 0, wl)) {
      sm100::tc_fence_after();
      uint16_t *orow = g.o + (int64_t(q_row0) + t * kAttnBM + r) * kAttnD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        sm100::tmem_ld32(tO + c * 32, v);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 0]), l), __fdiv_rn(__uint_as_float(v[q * 8 + 1]), l));
          w.y = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 2]), l), __fdiv_rn(__uint_as_float(v[q * 8 + 3]), l));
          w.z = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 4]), l), __fdiv_rn(__uint_as_float(v[q * 8 + 5]), l));
          w.w = pack_bf16x2(__fdiv_rn(__uint_as_float(v[q * 8 + 6]), l), __fdiv_rn(__uint_as_float(v[q * 8 + 7]), l));
          reinterpret_cast<uint4 *>(orow + c * 32)[q] = w;
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  // After an abort (final at the barrier above) the producer waits, bounded, for Q and the last fill of
  // each K and V stage, so no copy still lands in shared memory once the CTA has exited.
  if (warp == 0 && lane == 0 && *abort_flag) {
    sm100::mbar_wait(q_full, 0, wl);
    for (int i = (kj - 2 < 0 ? 0 : kj - 2); i < kj; ++i) sm100::mbar_wait(&k_full[i & 1], (i >> 1) & 1, wl);
    for (int i = (vj - 2 < 0 ? 0 : vj - 2); i < vj; ++i) sm100::mbar_wait(&v_full[i & 1], (i >> 1) & 1, wl);
  }
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

int launch_attention(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c) {
  const ptsim_attn_params &a = d.p.attn;
  if (a.dim != kAttnD) return fail(PTSIM_E_UNSUPPORTED, "attention runs head_dim 128, not %lld", (long long)a.dim);
  if (a.seq % kAttnBM != 0) return fail(PTSIM_E_UNSUPPORTED, "attention sequence %lld is not a multiple of 128", (long long)a.seq);
  for (int t : {a.q_arg, a.k_arg, a.v_arg, a.o_arg})
    if (d.arg_dtype[t] != PTSIM_DT_BF16) return fail(PTSIM_E_UNSUPPORTED, "attention tensors must be bf16");
  // Units are (batch, query head) pairs.
  const int64_t u0 = lo * d.unit_size, u1 = hi * d.unit_size < a.batch * a.hq ? hi * d.unit_size : a.batch * a.hq;
  if (u1 <= u0) return PTSIM_OK;
  AttnArgs g;
  memset(&g, 0, sizeof(g));
  int rc;
  if ((rc = make_tmap_2d(&g.tq, ptrs[a.q_arg], 128, uint64_t(a.batch * a.hq * a.seq), 128, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&g.tk, ptrs[a.k_arg], 128, uint64_t(a.batch * a.hkv * a.seq), 128, 64, 128))) return rc;
  if ((rc = make_tmap_2d(&g.tv, ptrs[a.v_arg], 128, uint64_t(a.batch * a.hkv * a.seq), 128, 64, 128))) return rc;
  g.o = reinterpret_cast<uint16_t *>(ptrs[a.o_arg]);
  g.hq = a.hq;
  g.hkv = a.hkv;
  g.seq = a.seq;
  g.q_tiles = int(a.seq / kAttnBM);
  g.causal = a.causal;
  g.unit_begin = u0;
  g.unit_end = u1;
  g.scale = a.scale;
  g.stall = (d.flags & PTSIM_FLAG_TEST_STALL) ? 1 : 0;
  if (int64_t(a.batch * a.hkv * a.seq) >= (int64_t(1) << 31)) return fail(PTSIM_E_UNSUPPORTED, "attention rows exceed int32");
  if (a.seq % (2 * kAttnBM) == 0) {
    PTSIM_CUDA(smem_limit_once<attn2_fwd_kernel>(kAttn2Smem, c.device));
    {
      // setmaxnreg.inc waits until the registers it asks for are free, so the warpgroups' shares must fit
      // the registers the block is launched with; refuse (rather than wait forever) if the build disagrees.
      static std::atomic<int> regs_ok{0};   // 0 unknown, 1 fits, 2 does not
      if (regs_ok.load() == 0) {
        cudaFuncAttributes fa;
        PTSIM_CUDA(cudaFuncGetAttributes(&fa, attn2_fwd_kernel));
        regs_ok.store(int64_t(fa.numRegs) * kAttn2Threads >= 128 * kAttn2ProducerRegs + 256 * kAttn2SoftmaxRegs ? 1 : 2);
      }
      if (regs_ok.load() != 1) return fail(PTSIM_E_RESOURCE, "attention register split does not fit this build's registers");
    }
    const int64_t grid = (u1 - u0) * (g.q_tiles / 2);
    PTSIM_CUDA(launch_pdl(attn2_fwd_kernel, dim3(unsigned(grid)), dim3(kAttn2Threads), kAttn2Smem, c.stream, g));
    return PTSIM_OK;
  }
  PTSIM_CUDA(smem_limit_once<attn_fwd_kernel>(kAttnSmem, c.device));
  const int64_t grid = (u1 - u0) * g.q_tiles;
  attn_fwd_kernel<<<unsigned(grid), kAttnThreads, kAttnSmem, c.stream>>>(g);
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

}  // namespace ptsim
