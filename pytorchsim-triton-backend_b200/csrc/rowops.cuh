// Row programs of the vector unit: softmax and RMSNorm over rows (the validation bundle's
// vector_softmax_* kernels, e.g. validation/pytorchsim/vector_softmax_4096x4096_bf16/00_*/..._triton.py:17-68,
// and the Qwen3 layer's RMSNorm qwen3_8b_layer_prefill_2048x2048_bf16/00_*/..._triton.py), the per-head
// QK-RMSNorm + rotary embedding (02_*/04_*), and whole-tensor sum/max (vector_sum_*, vector_max_*).
//
// On the NPU a program loads XBLOCK rows into the scratchpad, reduces each row across lanes on the XLU
// (PyTorchSimOps.td:124-136, PyTorchSimTpuOps.td:135-144) and applies the vector ops.  On the B200 a row
// is owned by TPR threads (a half warp, a warp or two warps); each thread keeps CH 16-byte chunks of the
// row in registers, so the row is read from HBM exactly once and written once; the cross-lane
// reductions are warp shuffles (plus one shared-memory exchange when a row spans two warps).
// Accumulation is fp32, as the programs' .to(tl.float32) casts state; the store rounds to the output
// dtype (RNE).
#pragma once
#include "common.cuh"
#include "sm100.cuh"
#include "vprog.cuh"

namespace ptsim {

enum RowKind { kSoftmax = 0, kRmsNorm = 1, kDivSum = 2, kRowSum = 3 };

struct RowLaunch {
  const void *in;
  const void *res;     // RMSNorm: a residual row added to the input (same stride and type), or null
  void *out;
  const void *weight;
  int64_t rows_begin, rows_end, cols, in_stride, out_stride;
  int64_t rows_total;  // rows of the whole launch: the kernel choice depends on it, never on [lo, hi)
  int32_t in_dt, out_dt, w_dt, pad;
  float eps;
};

template <int TPR>
__device__ __forceinline__ float row_allreduce(float v, bool is_max, float *smem_slot) {
  // Butterfly within the row's lanes (TPR <= 32), then across the row's warps through shared memory
  // (smem_slot: TPR / 32 floats owned by this row).  Every thread of the CTA must call it.
#pragma unroll
  for (int o = (TPR < 32 ? TPR : 32) / 2; o > 0; o >>= 1) {
    float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? nan_max(v, w) : __fadd_rn(v, w);
  }
  if constexpr (TPR > 32) {
    constexpr int W = TPR / 32;
    const int lane = threadIdx.x & 31;
    const int warp_in_row = (threadIdx.x % TPR) / 32;
    if (lane == 0) smem_slot[warp_in_row] = v;
    __syncthreads();
    float t = smem_slot[0];
#pragma unroll
    for (int w2 = 1; w2 < W; ++w2) t = is_max ? nan_max(t, smem_slot[w2]) : __fadd_rn(t, smem_slot[w2]);
    v = t;
  }
  return v;
}

// a / b with the reciprocal r = 1/b computed once per row: q = a*r, then one residual correction
// q' = q + (a - q*b) * r (Markstein's refinement of a reciprocal-based quotient), which returns the
// correctly rounded quotient for all but rare boundary cases at a fraction of the cost of a full division.
__device__ __forceinline__ float div_by(float a, float b, float r) {
  const float q = __fmul_rn(a, r);
  const float e = __fmaf_rn(-q, b, a);
  return __fmaf_rn(e, r, q);
}

// Fast path: bf16 rows whose length is TPR * 8 * CH.  A CTA of 256 threads owns 256 / TPR rows; each
// thread keeps CH 16-byte chunks of its row (8 * CH values) in registers: one HBM read, one write.
template <int KIND, int TPR, int CH>
__global__ void __launch_bounds__(256) row_fast_kernel(const __grid_constant__ RowLaunch L) {
  constexpr int RPC = 256 / TPR;                 // rows per CTA
  constexpr int W = TPR >= 32 ? TPR / 32 : 1;    // warps per row
  __shared__ float red_a[RPC * W], red_b[RPC * W];
  pdl_enter();
  const int lane_in_row = threadIdx.x % TPR;
  const int row_in_cta = threadIdx.x / TPR;
  const int64_t r = L.rows_begin + int64_t(blockIdx.x) * RPC + row_in_cta;
  const bool live = r < L.rows_end;
  float v[CH * 8];
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(L.in) + (live ? r : L.rows_begin) * L.in_stride);
    uint4 raw[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) raw[c] = live ? __ldcs(src + c * TPR + lane_in_row) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint32_t w[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) { v[c * 8 + 2 * j] = lo_bf16(w[j]); v[c * 8 + 2 * j + 1] = hi_bf16(w[j]); }
    }
    if (KIND == kRmsNorm && L.res != nullptr) {   // the row normalised is in + res, in fp32
      const uint4 *rsrc = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(L.res) + (live ? r : L.rows_begin) * L.in_stride);
#pragma unroll
      for (int c = 0; c < CH; ++c) raw[c] = live ? __ldcs(rsrc + c * TPR + lane_in_row) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const uint32_t w[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[c * 8 + 2 * j] = __fadd_rn(v[c * 8 + 2 * j], lo_bf16(w[j]));
          v[c * 8 + 2 * j + 1] = __fadd_rn(v[c * 8 + 2 * j + 1], hi_bf16(w[j]));
        }
      }
    }
  }
  uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(L.out) + (live ? r : L.rows_begin) * L.out_stride);
  if constexpr (KIND == kSoftmax) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < CH * 8; ++i) m = nan_max(m, v[i]);
    m = row_allreduce<TPR>(m, true, red_a + row_in_cta * W);
    const float kLog2e = 1.4426950408889634f;
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < CH * 8; ++i) {
      v[i] = ex2_fast(__fmul_rn(__fsub_rn(v[i], m), kLog2e));   // exp(x - m), once per element
      sum = __fadd_rn(sum, v[i]);
    }
    sum = row_allreduce<TPR>(sum, false, red_b + row_in_cta * W);
    const float rcp = __frcp_rn(sum);
    if (live) {
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          w[j] = pack_bf16x2(div_by(v[c * 8 + 2 * j], sum, rcp), div_by(v[c * 8 + 2 * j + 1], sum, rcp));
        __stcs(dst + c * TPR + lane_in_row, make_uint4(w[0], w[1], w[2], w[3]));
      }
    }
  } else {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < CH * 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    ss = row_allreduce<TPR>(ss, false, red_a + row_in_cta * W);
    const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, float(L.cols)), L.eps));
    if (live) {
      const uint4 *wsrc = reinterpret_cast<const uint4 *>(L.weight);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const uint4 wv = __ldg(wsrc + c * TPR + lane_in_row);
        const uint32_t g[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = pack_bf16x2(__fmul_rn(__fmul_rn(v[c * 8 + 2 * j], rs), lo_bf16(g[j])),
                             __fmul_rn(__fmul_rn(v[c * 8 + 2 * j + 1], rs), hi_bf16(g[j])));
        __stcs(dst + c * TPR + lane_in_row, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// Row-per-CTA path (bf16 rows of cols = 8 * CH * TPR, TPR in 64..512): CTA b owns row rows_begin + b;
// its TPR threads each load CH 16-byte chunks (chunk c * TPR + tid: every warp access is one contiguous
// 512-byte run) into registers with one streaming load each, reduce across the CTA (warp shuffles, then
// one shared-memory slot per warp), and store the row back with 16-byte streaming stores.  Launched with
// one CTA per row and sized for full occupancy (2048 threads per SM, <= 32 registers each; 1024 threads
// with 32 values a thread), so every SM keeps 64 KB of loads in flight and the scheduler backfills rows
// as CTAs finish.  Arithmetic
// runs on packed pairs (fp32 x2 FMA/ADD/MUL, bf16 x2 max); the softmax evaluates each exp once.
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t w) { return make_float2(lo_bf16(w), hi_bf16(w)); }

template <int KIND, int TPR, int CH>
__global__ void __launch_bounds__(TPR, (CH >= 4 ? 1024 : 2048) / TPR) row_cta_kernel(const __grid_constant__ RowLaunch L) {
  constexpr int NW = TPR / 32;
  __shared__ float red[2][NW];
  pdl_enter();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = L.rows_begin + blockIdx.x;
  const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(L.in) + row * L.in_stride);
  uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(L.out) + row * L.out_stride);
  uint32_t w[CH * 4];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const uint4 v = __ldcs(src + c * TPR + tid);
    w[c * 4 + 0] = v.x;
    w[c * 4 + 1] = v.y;
    w[c * 4 + 2] = v.z;
    w[c * 4 + 3] = v.w;
  }
  if constexpr (KIND == kSoftmax) {
    // Row max on packed bf16 pairs (NaN-propagating; exact, as max only selects).
    __nv_bfloat162 m2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) m2[j] = *reinterpret_cast<const __nv_bfloat162 *>(&w[j]);
#pragma unroll
    for (int i = 4; i < CH * 4; ++i) m2[i & 3] = __hmax2_nan(m2[i & 3], *reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
    m2[0] = __hmax2_nan(__hmax2_nan(m2[0], m2[1]), __hmax2_nan(m2[2], m2[3]));
    float m = nan_max(__low2float(m2[0]), __high2float(m2[0]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[0][warp] = m;
    __syncthreads();
    m = red[0][0];
#pragma unroll
    for (int i = 1; i < NW; ++i) m = nan_max(m, red[0][i]);
    // exp(x - m) = 2^((x - m) * log2 e), each evaluated once and kept for the division.
    const float2 negm = make_float2(-m, -m), l2e = make_float2(1.4426950408889634f, 1.4426950408889634f);
    float2 e[CH * 4];
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < CH * 4; ++i) {
      const float2 t = __fmul2_rn(__fadd2_rn(unpack_bf16x2(w[i]), negm), l2e);
      e[i] = make_float2(ex2_fast(t.x), ex2_fast(t.y));
      if (i & 1) acc1 = __fadd2_rn(acc1, e[i]);
      else acc0 = __fadd2_rn(acc0, e[i]);
    }
    acc0 = __fadd2_rn(acc0, acc1);
    float sum = __fadd_rn(acc0.x, acc0.y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    if (lane == 0) red[1][warp] = sum;
    __syncthreads();
    sum = red[1][0];
#pragma unroll
    for (int i = 1; i < NW; ++i) sum = __fadd_rn(sum, red[1][i]);
    // e / sum: reciprocal product plus one residual correction (div_by), on pairs.
    const float r = __frcp_rn(sum);
    const float2 r2 = make_float2(r, r), nsum2 = make_float2(-sum, -sum);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 q0 = __fmul2_rn(e[c * 4 + j], r2);
        const float2 q1 = __ffma2_rn(__ffma2_rn(q0, nsum2, e[c * 4 + j]), r2, q0);
        o[j] = pack_bf16x2(q1.x, q1.y);
      }
      __stcs(dst + c * TPR + tid, make_uint4(o[0], o[1], o[2], o[3]));
    }
  } else {
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < CH * 4; ++i) {
      const float2 x = unpack_bf16x2(w[i]);
      if (i & 1) acc1 = __fadd2_rn(acc1, __fmul2_rn(x, x));
      else acc0 = __fadd2_rn(acc0, __fmul2_rn(x, x));
    }
    acc0 = __fadd2_rn(acc0, acc1);
    float ss = __fadd_rn(acc0.x, acc0.y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) red[0][warp] = ss;
    __syncthreads();
    ss = red[0][0];
#pragma unroll
    for (int i = 1; i < NW; ++i) ss = __fadd_rn(ss, red[0][i]);
    const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, float(L.cols)), L.eps));
    const float2 rs2 = make_float2(rs, rs);
    const uint4 *wsrc = reinterpret_cast<const uint4 *>(L.weight);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint4 g = __ldg(wsrc + c * TPR + tid);
      const uint32_t gs[4] = {g.x, g.y, g.z, g.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 y = __fmul2_rn(__fmul2_rn(unpack_bf16x2(w[c * 4 + j]), rs2), unpack_bf16x2(gs[j]));
        o[j] = pack_bf16x2(y.x, y.y);
      }
      __stcs(dst + c * TPR + tid, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

template <int KIND, int TPR, int CH>
static int launch_row_cta(const RowLaunch &L, const LaunchCtx &c) {
  const int64_t rows = L.rows_end - L.rows_begin;
  if (rows > int64_t(0x7fffffff)) return fail(PTSIM_E_UNSUPPORTED, "%lld rows in one launch", (long long)rows);
  PTSIM_CUDA(launch_pdl(row_cta_kernel<KIND, TPR, CH>, dim3(unsigned(rows)), dim3(TPR), 0, c.stream, L));
  return PTSIM_OK;
}

// The (threads per row, chunks per thread) of the row-per-CTA path for `cols`: 16 values a thread where
// the thread count allows, else 32, else 8; 0 when no shape fits.
template <int KIND>
static int dispatch_row_cta(const RowLaunch &L, const LaunchCtx &c, bool *done) {
  *done = true;
  switch (L.cols) {
    case 1024: return launch_row_cta<KIND, 64, 2>(L, c);
    case 2048: return launch_row_cta<KIND, 128, 2>(L, c);
    case 4096: return launch_row_cta<KIND, 256, 2>(L, c);
    case 8192: return launch_row_cta<KIND, 512, 2>(L, c);
    case 16384: return launch_row_cta<KIND, 512, 4>(L, c);
    case 512: return launch_row_cta<KIND, 64, 1>(L, c);
  }
  *done = false;
  return PTSIM_OK;
}

__device__ __forceinline__ float ld_any(const void *p, int dt, int64_t i) {
  switch (dt) {
    case PTSIM_DT_F32: return reinterpret_cast<const float *>(p)[i];
    case PTSIM_DT_BF16: return bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(p)[i]);
    case PTSIM_DT_F16: return __half2float(reinterpret_cast<const __half *>(p)[i]);
  }
  return 0.f;
}
__device__ __forceinline__ void st_any(void *p, int dt, int64_t i, float v) {
  switch (dt) {
    case PTSIM_DT_F32: reinterpret_cast<float *>(p)[i] = v; break;
    case PTSIM_DT_BF16: reinterpret_cast<uint16_t *>(p)[i] = f32_to_bf16_bits(v); break;
    case PTSIM_DT_F16: reinterpret_cast<__half *>(p)[i] = __float2half_rn(v); break;
  }
}

// General path: any row length and float dtype; one warp per row, three passes over the row (the later
// passes hit L1/L2).
template <int KIND>
__global__ void __launch_bounds__(256) row_generic_kernel(const __grid_constant__ RowLaunch L) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = L.rows_begin + warp; r < L.rows_end; r += nwarps) {
    const int64_t ib = r * L.in_stride, ob = r * L.out_stride;
    if constexpr (KIND == kSoftmax) {
      float m = -INFINITY;
      for (int64_t c = lane; c < L.cols; c += 32) m = nan_max(m, ld_any(L.in, L.in_dt, ib + c));
      m = row_allreduce<32>(m, true, nullptr);
      float s = 0.f;
      for (int64_t c = lane; c < L.cols; c += 32) s = __fadd_rn(s, npu_exp(__fsub_rn(ld_any(L.in, L.in_dt, ib + c), m)));
      s = row_allreduce<32>(s, false, nullptr);
      for (int64_t c = lane; c < L.cols; c += 32)
        st_any(L.out, L.out_dt, ob + c, __fdiv_rn(npu_exp(__fsub_rn(ld_any(L.in, L.in_dt, ib + c), m)), s));
    } else if constexpr (KIND == kRowSum) {
      // sum(x) per row in fp32 (layer_layer_prefill_*/22_*: the top-k weight sums), stored at the row
      float s = 0.f;
      for (int64_t c = lane; c < L.cols; c += 32) s = __fadd_rn(s, ld_any(L.in, L.in_dt, ib + c));
      s = row_allreduce<32>(s, false, nullptr);
      if (lane == 0) st_any(L.out, L.out_dt, r * L.out_stride, s);
    } else if constexpr (KIND == kDivSum) {
      // x / sum(x) per row (layer_op_router_post_*/02_*: tmp4 = sum(x); x / tmp4 in fp32, cast on the store)
      float s = 0.f;
      for (int64_t c = lane; c < L.cols; c += 32) s = __fadd_rn(s, ld_any(L.in, L.in_dt, ib + c));
      s = row_allreduce<32>(s, false, nullptr);
      for (int64_t c = lane; c < L.cols; c += 32) st_any(L.out, L.out_dt, ob + c, __fdiv_rn(ld_any(L.in, L.in_dt, ib + c), s));
    } else {
      auto xval = [&](int64_t c) {
        const float x = ld_any(L.in, L.in_dt, ib + c);
        return L.res != nullptr ? __fadd_rn(x, ld_any(L.res, L.in_dt, ib + c)) : x;
      };
      float ss = 0.f;
      for (int64_t c = lane; c < L.cols; c += 32) { const float x = xval(c); ss = __fadd_rn(ss, __fmul_rn(x, x)); }
      ss = row_allreduce<32>(ss, false, nullptr);
      const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, float(L.cols)), L.eps));
      for (int64_t c = lane; c < L.cols; c += 32)
        st_any(L.out, L.out_dt, ob + c, __fmul_rn(__fmul_rn(xval(c), rs), ld_any(L.weight, L.w_dt, c)));
    }
  }
}

template <int KIND, int TPR, int CH>
static void launch_row_fast(const RowLaunch &L, const LaunchCtx &c) {
  constexpr int RPC = 256 / TPR;
  const int64_t rows = L.rows_end - L.rows_begin;
  (void)launch_pdl(row_fast_kernel<KIND, TPR, CH>, dim3(unsigned(ceil_div(rows, RPC))), dim3(256), 0, c.stream, L);
}

template <int KIND, int TPR>
static bool dispatch_ch(const RowLaunch &L, const LaunchCtx &c, int ch) {
  switch (ch) {
    case 1: launch_row_fast<KIND, TPR, 1>(L, c); return true;
    case 2: launch_row_fast<KIND, TPR, 2>(L, c); return true;
    case 3: launch_row_fast<KIND, TPR, 3>(L, c); return true;
    case 4: launch_row_fast<KIND, TPR, 4>(L, c); return true;
  }
  return false;
}

template <int KIND>
static int launch_row_kind(const RowLaunch &L, const LaunchCtx &c) {
  const bool bf16_io = L.in_dt == PTSIM_DT_BF16 && L.out_dt == PTSIM_DT_BF16 &&
                       (KIND == kSoftmax || L.w_dt == PTSIM_DT_BF16);
  const bool aligned = (reinterpret_cast<uintptr_t>(L.in) % 16 == 0) && (reinterpret_cast<uintptr_t>(L.out) % 16 == 0) &&
                       (KIND == kSoftmax || reinterpret_cast<uintptr_t>(L.weight) % 16 == 0) &&
                       (L.in_stride % 8 == 0) && (L.out_stride % 8 == 0);
  if (bf16_io && aligned && L.res == nullptr) {
    bool done = false;
    const int rc = dispatch_row_cta<KIND>(L, c, &done);
    if (done) return rc;
  }
  if (bf16_io && aligned && L.cols % 8 == 0) {
    // Spread a row over as many threads as keep at most 4 chunks (32 values) each in registers.
    const int64_t chunks = L.cols / 8;
    const int tprs[5] = {16, 32, 64, 128, 256};
    for (int t : tprs) {
      if (chunks % t || chunks / t > 4) continue;
      const int ch = int(chunks / t);
      bool ok = false;
      switch (t) {
        case 16: ok = dispatch_ch<KIND, 16>(L, c, ch); break;
        case 32: ok = dispatch_ch<KIND, 32>(L, c, ch); break;
        case 64: ok = dispatch_ch<KIND, 64>(L, c, ch); break;
        case 128: ok = dispatch_ch<KIND, 128>(L, c, ch); break;
        case 256: ok = dispatch_ch<KIND, 256>(L, c, ch); break;
      }
      if (ok) { PTSIM_CUDA(cudaGetLastError()); return PTSIM_OK; }
    }
  }
  int64_t blocks = ceil_div(L.rows_end - L.rows_begin, 8);
  if (blocks > int64_t(c.sm_count) * 8) blocks = int64_t(c.sm_count) * 8;
  PTSIM_CUDA(launch_pdl(row_generic_kernel<KIND>, dim3(unsigned(blocks)), dim3(256), 0, c.stream, L));
  return PTSIM_OK;
}

int launch_rowops(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c) {
  const ptsim_row_params &p = d.p.row;
  RowLaunch L;
  memset(&L, 0, sizeof(L));
  L.in = ptrs[p.in_arg];
  L.out = ptrs[p.out_arg];
  L.weight = p.weight_arg >= 0 ? ptrs[p.weight_arg] : nullptr;
  L.res = (d.kind == PTSIM_KIND_ROW_RMSNORM && p.res_arg_p1 > 0) ? ptrs[p.res_arg_p1 - 1] : nullptr;
  if (L.res != nullptr && (d.arg_dtype[p.res_arg_p1 - 1] != d.arg_dtype[p.in_arg] || reinterpret_cast<uintptr_t>(L.res) % 16 != 0))
    return fail(PTSIM_E_UNSUPPORTED, "RMSNorm residual row: the input's element type, 16-byte aligned");
  L.rows_begin = lo * d.unit_size;
  L.rows_end = hi * d.unit_size < p.rows ? hi * d.unit_size : p.rows;
  L.rows_total = p.rows;
  L.cols = p.cols;
  L.in_stride = p.in_row_stride;
  L.out_stride = p.out_row_stride;
  L.in_dt = d.arg_dtype[p.in_arg];
  L.out_dt = d.arg_dtype[p.out_arg];
  L.w_dt = p.weight_arg >= 0 ? d.arg_dtype[p.weight_arg] : PTSIM_DT_BF16;
  L.eps = p.eps;
  if (L.rows_end <= L.rows_begin) return PTSIM_OK;
  if (d.kind == PTSIM_KIND_ROW_SOFTMAX) return launch_row_kind<kSoftmax>(L, c);
  if (d.kind == PTSIM_KIND_ROW_DIVSUM || d.kind == PTSIM_KIND_ROW_SUM) {
    // Rows of a few values (the router's top-k weights): one warp per row.
    int64_t blocks = ceil_div(L.rows_end - L.rows_begin, 8);
    if (blocks > int64_t(c.sm_count) * 8) blocks = int64_t(c.sm_count) * 8;
    if (d.kind == PTSIM_KIND_ROW_SUM) PTSIM_CUDA(launch_pdl(row_generic_kernel<kRowSum>, dim3(unsigned(blocks)), dim3(256), 0, c.stream, L));
    else PTSIM_CUDA(launch_pdl(row_generic_kernel<kDivSum>, dim3(unsigned(blocks)), dim3(256), 0, c.stream, L));
    return PTSIM_OK;
  }
  return launch_row_kind<kRmsNorm>(L, c);
}

// ---------------------------------------------------------------------------------------------------
// QK-RMSNorm + RoPE (validation/pytorchsim/qwen3_8b_layer_prefill_2048x2048_bf16/02_*/..._triton.py):
// row (t, h) of `dim` = 128 values: r = rsqrt(mean(x^2) + eps); n = (x * r) * w; the rotated half is
// cat(-n[64:], n[:64]); out[t, h] stored head-major = n * cos[t] + rot * sin[t].  A half-warp per row,
// eight values per lane (one 16-byte load); lane l's rotation partner holds d +- 64, i.e. lane l ^ 8 of
// the same half.  A warp takes two rows per step and issues the loads of two steps before computing, so
// four rows of loads are in flight per warp; row indices are 32-bit (the launch is refused past 2^31).
// ---------------------------------------------------------------------------------------------------
struct QkLaunch {
  const uint16_t *in;
  const uint16_t *w;
  const float *cosb, *sinb;
  uint16_t *out;
  uint32_t row_begin, row_end, heads;
  int64_t tok_stride, head_stride;
  float eps;
  int32_t no_norm;   // the rotation alone (layer_op_rope_*): n = x
};

__global__ void __launch_bounds__(256) qk_rope_kernel(const __grid_constant__ QkLaunch L) {
  pdl_enter();
  const int lane = threadIdx.x & 31, sub = lane & 15, half = lane >> 4;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  const uint4 wv = L.no_norm ? make_uint4(0, 0, 0, 0) : __ldg(reinterpret_cast<const uint4 *>(L.w) + sub);
  const float w[8] = {lo_bf16(wv.x), hi_bf16(wv.x), lo_bf16(wv.y), hi_bf16(wv.y),
                      lo_bf16(wv.z), hi_bf16(wv.z), lo_bf16(wv.w), hi_bf16(wv.w)};
  const unsigned full = 0xffffffffu;
  for (uint32_t r0 = L.row_begin + 4 * warp; r0 < L.row_end; r0 += 4 * nwarps) {
    // Rows r0 + half (step 0) and r0 + 2 + half (step 1).
    uint4 xv[2];
    bool live[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const uint32_t row = r0 + 2 * s + half;
      live[s] = row < L.row_end;
      xv[s] = live[s] ? __ldcs(reinterpret_cast<const uint4 *>(L.in + size_t(row) * 128) + sub) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const uint32_t row = r0 + 2 * s + half;
      const uint32_t t = row / L.heads, h = row - t * L.heads;
      const uint32_t xs[4] = {xv[s].x, xv[s].y, xv[s].z, xv[s].w};
      float x[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[2 * j] = lo_bf16(xs[j]);
        x[2 * j + 1] = hi_bf16(xs[j]);
      }
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(x[j], x[j]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(full, ss, o));   // within the half
      const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, 128.f), L.eps));
      float n[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) n[j] = L.no_norm ? x[j] : __fmul_rn(__fmul_rn(x[j], rs), w[j]);
      const float4 *cp = reinterpret_cast<const float4 *>(L.cosb + size_t(t) * 128) + 2 * sub;
      const float4 *sp = reinterpret_cast<const float4 *>(L.sinb + size_t(t) * 128) + 2 * sub;
      const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
      const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float partner = __shfl_xor_sync(full, n[j], 8);
        const float rot = sub < 8 ? -partner : partner;
        o[j] = __fadd_rn(__fmul_rn(n[j], cv[j]), __fmul_rn(rot, sv[j]));
      }
      if (live[s])
        *reinterpret_cast<uint4 *>(L.out + int64_t(t) * L.tok_stride + int64_t(h) * L.head_stride + sub * 8) =
            make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
    }
  }
}

int launch_qkrope(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c) {
  const ptsim_qkrope_params &p = d.p.qk;
  if (p.dim != 128) return fail(PTSIM_E_UNSUPPORTED, "QK-norm+RoPE runs head_dim 128, not %lld", (long long)p.dim);
  if (p.out_tok_stride % 8 || p.out_head_stride % 8)
    return fail(PTSIM_E_UNSUPPORTED, "QK-norm+RoPE output strides must keep 16-byte alignment");
  if (p.tokens * p.heads >= (int64_t(1) << 31)) return fail(PTSIM_E_UNSUPPORTED, "QK-norm+RoPE over 2^31 rows");
  QkLaunch L;
  L.in = reinterpret_cast<const uint16_t *>(ptrs[p.in_arg]);
  L.w = p.no_norm ? nullptr : reinterpret_cast<const uint16_t *>(ptrs[p.weight_arg]);
  L.no_norm = p.no_norm;
  L.cosb = reinterpret_cast<const float *>(ptrs[p.cos_arg]);
  L.sinb = reinterpret_cast<const float *>(ptrs[p.sin_arg]);
  L.out = reinterpret_cast<uint16_t *>(ptrs[p.out_arg]);
  const int64_t rows = p.tokens * p.heads;
  L.row_begin = uint32_t(lo * d.unit_size);
  L.row_end = uint32_t(hi * d.unit_size < rows ? hi * d.unit_size : rows);
  L.heads = uint32_t(p.heads);
  L.tok_stride = p.out_tok_stride;
  L.head_stride = p.out_head_stride;
  L.eps = p.eps;
  if (L.row_end <= L.row_begin) return PTSIM_OK;
  // Four rows per warp per step, eight warps per block; enough blocks for one step of every row.
  int64_t blocks = ceil_div(int64_t(L.row_end - L.row_begin), 32);
  if (blocks > int64_t(c.sm_count) * 16) blocks = int64_t(c.sm_count) * 16;
  PTSIM_CUDA(launch_pdl(qk_rope_kernel, dim3(unsigned(blocks)), dim3(256), 0, c.stream, L));
  return PTSIM_OK;
}

// ---------------------------------------------------------------------------------------------------
// Whole-tensor sum / max to one fp32 value (validation/pytorchsim/vector_sum_4096x4096_bf16/00_*:
// lanes accumulate strided slices of the tensor, then one cross-lane reduction).  Pass 1: every thread
// accumulates a grid-strided slice in fp32, each CTA reduces its threads and writes one partial to the
// caller's workspace; pass 2: one CTA reduces the partials in a fixed order.  Deterministic.
// ---------------------------------------------------------------------------------------------------
constexpr int kReduceThreads = 256;

template <bool IS_MAX>
__device__ __forceinline__ float block_reduce(float v, float *sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = IS_MAX ? nan_max(v, w) : __fadd_rn(v, w);
  }
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : (IS_MAX ? -INFINITY : 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, v, o);
      v = IS_MAX ? nan_max(v, w) : __fadd_rn(v, w);
    }
  }
  return v;
}

template <bool IS_MAX>
__global__ void __launch_bounds__(kReduceThreads) reduce_pass1(const void *in, int dt, int64_t begin, int64_t end,
                                                               float *partials) {
  __shared__ float sh[32];
  float acc = IS_MAX ? -INFINITY : 0.f;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  if (dt == PTSIM_DT_BF16 && begin % 8 == 0 && (reinterpret_cast<uintptr_t>(in) % 16) == 0) {
    const uint16_t *p = reinterpret_cast<const uint16_t *>(in);
    const int64_t nvec = (end - begin) / 8;
    for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < nvec; g += stride) {
      const uint4 w = __ldcs(reinterpret_cast<const uint4 *>(p + begin) + g);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc = IS_MAX ? nan_max(acc, lo_bf16(ws[j])) : __fadd_rn(acc, lo_bf16(ws[j]));
        acc = IS_MAX ? nan_max(acc, hi_bf16(ws[j])) : __fadd_rn(acc, hi_bf16(ws[j]));
      }
    }
    for (int64_t i = begin + nvec * 8 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < end; i += stride) {
      const float x = bf16_bits_to_f32(p[i]);
      acc = IS_MAX ? nan_max(acc, x) : __fadd_rn(acc, x);
    }
  } else {
    for (int64_t i = begin + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < end; i += stride) {
      const float x = ld_any(in, dt, i);
      acc = IS_MAX ? nan_max(acc, x) : __fadd_rn(acc, x);
    }
  }
  acc = block_reduce<IS_MAX>(acc, sh);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc;
}

// Pass 1 over a fused operand (the decode layer's sums of squares, qwen3_8b_layer_decode_*/00_*, 05_*:
// x^2 or (x + residual)^2 per element, fp32 unrounded).
struct ReduceProgArgs {
  ptsim_vprog pro;
  VArgs t;
  int64_t numel;
  float *partials;
};

template <bool IS_MAX>
__global__ void __launch_bounds__(kReduceThreads) reduce_pass1_prog(const __grid_constant__ ReduceProgArgs a) {
  __shared__ float sh[32];
  float acc = IS_MAX ? -INFINITY : 0.f;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < a.numel; i += stride) {
    const float x = vprog_eval(a.pro, a.t, i, 0.f);
    acc = IS_MAX ? nan_max(acc, x) : __fadd_rn(acc, x);
  }
  acc = block_reduce<IS_MAX>(acc, sh);
  if (threadIdx.x == 0) a.partials[blockIdx.x] = acc;
}

template <bool IS_MAX>
__global__ void __launch_bounds__(kReduceThreads) reduce_pass2(const float *partials, int n, float *out) {
  __shared__ float sh[32];
  float acc = IS_MAX ? -INFINITY : 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc = IS_MAX ? nan_max(acc, partials[i]) : __fadd_rn(acc, partials[i]);
  acc = block_reduce<IS_MAX>(acc, sh);
  if (threadIdx.x == 0) *out = acc;
}

// Partials one launch writes: one per CTA of pass 1 (4 CTAs per SM, at most 1024).
static int reduce_blocks(int sm_count) { return sm_count * 4 < 1024 ? sm_count * 4 : 1024; }

// Scratch bytes a launch needs on a device of `sm_count` SMs: the pass-1 partials.
int reduce_workspace(int sm_count) { return reduce_blocks(sm_count) * int(sizeof(float)); }

int launch_reduce(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                  const LaunchCtx &c) {
  const ptsim_reduce_params &p = d.p.red;
  if (lo != 0 || hi != d.units)
    return fail(PTSIM_E_ARGS, "a whole-tensor reduction runs as one unit (lo=0, hi=%lld)", (long long)d.units);
  const int blocks = reduce_blocks(c.sm_count);
  if (ws == nullptr || ws_bytes < size_t(blocks) * sizeof(float))
    return fail(PTSIM_E_RESOURCE, "reduction needs %zu workspace bytes, got %zu", size_t(blocks) * sizeof(float), ws_bytes);
  float *partials = reinterpret_cast<float *>(ws);
  float *out = reinterpret_cast<float *>(ptrs[p.out_arg]);
  if (d.arg_dtype[p.out_arg] != PTSIM_DT_F32) return fail(PTSIM_E_UNSUPPORTED, "reduction output must be float32");
  const int dt = d.arg_dtype[p.in_arg];
  if (p.pro.ncode > 0) {
    ReduceProgArgs a;
    memset(&a, 0, sizeof(a));
    a.pro = p.pro;
    vargs_fill(a.t, d, ptrs);
    a.numel = p.numel;
    a.partials = partials;
    if (p.op == PTSIM_RED_MAX) {
      reduce_pass1_prog<true><<<blocks, kReduceThreads, 0, c.stream>>>(a);
      reduce_pass2<true><<<1, kReduceThreads, 0, c.stream>>>(partials, blocks, out);
    } else {
      reduce_pass1_prog<false><<<blocks, kReduceThreads, 0, c.stream>>>(a);
      reduce_pass2<false><<<1, kReduceThreads, 0, c.stream>>>(partials, blocks, out);
    }
    PTSIM_CUDA(cudaGetLastError());
    return PTSIM_OK;
  }
  if (p.op == PTSIM_RED_MAX) {
    reduce_pass1<true><<<blocks, kReduceThreads, 0, c.stream>>>(ptrs[p.in_arg], dt, 0, p.numel, partials);
    reduce_pass2<true><<<1, kReduceThreads, 0, c.stream>>>(partials, blocks, out);
  } else {
    reduce_pass1<false><<<blocks, kReduceThreads, 0, c.stream>>>(ptrs[p.in_arg], dt, 0, p.numel, partials);
    reduce_pass2<false><<<1, kReduceThreads, 0, c.stream>>>(partials, blocks, out);
  }
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

}  // namespace ptsim
