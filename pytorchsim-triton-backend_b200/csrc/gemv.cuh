// Matrix-vector product: the gemm_1x* programs of the validation bundle and the o-projection of the
// Qwen3 decode layer (Inductor's M = 1 matmul, validation/pytorchsim/gemm_1x4096x4096_bf16/00_*_triton.py):
// out[n] = bf16(sum_k fp32(a[k]) * fp32(B[k, n])), a multiply-reduce program the reference runs on its
// vector unit (its MXU refuses M = 1, targets/tpu/lower_matmul.py:464-489).  Every element of B is read
// once and used once (2 FLOP per 2 bytes), so this is an HBM stream on the CUDA cores, not tensor-core
// work.
//
// N-contiguous B ([K, N], the Inductor layout): one cluster of S CTAs per tile of CW columns, each CTA
// over K / S rows.  Thread t streams 8 adjacent columns of rows k0 + t / (CW / 8) + j * RG with 16-byte
// loads, eight in flight; the RG row groups of a CTA meet in shared memory, then rank 0 of the cluster adds
// the S partial columns in rank order through distributed shared memory -- a fixed summation order and
// no device scratch.
// K-major B ([N, K]): one warp per output column, 16-byte loads along K, a shuffle tree.
//
// Fused forms (the Qwen3 decode layer's programs, validation/pytorchsim/qwen3_8b_layer_decode_*/01_*, 06_*,
// 07_*): a vector prologue (ptsim_vprog over k: an RMSNorm x * rsqrt(ss / n + eps) * w, a SiLU gate times
// its up half) is evaluated once per CTA for its K slice into shared memory in fp32, unrounded, as the
// programs keep it; an epilogue (over n, the dot product in r7) adds residual rows before the store.

#pragma once
#include "sm100.cuh"
#include "tmap.cuh"
#include "vprog.cuh"

namespace ptsim {

constexpr int kGemvThreads = 256;
constexpr int kGemvUnroll = 8;

constexpr int kGemvMaxVecBytes = 160 * 1024;   // shared-memory vector slice of a prologue launch

struct GemvArgs {
  const uint16_t *a, *b, *r;   // a [K]; B; residual [N] or null
  uint16_t *c;                 // bf16 output, or null
  float *c_f32;                // fp32 output, or null
  int64_t N, K, ldb;
  int64_t k_per_cta;           // K rows per CTA of a cluster
  ptsim_vprog pro, epi;        // fused vector prologue / output epilogue (ncode 0: none)
  VArgs t;
  // PTSIM_FLAG_TEST_STALL (bulk path): CTA (0, 0) arms its first stage but issues none of its copies, and
  // every wait gives up after kTestWaitUs -- the timeout path under test.
  int32_t stall;
};

__device__ __forceinline__ void gemv_fma8(float (&acc)[8], float a, const uint4 &v) {
  acc[0] = fmaf(a, lo_bf16(v.x), acc[0]);
  acc[1] = fmaf(a, hi_bf16(v.x), acc[1]);
  acc[2] = fmaf(a, lo_bf16(v.y), acc[2]);
  acc[3] = fmaf(a, hi_bf16(v.y), acc[3]);
  acc[4] = fmaf(a, lo_bf16(v.z), acc[4]);
  acc[5] = fmaf(a, hi_bf16(v.z), acc[5]);
  acc[6] = fmaf(a, lo_bf16(v.w), acc[6]);
  acc[7] = fmaf(a, hi_bf16(v.w), acc[7]);
}

// The epilogue out of line: the plain kernels keep their registers for the stream.
__device__ __noinline__ float gemv_epilogue(const GemvArgs &g, int64_t n, float s) { return vprog_eval(g.epi, g.t, n, s); }

__device__ __forceinline__ void gemv_store(const GemvArgs &g, int64_t n, float s) {
  if (g.epi.ncode > 0) s = gemv_epilogue(g, n, s);
  else if (g.r != nullptr) s += bf16_bits_to_f32(g.r[n]);
  if (g.c_f32 != nullptr) g.c_f32[n] = s;
  else g.c[n] = f32_to_bf16_bits(s);
}

// TPRW threads per row of the tile (CW = 8 * TPRW columns); grid (column tiles, S) in clusters (1, S, 1).
// PRO: the vector comes from the prologue, staged for the CTA's K slice in dynamic shared memory.
template <int TPRW, bool PRO>
__global__ void __launch_bounds__(kGemvThreads) gemv_kn_kernel(const __grid_constant__ GemvArgs g) {
  constexpr int CW = TPRW * 8, RG = kGemvThreads / TPRW, U = kGemvUnroll;
  __shared__ float red[RG][CW];
  __shared__ float part[CW];
  extern __shared__ float vec[];
  const int tid = threadIdx.x;
  const int cg = tid % TPRW, rg = tid / TPRW;
  const int64_t n0 = int64_t(blockIdx.x) * CW + cg * 8;
  const int64_t k_begin = int64_t(blockIdx.y) * g.k_per_cta;
  const int64_t k_end = k_begin + g.k_per_cta < g.K ? k_begin + g.k_per_cta : g.K;
  if (PRO) {
    // four elements per thread per step, their loads in flight together
    for (int64_t k0 = k_begin + tid; k0 < k_end; k0 += 4 * kGemvThreads) {
      int64_t idx[4];
      bool live[4];
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        idx[j] = k0 + j * kGemvThreads;
        live[j] = idx[j] < k_end;
      }
      vprog_eval_batch<4>(g.pro, g.t, idx, live, o);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (live[j]) vec[idx[j] - k_begin] = o[j];
    }
    __syncthreads();
  }
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  if (n0 < g.N) {
    const uint16_t *bp = g.b + n0;
    int64_t k = k_begin + rg;
    for (; k + (U - 1) * RG < k_end; k += U * RG) {
      uint4 v[U];
      float av[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        v[u] = __ldcs(reinterpret_cast<const uint4 *>(bp + (k + u * RG) * g.ldb));
        av[u] = PRO ? vec[k + u * RG - k_begin] : bf16_bits_to_f32(__ldg(g.a + k + u * RG));
      }
#pragma unroll
      for (int u = 0; u < U; ++u) gemv_fma8(acc, av[u], v[u]);
    }
    for (; k < k_end; k += RG) {
      const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(bp + k * g.ldb));
      gemv_fma8(acc, PRO ? vec[k - k_begin] : bf16_bits_to_f32(__ldg(g.a + k)), v);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[rg][cg * 8 + j] = acc[j];
  __syncthreads();
  if (tid < CW) {
    float s = 0.f;
#pragma unroll 8
    for (int i = 0; i < RG; ++i) s += red[i][tid];
    part[tid] = s;
  }
  // Every CTA's partial columns are written (and, by the release/acquire of the cluster barrier, visible
  // to the cluster) before rank 0 reads them; the second barrier keeps the peers resident until it has.
  sm100::cluster_sync();
  if (blockIdx.y == 0 && tid < CW) {
    const int64_t n = int64_t(blockIdx.x) * CW + tid;
    if (n < g.N) {
      float s = part[tid];
      const uint32_t addr = sm100::smem_u32(&part[tid]);
      for (uint32_t q = 1; q < gridDim.y; ++q) s += sm100::ld_cluster_f32(sm100::mapa_shared(addr, q));
      gemv_store(g, n, s);
    }
  }
  sm100::cluster_sync();
}

// Row-streaming path (N-contiguous B, N % 8 == 0, with scratch): a CTA covers 2048 adjacent columns (4 KB of each
// row), K is cut over grid.y (about one CTA per SM in all); every CTA writes its partial columns to scratch and
// gemv_reduce_kernel sums them in split order (fixed) before the epilogue and the store.
constexpr int kGrCols = 2048;

// B comes in through the bulk-copy engine, not through loads.  One
// producer thread copies each row's 4 KB run of the tile (cp.async.bulk, one request per row) into a ring of
// kGbStages stages of kGbRows rows, 192 KB in flight per CTA with no register cost; 256 consumer threads each own
// 8 columns of the tile and read their 16 bytes of every row from shared memory, so a column's partial sum is
// one thread's and the CTA writes its partial columns straight to scratch.
constexpr int kGbRows = 8, kGbStages = 6;
constexpr int kGbStageBytes = kGbRows * kGrCols * 2;   // 32 KB
constexpr int kGbConsumers = 256, kGbThreads = kGbConsumers + 32;
constexpr int64_t kGbMaxRows = 4096;                   // vector rows a CTA stages (16 KB)

template <bool PRO>
__global__ void __launch_bounds__(kGbThreads, 1) gemv_bulk_kernel(const __grid_constant__ GemvArgs g, float *part) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // the reduce may launch (and wait) early
  extern __shared__ __align__(128) uint8_t gb_smem[];
  uint8_t *ring = gb_smem;
  float *vec = reinterpret_cast<float *>(gb_smem + kGbStages * kGbStageBytes);
  __shared__ __align__(8) uint64_t full[kGbStages], empty[kGbStages];
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n0 = int64_t(blockIdx.x) * kGrCols;
  const int64_t ncols = g.N - n0 < kGrCols ? g.N - n0 : kGrCols;
  const uint32_t row_bytes = uint32_t(ncols * 2);
  const int64_t k_begin = int64_t(blockIdx.y) * g.k_per_cta;
  const int64_t k_end = k_begin + g.k_per_cta < g.K ? k_begin + g.k_per_cta : g.K;
  const int64_t nrows = k_end - k_begin;
  const int nst = int((nrows + kGbRows - 1) / kGbRows);
  const uint32_t wl = g.stall ? kTestWaitUs : kWaitUs;
  if (tid == 0) {
    for (int st = 0; st < kGbStages; ++st) {
      sm100::mbar_init(&full[st], 1);
      sm100::mbar_init(&empty[st], kGbConsumers / 32);
    }
    sm100::fence_barrier_init();
    abort_flag = 0;
  }
  __syncthreads();
  if (warp == kGbConsumers / 32) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nst; ++i) {
        const int st = i % kGbStages;
        if (i >= kGbStages && !sm100::mbar_wait(&empty[st], uint32_t((i / kGbStages - 1) & 1), wl)) {
          atomicExch(&abort_flag, 1);
          break;
        }
        if (*reinterpret_cast<volatile int *>(&abort_flag)) break;
        const int64_t r0 = int64_t(i) * kGbRows;
        const int rows = nrows - r0 < kGbRows ? int(nrows - r0) : kGbRows;
        sm100::mbar_arrive_expect_tx(&full[st], uint32_t(rows) * row_bytes);
        issued = i + 1;
        if (g.stall && blockIdx.x == 0 && blockIdx.y == 0 && i == 0) continue;   // test hook: armed, no copy
        for (int r = 0; r < rows; ++r)
          sm100::bulk_load_g2s(ring + st * kGbStageBytes + r * (kGrCols * 2), g.b + (k_begin + r0 + r) * g.ldb + n0,
                               row_bytes, &full[st]);
        issued = i + 1;
      }
      // Every copy issued lands before the CTA moves on (bounded waits).
      for (int i = issued - kGbStages > 0 ? issued - kGbStages : 0; i < issued; ++i)
        sm100::mbar_wait(&full[i % kGbStages], uint32_t((i / kGbStages) & 1), wl);
    }
  } else {
    if (PRO) {
      for (int64_t k0 = tid; k0 < nrows; k0 += 4 * kGbConsumers) {
        int64_t idx[4];
        bool live[4];
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          idx[j] = k_begin + k0 + j * kGbConsumers;
          live[j] = idx[j] < k_end;
        }
        vprog_eval_batch<4>(g.pro, g.t, idx, live, o);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (live[j]) vec[k0 + j * kGbConsumers] = o[j];
      }
    } else {
      for (int64_t k = tid; k < nrows; k += kGbConsumers) vec[k] = bf16_bits_to_f32(__ldg(g.a + k_begin + k));
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kGbConsumers));   // the vector slice, seen by every consumer
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    const int64_t col = int64_t(tid) * 8;
    const bool active = col < ncols;
    for (int i = 0; i < nst; ++i) {
      const int st = i % kGbStages;
      if (*reinterpret_cast<volatile int *>(&abort_flag)) break;
      if (!sm100::mbar_wait(&full[st], uint32_t((i / kGbStages) & 1), wl)) {
        atomicExch(&abort_flag, 1);
        break;
      }
      const int64_t r0 = int64_t(i) * kGbRows;
      const int rows = nrows - r0 < kGbRows ? int(nrows - r0) : kGbRows;
      if (active) {
        const uint8_t *box = ring + st * kGbStageBytes + tid * 16;
        for (int r = 0; r < rows; ++r)
          gemv_fma8(acc, vec[r0 + r], *reinterpret_cast<const uint4 *>(box + r * (kGrCols * 2)));
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty[st]);
    }
    if (active) {
      float *dst = part + int64_t(blockIdx.y) * g.N + n0 + col;
      reinterpret_cast<float4 *>(dst)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      reinterpret_cast<float4 *>(dst)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// out[n] = the splits' partial columns summed, then the epilogue / residual and the store.  A CTA takes 32
// columns with 8 threads each: thread j sums splits j, j + 8, ... in order (eight loads in flight), and the
// 8 sums are added in j order -- a fixed order, so every launch gives the same bits.  Launched as the bulk
// kernel's programmatic dependent: it waits for that grid (and its partial stores) before reading.
__global__ void __launch_bounds__(kGemvThreads) gemv_reduce_kernel(const __grid_constant__ GemvArgs g, const float *part,
                                                                     int splits) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float sh[8][32];
  const int c = threadIdx.x & 31, j = threadIdx.x >> 5;
  const int64_t n = int64_t(blockIdx.x) * 32 + c;
  float s = 0.f;
  if (n < g.N)
    for (int q0 = j; q0 < splits; q0 += 64) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = q0 + 8 * u < splits ? __ldcs(part + int64_t(q0 + 8 * u) * g.N + n) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) s += v[u];
    }
  sh[j][c] = s;
  __syncthreads();
  if (j == 0 && n < g.N) {
    float t = sh[0][c];
#pragma unroll
    for (int q = 1; q < 8; ++q) t += sh[q][c];
    gemv_store(g, n, t);
  }
}

// The row-streaming plan: 2048-column tiles, about one CTA per SM, at least 32 rows and at most kGbMaxRows (the
// staged vector) per CTA.
// Matrices from 32M elements (64 MB) up stream on this path; smaller ones run the single-launch cluster path,
// where the second launch and the short K slices of a split over every SM cost more than they save.
constexpr int64_t kGrMinElems = int64_t(32) << 20;
struct GemvRowsPlan {
  int splits;
  int64_t tiles, k_per_cta;
};
static GemvRowsPlan plan_gemv_rows(int64_t N, int64_t K, int sm_count) {
  GemvRowsPlan pl;
  pl.tiles = ceil_div(N, int64_t(kGrCols));
  int64_t s = int64_t(sm_count) / pl.tiles;
  if (s > K / 32) s = K / 32;
  if (s < 1) s = 1;
  while (ceil_div(K, s) > kGbMaxRows) ++s;
  pl.k_per_cta = ceil_div(K, s);
  pl.splits = int(ceil_div(K, pl.k_per_cta));
  return pl;
}

// Scratch of a matrix-vector launch (the row-streaming path's partial columns), 0 for other GEMMs.
int64_t gemv_workspace(const ptsim_desc &d, int sm_count) {
  const ptsim_gemm_params &p = d.p.gemm;
  if (p.M != 1 || p.b_kmajor || p.N % 8 != 0 || p.ldb % 8 != 0 || p.K * p.N < kGrMinElems) return 0;
  const GemvRowsPlan pl = plan_gemv_rows(p.N, p.K, sm_count);
  return int64_t(pl.splits) * p.N * int64_t(sizeof(float));
}

// K-major B: warp w of CTA b computes column n = 8 b + w; lanes take 8 consecutive k, 256 k per step.
__global__ void __launch_bounds__(kGemvThreads) gemv_nk_kernel(const __grid_constant__ GemvArgs g) {
  const int lane = threadIdx.x & 31;
  const int64_t n = int64_t(blockIdx.x) * (kGemvThreads / 32) + (threadIdx.x >> 5);
  if (n >= g.N) return;
  const uint16_t *row = g.b + n * g.ldb;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  int64_t k = int64_t(lane) * 8;
  for (; k + 3 * 256 < g.K; k += 4 * 256) {
    uint4 v[4], a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = __ldcs(reinterpret_cast<const uint4 *>(row + k + u * 256));
      a[u] = __ldg(reinterpret_cast<const uint4 *>(g.a + k + u * 256));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc[0] = fmaf(lo_bf16(a[u].x), lo_bf16(v[u].x), acc[0]);
      acc[1] = fmaf(hi_bf16(a[u].x), hi_bf16(v[u].x), acc[1]);
      acc[2] = fmaf(lo_bf16(a[u].y), lo_bf16(v[u].y), acc[2]);
      acc[3] = fmaf(hi_bf16(a[u].y), hi_bf16(v[u].y), acc[3]);
      acc[4] = fmaf(lo_bf16(a[u].z), lo_bf16(v[u].z), acc[4]);
      acc[5] = fmaf(hi_bf16(a[u].z), hi_bf16(v[u].z), acc[5]);
      acc[6] = fmaf(lo_bf16(a[u].w), lo_bf16(v[u].w), acc[6]);
      acc[7] = fmaf(hi_bf16(a[u].w), hi_bf16(v[u].w), acc[7]);
    }
  }
  for (; k < g.K; k += 256) {
    const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(row + k));
    const uint4 a = __ldg(reinterpret_cast<const uint4 *>(g.a + k));
    acc[0] = fmaf(lo_bf16(a.x), lo_bf16(v.x), acc[0]);
    acc[1] = fmaf(hi_bf16(a.x), hi_bf16(v.x), acc[1]);
    acc[2] = fmaf(lo_bf16(a.y), lo_bf16(v.y), acc[2]);
    acc[3] = fmaf(hi_bf16(a.y), hi_bf16(v.y), acc[3]);
    acc[4] = fmaf(lo_bf16(a.z), lo_bf16(v.z), acc[4]);
    acc[5] = fmaf(hi_bf16(a.z), hi_bf16(v.z), acc[5]);
    acc[6] = fmaf(lo_bf16(a.w), lo_bf16(v.w), acc[6]);
    acc[7] = fmaf(hi_bf16(a.w), hi_bf16(v.w), acc[7]);
  }
  float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) gemv_store(g, n, s);
}

// The tile plan of an N-contiguous GEMV: the widest column tile whose clusters (K split in up to 8,
// each CTA at least 128 rows) give every SM two CTAs; else 64-column tiles with the deepest split.
struct GemvPlan {
  int tprw, splits;
  int64_t tiles, k_per_cta;
};

static GemvPlan plan_gemv(int64_t N, int64_t K, int sm_count) {
  GemvPlan pl{8, 1, 0, K};
  for (int tprw : {32, 16, 8}) {
    const int64_t tiles = ceil_div(N, int64_t(tprw) * 8);
    int s = 1;
    while (s < 8 && tiles * s < 2 * sm_count && K / (2 * s) >= 128) s *= 2;
    pl = GemvPlan{tprw, s, tiles, ceil_div(K, s)};
    if (tiles * s >= 2 * sm_count) break;
  }
  return pl;
}

template <int TPRW, bool PRO>
static int run_gemv_kn(const GemvArgs &g, const GemvPlan &pl, const LaunchCtx &c) {
  const int vec_bytes = PRO ? int(pl.k_per_cta * int64_t(sizeof(float))) : 0;
  if (PRO) PTSIM_CUDA((smem_limit_once<gemv_kn_kernel<TPRW, true>>(kGemvMaxVecBytes, c.device)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(pl.tiles), unsigned(pl.splits), 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = size_t(vec_bytes);
  cfg.stream = c.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = unsigned(pl.splits);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PTSIM_CUDA(cudaLaunchKernelEx(&cfg, gemv_kn_kernel<TPRW, PRO>, g));
  return PTSIM_OK;
}

// The GEMM descriptor with M = 1 (checked by the caller), on the CUDA cores.
static int launch_gemv(const ptsim_desc &d, void *const *ptrs, void *ws, size_t ws_bytes, const LaunchCtx &c) {
  const ptsim_gemm_params &p = d.p.gemm;
  GemvArgs g;
  memset(&g, 0, sizeof(g));
  g.a = reinterpret_cast<const uint16_t *>(ptrs[p.a_arg]);
  g.b = reinterpret_cast<const uint16_t *>(ptrs[p.b_arg]);
  g.r = p.r_arg >= 0 ? reinterpret_cast<const uint16_t *>(ptrs[p.r_arg]) : nullptr;
  if (d.arg_dtype[p.c_arg] == PTSIM_DT_F32) g.c_f32 = reinterpret_cast<float *>(ptrs[p.c_arg]);
  else g.c = reinterpret_cast<uint16_t *>(ptrs[p.c_arg]);
  g.N = p.N;
  g.K = p.K;
  g.ldb = p.ldb;
  g.pro = p.pro;
  g.epi = p.epi;
  vargs_fill(g.t, d, ptrs);
  g.stall = (d.flags & PTSIM_FLAG_TEST_STALL) ? 1 : 0;
  const bool pro = p.pro.ncode > 0;
  if (reinterpret_cast<uintptr_t>(g.b) % 16 != 0) return fail(PTSIM_E_ARGS, "GEMV matrix is not 16-byte aligned");
  if (p.b_kmajor) {
    if (pro) return fail(PTSIM_E_UNSUPPORTED, "a GEMV vector prologue over an [N, K] matrix");
    if (p.K % 8 != 0 || p.ldb % 8 != 0 || reinterpret_cast<uintptr_t>(g.a) % 16 != 0)
      return fail(PTSIM_E_UNSUPPORTED, "GEMV over [N, K] needs K and the row stride multiples of 8 and a 16-byte aligned vector");
    const int64_t blocks = ceil_div(p.N, kGemvThreads / 32);
    gemv_nk_kernel<<<unsigned(blocks), kGemvThreads, 0, c.stream>>>(g);
    PTSIM_CUDA(cudaGetLastError());
    return PTSIM_OK;
  }
  if (p.N % 8 != 0 || p.ldb % 8 != 0)
    return fail(PTSIM_E_UNSUPPORTED, "GEMV over [K, N] needs N and the row stride multiples of 8");
  {
    const GemvRowsPlan pr = plan_gemv_rows(p.N, p.K, c.sm_count);
    const int64_t need = int64_t(pr.splits) * p.N * int64_t(sizeof(float));
    if (p.K * p.N >= kGrMinElems && ws != nullptr && int64_t(ws_bytes) >= need && reinterpret_cast<uintptr_t>(ws) % 16 == 0) {
      GemvArgs gr = g;
      gr.k_per_cta = pr.k_per_cta;
      float *part = reinterpret_cast<float *>(ws);
      const dim3 grid(unsigned(pr.tiles), unsigned(pr.splits));
      const size_t smem = size_t(kGbStages) * kGbStageBytes + size_t(pr.k_per_cta) * sizeof(float);
      const int cap = int(kGbStages * kGbStageBytes + kGbMaxRows * 4);
      if (pro) PTSIM_CUDA((smem_limit_once<gemv_bulk_kernel<true>>(cap, c.device)));
      else PTSIM_CUDA((smem_limit_once<gemv_bulk_kernel<false>>(cap, c.device)));
      if (pro) gemv_bulk_kernel<true><<<grid, kGbThreads, smem, c.stream>>>(gr, part);
      else gemv_bulk_kernel<false><<<grid, kGbThreads, smem, c.stream>>>(gr, part);
      PTSIM_CUDA(cudaGetLastError());
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(unsigned(ceil_div(p.N, int64_t(32))), 1, 1);
      cfg.blockDim = dim3(kGemvThreads, 1, 1);
      cfg.stream = c.stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      PTSIM_CUDA(cudaLaunchKernelEx(&cfg, gemv_reduce_kernel, static_cast<const GemvArgs &>(gr),
                                    static_cast<const float *>(part), int(pr.splits)));
      return PTSIM_OK;
    }
  }
  const GemvPlan pl = plan_gemv(p.N, p.K, c.sm_count);
  g.k_per_cta = pl.k_per_cta;
  if (pro) {
    if (pl.k_per_cta * int64_t(sizeof(float)) > kGemvMaxVecBytes)
      return fail(PTSIM_E_UNSUPPORTED, "a GEMV vector prologue over %lld rows per CTA", (long long)pl.k_per_cta);
    if (pl.tprw == 32) return run_gemv_kn<32, true>(g, pl, c);
    if (pl.tprw == 16) return run_gemv_kn<16, true>(g, pl, c);
    return run_gemv_kn<8, true>(g, pl, c);
  }
  if (pl.tprw == 32) return run_gemv_kn<32, false>(g, pl, c);
  if (pl.tprw == 16) return run_gemv_kn<16, false>(g, pl, c);
  return run_gemv_kn<8, false>(g, pl, c);
}

}  // namespace ptsim
