// Mixture-of-experts routing programs of the validation bundle (the Qwen3-30B-A3B layer ops):
//
//   topk_kernel  validation/pytorchsim/layer_op_router_post_*/01__topk_kernel: per row of E values, K passes;
//                pass n takes the best value (largest, or smallest) among the program's EP candidate columns
//                (columns past E hold the spent value, -inf for largest), then the smallest column holding
//                it, and overwrites that column with the spent value.  Spent columns stay candidates, so a
//                row with fewer than K finite values repeats an index, exactly as the reference does.  One
//                warp per row, the row in registers, warp shuffles for the best value and the first column.
//   sort_kernel  validation/pytorchsim/layer_op_dispatch_*/00__sort_kernel: each row sorted by the key
//                k = x (int) or the order-preserving integer of an fp32 x (NaN canonical and last, -0 equal
//                to +0), complemented when descending, ties broken by source position -- a unique order,
//                so any correct sort gives the reference's output.  One 1024-thread CTA per row:
//                  - keys spanning at most 256 values (the expert ids being routed): a stable counting sort,
//                    each warp owning a contiguous segment; per-warp histograms by __match_any_sync, one
//                    prefix over (key, warp), and a second pass that scatters every key to its offset plus
//                    its rank among equal keys before it in the warp's chunk;
//                  - otherwise a bitonic sort of (key, position) pairs in shared memory, up to 8192 keys;
//                  - a longer row with a wider key range records PTSIM_E_UNSUPPORTED in the status word.
#pragma once
#include <climits>
#include "common.cuh"

namespace ptsim {

struct TopkArgs {
  const void *x;
  void *v;
  int64_t *idx;
  int64_t row_begin, row_end, cols, k, cols_padded;
  int32_t x_dt, v_dt, largest, pad;
};

template <int NPL>
__global__ void __launch_bounds__(256) topk_kernel(const __grid_constant__ TopkArgs g) {
  const int lane = threadIdx.x & 31;
  const int64_t r = g.row_begin + ((int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  if (r >= g.row_end) return;
  const float spent = g.largest ? -INFINITY : INFINITY;
  float x[NPL];
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int64_t c = int64_t(j) * 32 + lane;
    x[j] = c < g.cols ? ld_any(g.x, g.x_dt, r * g.cols + c) : spent;
  }
  for (int64_t n = 0; n < g.k; ++n) {
    float b = spent;
#pragma unroll
    for (int j = 0; j < NPL; ++j)
      if (int64_t(j) * 32 + lane < g.cols_padded) b = g.largest ? fmaxf(b, x[j]) : fminf(b, x[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, b, o);
      b = g.largest ? fmaxf(b, w) : fminf(b, w);
    }
    int at = 0x7fffffff;
#pragma unroll
    for (int j = NPL - 1; j >= 0; --j) {
      const int c = j * 32 + lane;
      if (c < g.cols_padded && x[j] == b) at = c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) at = min(at, __shfl_xor_sync(0xffffffffu, at, o));
    if (lane == 0) {
      st_any(g.v, g.v_dt, r * g.k + n, b);
      g.idx[r * g.k + n] = at;
    }
#pragma unroll
    for (int j = 0; j < NPL; ++j)
      if (j * 32 + lane == at) x[j] = spent;
  }
}

struct SortArgs {
  const void *x;
  void *v;
  int64_t *idx;
  int64_t row_begin, cols;
  int32_t x_dt, v_dt, descending, float_keys;
};

constexpr int kSortThreads = 1024;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortCountRange = 256;
constexpr int kSortBitonicMax = 8192;
constexpr int kSortSmem = kSortBitonicMax * 12 + 512;   // keys (8 B) + positions (4 B); the histogram fits inside

__device__ __forceinline__ int64_t sort_key(const SortArgs &g, int64_t at) {
  int64_t k;
  if (g.float_keys) {
    const float f = reinterpret_cast<const float *>(g.x)[at];
    const int32_t bits = f != f ? 0x7FC00000 : (f == 0.0f ? 0 : __float_as_int(f));
    k = int64_t(bits ^ ((bits >> 31) & 0x7FFFFFFF));
  } else {
    k = g.x_dt == PTSIM_DT_I32 ? int64_t(reinterpret_cast<const int32_t *>(g.x)[at])
                               : reinterpret_cast<const int64_t *>(g.x)[at];
  }
  return g.descending ? ~k : k;
}

__device__ __forceinline__ void sort_store(const SortArgs &g, int64_t at, int64_t k, int64_t src) {
  if (g.descending) k = ~k;
  if (g.float_keys) {
    const int32_t bits = int32_t(k);
    st_any(g.v, g.v_dt, at, __int_as_float(bits ^ ((bits >> 31) & 0x7FFFFFFF)));
  } else if (g.v_dt == PTSIM_DT_I32) {
    reinterpret_cast<int32_t *>(g.v)[at] = int32_t(k);
  } else {
    reinterpret_cast<int64_t *>(g.v)[at] = k;
  }
  g.idx[at] = src;
}

__global__ void __launch_bounds__(kSortThreads, 1) sort_kernel(const __grid_constant__ SortArgs g) {
  extern __shared__ __align__(16) uint8_t sort_smem[];
  __shared__ long long s_min[kSortWarps], s_max[kSortWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r = g.row_begin + blockIdx.x;
  const int64_t base = r * g.cols;
  const int64_t n = g.cols;
  // 1. the row's key range
  long long lo = LLONG_MAX, hi = LLONG_MIN;
  for (int64_t c0 = tid; c0 < n; c0 += 8 * kSortThreads) {
    long long k[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {   // eight loads in flight per thread
      const int64_t c = c0 + int64_t(u) * kSortThreads;
      k[u] = c < n ? sort_key(g, base + c) : lo;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (c0 + int64_t(u) * kSortThreads >= n) break;
      lo = k[u] < lo ? k[u] : lo;
      hi = k[u] > hi ? k[u] : hi;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long a = __shfl_xor_sync(0xffffffffu, lo, o), b = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = a < lo ? a : lo;
    hi = b > hi ? b : hi;
  }
  if (lane == 0) {
    s_min[warp] = lo;
    s_max[warp] = hi;
  }
  __syncthreads();
  lo = s_min[0];
  hi = s_max[0];
  for (int w = 1; w < kSortWarps; ++w) {
    lo = s_min[w] < lo ? s_min[w] : lo;
    hi = s_max[w] > hi ? s_max[w] : hi;
  }
  if (n == 0) return;
  const unsigned long long span = static_cast<unsigned long long>(hi) - static_cast<unsigned long long>(lo);
  if (span < kSortCountRange) {
    // 2a. stable counting sort; hist[w][key] = warp w's count, then its first output position.
    int *hist = reinterpret_cast<int *>(sort_smem);   // [kSortWarps][kSortCountRange]
    for (int i = tid; i < kSortWarps * kSortCountRange; i += kSortThreads) hist[i] = 0;
    __syncthreads();
    const int64_t seg = ceil_div(n, kSortWarps);
    const int64_t s0 = warp * seg, s1 = s0 + seg < n ? s0 + seg : n;
    // The keys' offsets from the minimum fit a byte: rows up to kSortBitonicMax * 8 keep them in shared
    // memory after the histogram pass, so the scatter pass reads no global memory.
    uint8_t *k8 = sort_smem + kSortWarps * kSortCountRange * 4;
    const bool cache = n <= int64_t(kSortSmem - kSortWarps * kSortCountRange * 4);
    for (int64_t c0 = s0; c0 < s1; c0 += 32 * 32) {
      int key[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) {   // a whole 1024-key block in flight per warp
        const int64_t c = c0 + u * 32 + lane;
        key[u] = c < s1 ? int(sort_key(g, base + c) - lo) : -1;
      }
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        if (c0 + u * 32 >= s1) break;
        const unsigned m = __match_any_sync(0xffffffffu, key[u]);
        if (key[u] >= 0 && lane == __ffs(m) - 1) hist[warp * kSortCountRange + key[u]] += __popc(m);
        if (cache && key[u] >= 0) k8[c0 + u * 32 + lane] = uint8_t(key[u]);
        __syncwarp();
      }
    }
    __syncthreads();
    if (warp == 0) {
      // totals per key (8 keys per lane), an exclusive scan across keys, then per-warp offsets
      int run = 0;
      for (int j = 0; j < kSortCountRange / 32; ++j)
        for (int w = 0; w < kSortWarps; ++w) run += hist[w * kSortCountRange + lane * 8 + j];
      int incl = run;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int off = incl - run;
      for (int j = 0; j < kSortCountRange / 32; ++j) {
        const int key = lane * 8 + j;
        for (int w = 0; w < kSortWarps; ++w) {
          const int cnt = hist[w * kSortCountRange + key];
          hist[w * kSortCountRange + key] = off;
          off += cnt;
        }
      }
    }
    __syncthreads();
    for (int64_t c0 = s0; c0 < s1; c0 += 32) {
      const int64_t c = c0 + lane;
      const int key = c < s1 ? (cache ? int(k8[c]) : int(sort_key(g, base + c) - lo)) : -1;
      const int64_t k = int64_t(lo) + key;
      const unsigned m = __match_any_sync(0xffffffffu, key);
      if (key >= 0) {
        const int rank = __popc(m & ((1u << lane) - 1u));
        sort_store(g, base + hist[warp * kSortCountRange + key] + rank, k, c);
      }
      __syncwarp();
      if (key >= 0 && lane == __ffs(m) - 1) hist[warp * kSortCountRange + key] += __popc(m);
      __syncwarp();
    }
    return;
  }
  if (n > kSortBitonicMax) {
    if (tid == 0) record_status(PTSIM_E_UNSUPPORTED);
    return;
  }
  // 2b. bitonic sort of (key, position) over the next power of two; padding sorts last.
  int p2 = 1;
  while (p2 < n) p2 <<= 1;
  long long *sk = reinterpret_cast<long long *>(sort_smem);
  int *sp = reinterpret_cast<int *>(sort_smem + kSortBitonicMax * 8);
  for (int i = tid; i < p2; i += kSortThreads) {
    sk[i] = i < n ? sort_key(g, base + i) : LLONG_MAX;
    sp[i] = i;
  }
  __syncthreads();
  for (int size = 2; size <= p2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < (p2 >> 1); i += kSortThreads) {
        const int a = 2 * stride * (i / stride) + (i % stride), b = a + stride;
        const bool up = (a & size) == 0;
        const long long ka = sk[a], kb = sk[b];
        const int pa = sp[a], pb = sp[b];
        const bool greater = ka > kb || (ka == kb && pa > pb);
        if (greater == up) {
          sk[a] = kb;
          sk[b] = ka;
          sp[a] = pb;
          sp[b] = pa;
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < n; i += kSortThreads) sort_store(g, base + i, sk[i], sp[i]);
}

// ---------------------------------------------------------------------------------------------------
// Row gather (index_select): the MoE dispatch's token copy (validation/pytorchsim/layer_op_dispatch_*/01_*:
// out[x] = table[x % C + C * t(idx[x // C])], t = Python floor division of the sorted position by top-k
// with negative results wrapped by the token count) and any program of that shape.  The lowering states t
// as an int64 program (ptsim_iinsn); one warp per output row evaluates it once and copies the row.
// ---------------------------------------------------------------------------------------------------
struct GatherArgs {
  const void *table;
  void *out;
  const void *idx;
  int64_t row_begin, row_end, cols, table_rows;
  int32_t table_dt, out_dt, idx_dt, ncode;
  int32_t vec, pad;
  ptsim_map idx_map;
  ptsim_iinsn code[PTSIM_MAX_ICODE];
};

__device__ __forceinline__ int64_t gather_row_of(const GatherArgs &g, int64_t r) {
  const ptsim_map &m = g.idx_map;
  int64_t at = m.offset;
  for (int d = 0; d < m.ndigit; ++d) {
    int64_t q = r / m.div[d];
    if (m.mod[d] > 0) q %= m.mod[d];
    at += q * m.stride[d];
  }
  const int64_t loaded = g.idx_dt == PTSIM_DT_I32 ? int64_t(reinterpret_cast<const int32_t *>(g.idx)[at])
                                                   : reinterpret_cast<const int64_t *>(g.idx)[at];
  int64_t reg[PTSIM_MAX_ICODE];
  int64_t res = 0;
  for (int i = 0; i < g.ncode; ++i) {
    const ptsim_iinsn &in = g.code[i];
    const int64_t a = reg[in.a & 31], b = reg[in.b & 31];
    int64_t v;
    switch (in.op) {
      case PTSIM_I_LOAD: v = loaded; break;
      case PTSIM_I_CONST: v = in.imm; break;
      case PTSIM_I_ADD: v = int64_t(uint64_t(a) + uint64_t(b)); break;
      case PTSIM_I_SUB: v = int64_t(uint64_t(a) - uint64_t(b)); break;
      case PTSIM_I_MUL: v = int64_t(uint64_t(a) * uint64_t(b)); break;
      case PTSIM_I_DIV: v = b == 0 ? 0 : (a == LLONG_MIN && b == -1 ? a : a / b); break;
      case PTSIM_I_MOD: v = b == 0 ? 0 : (a == LLONG_MIN && b == -1 ? 0 : a % b); break;
      case PTSIM_I_INV: v = ~a; break;
      case PTSIM_I_LT: v = a < b; break;
      case PTSIM_I_LE: v = a <= b; break;
      case PTSIM_I_GT: v = a > b; break;
      case PTSIM_I_GE: v = a >= b; break;
      case PTSIM_I_EQ: v = a == b; break;
      case PTSIM_I_NE: v = a != b; break;
      case PTSIM_I_WHERE: v = reg[in.c & 31] ? a : b; break;
      case PTSIM_I_AND: v = a & b; break;
      case PTSIM_I_OR: v = a | b; break;
      case PTSIM_I_XOR: v = a ^ b; break;
      case PTSIM_I_SHR: v = a >> (b & 63); break;
      case PTSIM_I_SHL: v = int64_t(uint64_t(a) << (b & 63)); break;
      default: v = 0; break;
    }
    reg[in.dst & 31] = v;
    res = v;
  }
  return res;
}

__global__ void __launch_bounds__(256) gather_rows_kernel(const __grid_constant__ GatherArgs g) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  // Each warp takes kGatherRows consecutive rows at a time: lane i < kGatherRows evaluates row i's index
  // program (once per row, not once per lane), then the warp copies the rows, each row's table index
  // broadcast by shuffle.
  constexpr int kGatherRows = 8;
  for (int64_t r0 = g.row_begin + ((int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * kGatherRows;
       r0 < g.row_end; r0 += warps * kGatherRows) {
    const int64_t mine = lane < kGatherRows && r0 + lane < g.row_end ? gather_row_of(g, r0 + lane) : 0;
    const int nrow = g.row_end - r0 < kGatherRows ? int(g.row_end - r0) : kGatherRows;
    for (int j = 0; j < nrow; ++j) {
    const int64_t r = r0 + j;
    const int64_t t = __shfl_sync(0xffffffffu, mine, j);
    if (t < 0 || t >= g.table_rows) {
      if (lane == 0) record_status(PTSIM_E_OOB);
      continue;
    }
    if (g.vec) {
      // same element type, 16-byte rows: raw copy
      const int64_t n16 = g.cols * dtype_size(g.out_dt) / 16;
      const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(g.table) + t * g.cols * dtype_size(g.table_dt));
      uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(g.out) + r * g.cols * dtype_size(g.out_dt));
      int64_t i = lane;
      for (; i + 7 * 32 < n16; i += 8 * 32) {   // eight 16-byte loads in flight per lane
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldg(src + i + u * 32);
#pragma unroll
        for (int u = 0; u < 8; ++u) __stcs(dst + i + u * 32, v[u]);
      }
      for (; i < n16; i += 32) __stcs(dst + i, __ldg(src + i));
    } else {
      for (int64_t c2 = lane; c2 < g.cols; c2 += 32)
        st_any(g.out, g.out_dt, r * g.cols + c2, ld_any(g.table, g.table_dt, t * g.cols + c2));
    }
    }
  }
}

int launch_gather_rows(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c) {
  const ptsim_gather_params &p = d.p.gat;
  GatherArgs g;
  memset(&g, 0, sizeof(g));
  g.table = ptrs[p.table_arg];
  g.out = ptrs[p.out_arg];
  g.idx = ptrs[p.idx_arg];
  g.row_begin = lo * d.unit_size;
  g.row_end = hi * d.unit_size < p.rows ? hi * d.unit_size : p.rows;
  g.cols = p.cols;
  g.table_rows = p.table_rows;
  g.table_dt = d.arg_dtype[p.table_arg];
  g.out_dt = d.arg_dtype[p.out_arg];
  g.idx_dt = d.arg_dtype[p.idx_arg];
  g.ncode = p.ncode;
  g.idx_map = p.idx_map;
  memcpy(g.code, p.code, sizeof(g.code));
  if (g.idx_dt != PTSIM_DT_I64 && g.idx_dt != PTSIM_DT_I32) return fail(PTSIM_E_UNSUPPORTED, "gather indices must be int32 or int64");
  const bool floaty = [](int dt) { return dt == PTSIM_DT_F32 || dt == PTSIM_DT_BF16 || dt == PTSIM_DT_F16; }(g.table_dt);
  if (g.table_dt != g.out_dt && !(floaty && (g.out_dt == PTSIM_DT_F32 || g.out_dt == PTSIM_DT_BF16 || g.out_dt == PTSIM_DT_F16)))
    return fail(PTSIM_E_UNSUPPORTED, "gather converts between float types only");
  const int esz = dtype_size(g.out_dt);
  g.vec = g.table_dt == g.out_dt && (g.cols * esz) % 16 == 0 && reinterpret_cast<uintptr_t>(g.table) % 16 == 0 &&
          reinterpret_cast<uintptr_t>(g.out) % 16 == 0;
  if (!g.vec && !floaty) return fail(PTSIM_E_UNSUPPORTED, "gather of integer rows needs 16-byte rows");
  if (g.row_end <= g.row_begin) return PTSIM_OK;
  int64_t blocks = ceil_div(g.row_end - g.row_begin, 8 * 8);   // 8 warps of 8 rows
  if (blocks > int64_t(c.sm_count) * 16) blocks = int64_t(c.sm_count) * 16;
  gather_rows_kernel<<<unsigned(blocks), 256, 0, c.stream>>>(g);
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

// ---------------------------------------------------------------------------------------------------
// Gather-sum: the MoE combine (validation/pytorchsim/layer_op_combine_*/03_*: out[t, d] = sum over the top-k
// terms k of w[t, k] * expert_out[p(t, k), d], p the row where token t's k-th expert wrote it, read through
// the expert id, that expert's running offsets and the slot).  The index programs of 32 (row, term) pairs
// run at once on one warp; each row is then accumulated over its terms in order by 256 threads, 8 columns
// per thread per step with 16-byte loads.
// ---------------------------------------------------------------------------------------------------
struct GsumArgs {
  const void *arg[PTSIM_MAX_ARGS];
  int64_t numel[PTSIM_MAX_ARGS];
  int32_t dt[PTSIM_MAX_ARGS];
  void *out;
  const void *table;
  int64_t row_begin, row_end, cols, terms, table_rows;
  int32_t out_dt, table_dt, w_arg, ncode;
  ptsim_map w_map;
  ptsim_map maps[PTSIM_GSUM_MAPS];
  ptsim_iinsn code[PTSIM_MAX_ICODE];
  int32_t wdiv, nres, wdiv_arg, res_dt;   // weight divisor; residual rows (same element type each)
  const void *res[2];
  int64_t wdiv_offset, wdiv_stride;
};

__device__ __forceinline__ int64_t map_at(const ptsim_map &m, int64_t f) {
  int64_t at = m.offset;
  for (int d = 0; d < m.ndigit; ++d) {
    int64_t q = f / m.div[d];
    if (m.mod[d] > 0) q %= m.mod[d];
    at += q * m.stride[d];
  }
  return at;
}

// Element `at` of argument `a` as int64 (integer arguments) -- false when `at` is outside it.
__device__ __forceinline__ bool load_int(const GsumArgs &g, int a, int64_t at, int64_t &v) {
  if (a < 0 || a >= PTSIM_MAX_ARGS || at < 0 || at >= g.numel[a]) return false;
  switch (g.dt[a]) {
    case PTSIM_DT_I64: v = reinterpret_cast<const int64_t *>(g.arg[a])[at]; return true;
    case PTSIM_DT_I32: v = reinterpret_cast<const int32_t *>(g.arg[a])[at]; return true;
    case PTSIM_DT_I16: v = reinterpret_cast<const int16_t *>(g.arg[a])[at]; return true;
    case PTSIM_DT_I8: v = reinterpret_cast<const int8_t *>(g.arg[a])[at]; return true;
    case PTSIM_DT_U8: v = reinterpret_cast<const uint8_t *>(g.arg[a])[at]; return true;
  }
  return false;
}

// The table row of term f = r * terms + k, or -1 when an index read fell outside its tensor.
__device__ int64_t gsum_row_of(const GsumArgs &g, int64_t f) {
  int64_t reg[PTSIM_MAX_ICODE];
  int64_t res = 0;
  for (int i = 0; i < g.ncode; ++i) {
    const ptsim_iinsn &in = g.code[i];
    const int64_t a = reg[in.a & 31], b = reg[in.b & 31];
    int64_t v = 0;
    switch (in.op) {
      case PTSIM_I_LOAD:
        if (in.a >= PTSIM_GSUM_MAPS || !load_int(g, g.maps[in.a].arg, map_at(g.maps[in.a], f), v)) return -1;
        break;
      case PTSIM_I_LOADI:
        if (!load_int(g, in.c, a, v)) return -1;
        break;
      case PTSIM_I_CONST: v = in.imm; break;
      case PTSIM_I_ADD: v = int64_t(uint64_t(a) + uint64_t(b)); break;
      case PTSIM_I_SUB: v = int64_t(uint64_t(a) - uint64_t(b)); break;
      case PTSIM_I_MUL: v = int64_t(uint64_t(a) * uint64_t(b)); break;
      case PTSIM_I_DIV: v = b == 0 ? 0 : (a == LLONG_MIN && b == -1 ? a : a / b); break;
      case PTSIM_I_MOD: v = b == 0 ? 0 : (a == LLONG_MIN && b == -1 ? 0 : a % b); break;
      case PTSIM_I_INV: v = ~a; break;
      case PTSIM_I_LT: v = a < b; break;
      case PTSIM_I_LE: v = a <= b; break;
      case PTSIM_I_GT: v = a > b; break;
      case PTSIM_I_GE: v = a >= b; break;
      case PTSIM_I_EQ: v = a == b; break;
      case PTSIM_I_NE: v = a != b; break;
      case PTSIM_I_WHERE: v = reg[in.c & 31] ? a : b; break;
      case PTSIM_I_AND: v = a & b; break;
      case PTSIM_I_OR: v = a | b; break;
      case PTSIM_I_XOR: v = a ^ b; break;
      case PTSIM_I_SHR: v = a >> (b & 63); break;
      case PTSIM_I_SHL: v = int64_t(uint64_t(a) << (b & 63)); break;
    }
    reg[in.dst & 31] = v;
    res = v;
  }
  return res;
}

// One output row's 8-column slice: the slice of every term's table row loaded (all TERMS loads in flight when
// the term count is a template constant), then accumulated in term order, the residual rows added, stored.
template <int TERMS>
__device__ __forceinline__ void gsum_slice(const GsumArgs &g, const int64_t *rows, const float *ws, int nterms,
                                           int64_t orow, int64_t c8) {
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const bool vec = g.table_dt == PTSIM_DT_BF16 && c8 + 8 <= g.cols && (g.cols % 8) == 0;
  if (TERMS > 0 && vec) {
    uint4 v[TERMS > 0 ? TERMS : 1];
#pragma unroll
    for (int k = 0; k < TERMS; ++k)
      v[k] = rows[k] >= 0 ? __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(g.table) + rows[k] * g.cols + c8))
                          : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < TERMS; ++k) {
      if (rows[k] < 0) continue;
      const uint32_t wsv[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] = fmaf(lo_bf16(wsv[e]), ws[k], acc[2 * e]);
        acc[2 * e + 1] = fmaf(hi_bf16(wsv[e]), ws[k], acc[2 * e + 1]);
      }
    }
  } else {
    for (int k = 0; k < nterms; ++k) {
      const int64_t t = rows[k];
      if (t < 0) continue;
      for (int e = 0; e < 8 && c8 + e < g.cols; ++e) acc[e] = fmaf(ld_any(g.table, g.table_dt, t * g.cols + c8 + e), ws[k], acc[e]);
    }
  }
  if (g.nres > 0) {   // (res0 + res1) + sum, read at the output's own index before it is written
    for (int e = 0; e < 8 && c8 + e < g.cols; ++e) {
      const int64_t at = orow * g.cols + c8 + e;
      float rs = ld_any(g.res[0], g.res_dt, at);
      if (g.nres > 1) rs = __fadd_rn(rs, ld_any(g.res[1], g.res_dt, at));
      acc[e] = __fadd_rn(rs, acc[e]);
    }
  }
  if (g.out_dt == PTSIM_DT_BF16 && c8 + 8 <= g.cols && (g.cols % 8) == 0) {
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    __stcs(reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(g.out) + orow * g.cols + c8), o);
  } else {
    for (int e = 0; e < 8 && c8 + e < g.cols; ++e) st_any(g.out, g.out_dt, orow * g.cols + c8 + e, acc[e]);
  }
}

// Warp-specialised: warp 8 runs a group's (row, term) index programs (32 at once, lane l: row r0 + l / terms,
// term l % terms) into one half of a double-buffered table while warps 0-7 stream the group before it from
// the other half; named barriers hand each half over (1 + b: filled, 3 + b: drained, 288 threads each).
__device__ __forceinline__ void named_bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void named_bar_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }

constexpr int kGsumThreads = 288;

template <int TERMS>
__global__ void __launch_bounds__(kGsumThreads) gather_sum_kernel(const __grid_constant__ GsumArgs g) {
  __shared__ int64_t s_row[2][32];
  __shared__ float s_w[2][32];
  const int nterms = TERMS > 0 ? TERMS : int(g.terms);
  const int per = 32 / nterms;
  const int64_t stride = int64_t(gridDim.x) * per;
  const int64_t first = g.row_begin + int64_t(blockIdx.x) * per;
  const int64_t ngroups = first < g.row_end ? (g.row_end - first + stride - 1) / stride : 0;
  const int warp = threadIdx.x >> 5;
  if (warp == 8) {
    const int lane = threadIdx.x & 31;
    for (int64_t i = 0; i < ngroups; ++i) {
      const int b = int(i & 1);
      const int64_t r0 = first + i * stride;
      if (i >= 2) named_bar_sync(3 + b, kGsumThreads);   // the consumers are done with this half
      int64_t trow = -1;
      float w = 0.f;
      const int64_t r = r0 + lane / nterms;
      if (lane < per * nterms && r < g.row_end) {
        const int64_t f = r * g.terms + lane % nterms;
        trow = gsum_row_of(g, f);
        const int64_t wat = map_at(g.w_map, f);
        const int64_t dat = g.wdiv_offset + r * g.wdiv_stride;
        if (trow < 0 || trow >= g.table_rows || wat < 0 || wat >= g.numel[g.w_arg] ||
            (g.wdiv && (dat < 0 || dat >= g.numel[g.wdiv_arg]))) {
          record_status(PTSIM_E_OOB);
          trow = -1;
        } else {
          w = ld_any(g.arg[g.w_arg], g.dt[g.w_arg], wat);
          if (g.wdiv) w = __fdiv_rn(w, ld_any(g.arg[g.wdiv_arg], g.dt[g.wdiv_arg], dat));
        }
      }
      s_row[b][lane] = trow;
      s_w[b][lane] = w;
      named_bar_arrive(1 + b, kGsumThreads);
    }
    // Match the consumers' drained-arrivals of the last group of each half.
    for (int64_t i = ngroups >= 2 ? ngroups - 2 : 0; i < ngroups; ++i) named_bar_sync(3 + int(i & 1), kGsumThreads);
  } else {
    for (int64_t i = 0; i < ngroups; ++i) {
      const int b = int(i & 1);
      const int64_t r0 = first + i * stride;
      named_bar_sync(1 + b, kGsumThreads);
      for (int j = 0; j < per && r0 + j < g.row_end; ++j)
        for (int64_t c8 = int64_t(threadIdx.x) * 8; c8 < g.cols; c8 += 256 * 8)
          gsum_slice<TERMS>(g, s_row[b] + j * nterms, s_w[b] + j * nterms, nterms, r0 + j, c8);
      named_bar_arrive(3 + b, kGsumThreads);
    }
  }
}

int launch_gather_sum(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c) {
  const ptsim_gsum_params &p = d.p.gsum;
  GsumArgs g;
  memset(&g, 0, sizeof(g));
  for (int a = 0; a < d.nargs; ++a) {
    g.arg[a] = ptrs[a];
    g.numel[a] = d.arg_numel[a];
    g.dt[a] = d.arg_dtype[a];
  }
  if (p.terms < 1 || p.terms > 32) return fail(PTSIM_E_UNSUPPORTED, "gather-sum over %lld terms (runs 1-32)", (long long)p.terms);
  const bool floaty = [](int dt) { return dt == PTSIM_DT_F32 || dt == PTSIM_DT_BF16 || dt == PTSIM_DT_F16; }(d.arg_dtype[p.table_arg]);
  if (!floaty || (d.arg_dtype[p.out_arg] != PTSIM_DT_F32 && d.arg_dtype[p.out_arg] != PTSIM_DT_BF16 &&
                  d.arg_dtype[p.out_arg] != PTSIM_DT_F16))
    return fail(PTSIM_E_UNSUPPORTED, "gather-sum runs float tables and outputs");
  g.out = ptrs[p.out_arg];
  g.table = ptrs[p.table_arg];
  g.row_begin = lo * d.unit_size;
  g.row_end = hi * d.unit_size < p.rows ? hi * d.unit_size : p.rows;
  g.cols = p.cols;
  g.terms = p.terms;
  g.table_rows = p.table_rows;
  g.out_dt = d.arg_dtype[p.out_arg];
  g.table_dt = d.arg_dtype[p.table_arg];
  g.w_arg = p.w_arg;
  g.ncode = p.ncode;
  g.w_map = p.w_map;
  memcpy(g.maps, p.maps, sizeof(g.maps));
  memcpy(g.code, p.code, sizeof(g.code));
  g.wdiv = p.wdiv;
  g.wdiv_arg = p.wdiv_arg;
  g.wdiv_offset = p.wdiv_offset;
  g.wdiv_stride = p.wdiv_stride;
  g.nres = p.nres;
  for (int k = 0; k < p.nres; ++k) {
    g.res[k] = ptrs[p.res_arg[k]];
    if (d.arg_numel[p.res_arg[k]] < p.rows * p.cols || d.arg_dtype[p.res_arg[k]] != d.arg_dtype[p.res_arg[0]])
      return fail(PTSIM_E_UNSUPPORTED, "gather-sum residual %d: as many elements as the output, one element type", k);
  }
  g.res_dt = p.nres > 0 ? d.arg_dtype[p.res_arg[0]] : 0;
  if ((reinterpret_cast<uintptr_t>(g.table) | reinterpret_cast<uintptr_t>(g.out)) % 16 != 0)
    return fail(PTSIM_E_ARGS, "gather-sum table and output must be 16-byte aligned");
  if (g.row_end <= g.row_begin) return PTSIM_OK;
  const int per = 32 / int(p.terms);
  // Three CTAs per SM (288 threads, 64 registers), each taking several groups so the index programs of the
  // next one run under the current one's stream.
  int64_t blocks = ceil_div(g.row_end - g.row_begin, per);
  if (blocks > int64_t(c.sm_count) * 3) blocks = int64_t(c.sm_count) * 3;
  if (p.terms == 8) gather_sum_kernel<8><<<unsigned(blocks), kGsumThreads, 0, c.stream>>>(g);
  else gather_sum_kernel<0><<<unsigned(blocks), kGsumThreads, 0, c.stream>>>(g);
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

int launch_topk(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c) {
  const ptsim_select_params &p = d.p.sel;
  const int xdt = d.arg_dtype[p.in_arg], vdt = d.arg_dtype[p.val_arg];
  if ((xdt != PTSIM_DT_F32 && xdt != PTSIM_DT_BF16) || (vdt != PTSIM_DT_F32 && vdt != PTSIM_DT_BF16) ||
      d.arg_dtype[p.idx_arg] != PTSIM_DT_I64)
    return fail(PTSIM_E_UNSUPPORTED, "top-k runs fp32/bf16 values with int64 indices");
  if (p.cols_padded < p.cols || p.cols_padded > 1024 || p.k < 0 || p.k > p.cols_padded)
    return fail(PTSIM_E_UNSUPPORTED, "top-k over %lld candidate columns, k = %lld (runs up to 1024 columns)",
                (long long)p.cols_padded, (long long)p.k);
  TopkArgs g;
  g.x = ptrs[p.in_arg];
  g.v = ptrs[p.val_arg];
  g.idx = reinterpret_cast<int64_t *>(ptrs[p.idx_arg]);
  g.row_begin = lo * d.unit_size;
  g.row_end = hi * d.unit_size < p.rows ? hi * d.unit_size : p.rows;
  g.cols = p.cols;
  g.k = p.k;
  g.cols_padded = p.cols_padded;
  g.x_dt = xdt;
  g.v_dt = vdt;
  g.largest = p.descending;
  g.pad = 0;
  if (g.row_end <= g.row_begin) return PTSIM_OK;
  const unsigned blocks = unsigned(ceil_div(g.row_end - g.row_begin, 8));
  const int npl = int(ceil_div(p.cols_padded, 32));
  if (npl <= 1) topk_kernel<1><<<blocks, 256, 0, c.stream>>>(g);
  else if (npl <= 2) topk_kernel<2><<<blocks, 256, 0, c.stream>>>(g);
  else if (npl <= 4) topk_kernel<4><<<blocks, 256, 0, c.stream>>>(g);
  else if (npl <= 8) topk_kernel<8><<<blocks, 256, 0, c.stream>>>(g);
  else if (npl <= 16) topk_kernel<16><<<blocks, 256, 0, c.stream>>>(g);
  else topk_kernel<32><<<blocks, 256, 0, c.stream>>>(g);
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

// ---------------------------------------------------------------------------------------------------
// Long rows (more than kSortBitonicMax keys, e.g. the dispatch's 8T expert ids): the stable counting sort over
// CTAs of 1024 keys (one key per thread) in three launches -- each chunk's key range; the row's range (keys
// spanning 256 values or more record PTSIM_E_UNSUPPORTED, as the one-CTA path does) and each chunk's
// histogram; then every chunk's base offset per key (the keys below it in the whole row plus the same key in
// earlier chunks), the ranks of its keys among earlier warps (per-warp counts in shared memory) and earlier
// lanes (__match_any_sync), and the scatter.  Grid (chunks, rows); scratch: per row and chunk the range (2 int64)
// and the histogram (256 int32).
// ---------------------------------------------------------------------------------------------------
constexpr int kSortChunk = 1024;

struct SortMultiArgs {
  SortArgs g;
  int64_t chunks;
  long long *range;   // [rows][chunks][2]
  int *hist;          // [rows][chunks][kSortCountRange]
};

__device__ __forceinline__ void block_minmax(long long &lo, long long &hi, long long *s_min, long long *s_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long a = __shfl_xor_sync(0xffffffffu, lo, o), b = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = a < lo ? a : lo;
    hi = b > hi ? b : hi;
  }
  if (lane == 0) {
    s_min[warp] = lo;
    s_max[warp] = hi;
  }
  __syncthreads();
  lo = s_min[0];
  hi = s_max[0];
  for (int w = 1; w < int(blockDim.x >> 5); ++w) {
    lo = s_min[w] < lo ? s_min[w] : lo;
    hi = s_max[w] > hi ? s_max[w] : hi;
  }
}

// The histogram and scatter launches are programmatic dependents: each kernel releases the next as it starts
// (griddepcontrol.launch_dependents), and the next waits (griddepcontrol.wait) for the previous grid to finish
// and flush before it reads that grid's scratch, so the launches overlap instead of queueing.
__global__ void __launch_bounds__(kSortChunk) sort_range_kernel(const __grid_constant__ SortMultiArgs a) {
  __shared__ long long s_min[32], s_max[32];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t row = a.g.row_begin + blockIdx.y, ri = blockIdx.y;
  const int64_t c = int64_t(blockIdx.x) * kSortChunk + threadIdx.x;
  long long lo = LLONG_MAX, hi = LLONG_MIN;
  if (c < a.g.cols) lo = hi = sort_key(a.g, row * a.g.cols + c);
  block_minmax(lo, hi, s_min, s_max);
  if (threadIdx.x == 0) {
    a.range[(ri * a.chunks + blockIdx.x) * 2] = lo;
    a.range[(ri * a.chunks + blockIdx.x) * 2 + 1] = hi;
  }
}

// The row's key range from its chunks' ranges (every thread holds it after the call).
__device__ __forceinline__ void row_range(const SortMultiArgs &a, int64_t ri, long long &lo, long long &hi,
                                          long long *s_min, long long *s_max) {
  lo = LLONG_MAX;
  hi = LLONG_MIN;
  for (int64_t q = threadIdx.x; q < a.chunks; q += blockDim.x) {
    const long long l = a.range[(ri * a.chunks + q) * 2], h = a.range[(ri * a.chunks + q) * 2 + 1];
    lo = l < lo ? l : lo;
    hi = h > hi ? h : hi;
  }
  block_minmax(lo, hi, s_min, s_max);
}

__global__ void __launch_bounds__(kSortChunk) sort_hist_kernel(const __grid_constant__ SortMultiArgs a) {
  __shared__ long long s_min[32], s_max[32];
  __shared__ int h[kSortCountRange];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t row = a.g.row_begin + blockIdx.y, ri = blockIdx.y;
  long long lo, hi;
  row_range(a, ri, lo, hi, s_min, s_max);
  if (static_cast<unsigned long long>(hi) - static_cast<unsigned long long>(lo) >= kSortCountRange) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_status(PTSIM_E_UNSUPPORTED);
    return;
  }
  for (int i = threadIdx.x; i < kSortCountRange; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t c = int64_t(blockIdx.x) * kSortChunk + threadIdx.x;
  if (c < a.g.cols) atomicAdd(&h[int(sort_key(a.g, row * a.g.cols + c) - lo)], 1);
  __syncthreads();
  for (int i = threadIdx.x; i < kSortCountRange; i += blockDim.x)
    a.hist[(ri * a.chunks + blockIdx.x) * kSortCountRange + i] = h[i];
}

__global__ void __launch_bounds__(kSortChunk) sort_scatter_kernel(const __grid_constant__ SortMultiArgs a) {
  __shared__ long long s_min[32], s_max[32];
  __shared__ int tot[4][kSortCountRange], bef[4][kSortCountRange];
  __shared__ int off[kSortCountRange];
  __shared__ int wh[kSortWarps][kSortCountRange];   // per-warp counts, then per-warp first positions
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = a.g.row_begin + blockIdx.y, ri = blockIdx.y;
  long long lo, hi;
  row_range(a, ri, lo, hi, s_min, s_max);
  if (static_cast<unsigned long long>(hi) - static_cast<unsigned long long>(lo) >= kSortCountRange) return;
  // totals of every key over the row, and over the chunks before this one (4 threads per key)
  {
    const int key = tid % kSortCountRange, q = tid / kSortCountRange;
    int t = 0, b = 0;
    for (int64_t ch = q; ch < a.chunks; ch += 4) {
      const int v = a.hist[(ri * a.chunks + ch) * kSortCountRange + key];
      t += v;
      if (ch < int64_t(blockIdx.x)) b += v;
    }
    tot[q][key] = t;
    bef[q][key] = b;
  }
  const int64_t c = int64_t(blockIdx.x) * kSortChunk + tid;
  const int key = c < a.g.cols ? int(sort_key(a.g, row * a.g.cols + c) - lo) : -1;
  for (int i = tid; i < kSortWarps * kSortCountRange; i += kSortChunk) (&wh[0][0])[i] = 0;
  __syncthreads();
  if (warp == 0) {
    // exclusive scan of the totals over keys (8 keys per lane), plus the earlier chunks' count of each key
    int run = 0;
    for (int j = 0; j < kSortCountRange / 32; ++j) {
      const int k = lane * 8 + j;
      run += tot[0][k] + tot[1][k] + tot[2][k] + tot[3][k];
    }
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int o = incl - run;
    for (int j = 0; j < kSortCountRange / 32; ++j) {
      const int k = lane * 8 + j;
      off[k] = o + bef[0][k] + bef[1][k] + bef[2][k] + bef[3][k];
      o += tot[0][k] + tot[1][k] + tot[2][k] + tot[3][k];
    }
  }
  const unsigned m = __match_any_sync(0xffffffffu, key);
  if (key >= 0 && lane == __ffs(m) - 1) wh[warp][key] = __popc(m);
  __syncthreads();
  if (tid < kSortCountRange) {   // per-warp first positions of each key, warps in order
    int base = off[tid];
    for (int w = 0; w < kSortWarps; ++w) {
      const int n = wh[w][tid];
      wh[w][tid] = base;
      base += n;
    }
  }
  __syncthreads();
  if (key >= 0) {
    const int rank = __popc(m & ((1u << lane) - 1u));
    sort_store(a.g, row * a.g.cols + wh[warp][key] + rank, int64_t(lo) + key, c);
  }
}

// Scratch of a SORT launch: the multi-CTA path's ranges and histograms for every row (0 for rows it never takes).
int64_t sort_workspace(const ptsim_desc &d) {
  const ptsim_select_params &p = d.p.sel;
  if (p.cols <= kSortBitonicMax) return 0;
  const int64_t chunks = ceil_div(p.cols, int64_t(kSortChunk));
  return p.rows * chunks * int64_t(2 * sizeof(long long) + kSortCountRange * sizeof(int));
}

int launch_sort(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                const LaunchCtx &c) {
  const ptsim_select_params &p = d.p.sel;
  const int xdt = d.arg_dtype[p.in_arg], vdt = d.arg_dtype[p.val_arg];
  if (d.arg_dtype[p.idx_arg] != PTSIM_DT_I64) return fail(PTSIM_E_UNSUPPORTED, "sort writes int64 indices");
  if (p.float_keys ? (xdt != PTSIM_DT_F32 || (vdt != PTSIM_DT_F32 && vdt != PTSIM_DT_BF16))
                   : ((xdt != PTSIM_DT_I64 && xdt != PTSIM_DT_I32) || (vdt != PTSIM_DT_I64 && vdt != PTSIM_DT_I32)))
    return fail(PTSIM_E_UNSUPPORTED, "sort runs int32/int64 keys, or fp32 keys ordered by their bits");
  SortArgs g;
  g.x = ptrs[p.in_arg];
  g.v = ptrs[p.val_arg];
  g.idx = reinterpret_cast<int64_t *>(ptrs[p.idx_arg]);
  g.row_begin = lo * d.unit_size;
  const int64_t row_end = hi * d.unit_size < p.rows ? hi * d.unit_size : p.rows;
  g.cols = p.cols;
  g.x_dt = xdt;
  g.v_dt = vdt;
  g.descending = p.descending;
  g.float_keys = p.float_keys;
  if (row_end <= g.row_begin) return PTSIM_OK;
  const int64_t rows = row_end - g.row_begin;
  if (p.cols > kSortBitonicMax && rows <= 65535 && ws != nullptr && int64_t(ws_bytes) >= sort_workspace(d) &&
      reinterpret_cast<uintptr_t>(ws) % 16 == 0) {
    SortMultiArgs a;
    a.g = g;
    a.chunks = ceil_div(p.cols, int64_t(kSortChunk));
    a.range = reinterpret_cast<long long *>(ws);
    a.hist = reinterpret_cast<int *>(a.range + rows * a.chunks * 2);
    const dim3 grid(unsigned(a.chunks), unsigned(rows));
    sort_range_kernel<<<grid, kSortChunk, 0, c.stream>>>(a);
    PTSIM_CUDA(cudaGetLastError());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kSortChunk, 1, 1);
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PTSIM_CUDA(cudaLaunchKernelEx(&cfg, sort_hist_kernel, a));
    PTSIM_CUDA(cudaLaunchKernelEx(&cfg, sort_scatter_kernel, a));
    return PTSIM_OK;
  }
  PTSIM_CUDA((smem_limit_once<sort_kernel>(kSortSmem, c.device)));
  sort_kernel<<<unsigned(row_end - g.row_begin), kSortThreads, kSortSmem, c.stream>>>(g);
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

}  // namespace ptsim
