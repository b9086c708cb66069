// Integer tables: the MoE routing bookkeeping (validation/pytorchsim/layer_op_gmm_*/01_* to 03_*,
// layer_op_combine_*/00_* to 02_*): expert counts, their running totals, group offsets, the slot of each
// routed row.  An int64 program runs for every element (x, r) of a [rows, cols] space and each output
// stores one of its registers per element, as the row's total over r, or as the inclusive running total
// over r.
//
// Layout: a CTA is TX rows x TR segments (TX * TR = 256 threads, x fastest so consecutive lanes store
// consecutive rows where the table is x-contiguous, as the combine's [8T, 128] running counts are).  A
// thread walks its segment of r in order.  When the r range is long against the rows (the combine's 128
// experts over 8T routed rows) it is split into chunks over a second grid dimension: a first kernel
// writes every segment's totals and every chunk's totals to the workspace, the second adds the totals
// before its own segment to its running values.  Otherwise one kernel scans the CTA's segments in shared
// memory.  Integer sums are exact in any order, so the split changes no result.
// ---------------------------------------------------------------------------------------------------
#pragma once
#include "common.cuh"

namespace ptsim {

constexpr int kItabThreads = 256;

struct ItabArgs {
  const void *arg[PTSIM_MAX_ARGS];
  int64_t numel[PTSIM_MAX_ARGS];
  int32_t dt[PTSIM_MAX_ARGS];
  int64_t rows, cols, row_begin, row_end;
  int64_t chunk_len;      // columns per chunk (cols when unsplit)
  int32_t ncode, nout, nacc, chunks;
  int32_t tx, tr;         // CTA layout: tx rows x tr segments
  int32_t acc_of[PTSIM_ITAB_OUTS];   // accumulator slot of a SUM / SCAN output, -1 for ELEM
  ptsim_map maps[PTSIM_ITAB_MAPS];
  ptsim_itab_out out[PTSIM_ITAB_OUTS];
  ptsim_iinsn code[PTSIM_MAX_ICODE];
  int64_t *seg;           // [chunks][tr][launch rows][nacc] segment totals (split launches)
  int64_t *chunk;         // [chunks][launch rows][nacc] chunk totals (split launches)
};

__device__ __forceinline__ int64_t itab_map(const ptsim_map &m, int64_t f) {
  int64_t at = m.offset;
  for (int d = 0; d < m.ndigit; ++d) {
    int64_t q = f / m.div[d];
    if (m.mod[d] > 0) q %= m.mod[d];
    at += q * m.stride[d];
  }
  return at;
}

__device__ __forceinline__ int64_t itab_load(const ItabArgs &g, int a, int64_t at) {
  if (a < 0 || a >= PTSIM_MAX_ARGS || at < 0 || at >= g.numel[a]) {
    record_status(PTSIM_E_OOB);
    return 0;
  }
  switch (g.dt[a]) {
    case PTSIM_DT_I64: return reinterpret_cast<const int64_t *>(g.arg[a])[at];
    case PTSIM_DT_I32: return reinterpret_cast<const int32_t *>(g.arg[a])[at];
    case PTSIM_DT_I16: return reinterpret_cast<const int16_t *>(g.arg[a])[at];
    case PTSIM_DT_I8: return reinterpret_cast<const int8_t *>(g.arg[a])[at];
    case PTSIM_DT_U8: return reinterpret_cast<const uint8_t *>(g.arg[a])[at];
  }
  record_status(PTSIM_E_OOB);
  return 0;
}

__device__ __forceinline__ void itab_store(const ItabArgs &g, int a, int64_t at, int64_t v) {
  if (at < 0 || at >= g.numel[a]) {
    record_status(PTSIM_E_OOB);
    return;
  }
  void *p = const_cast<void *>(g.arg[a]);
  switch (g.dt[a]) {
    case PTSIM_DT_I64: reinterpret_cast<int64_t *>(p)[at] = v; break;
    case PTSIM_DT_I32: reinterpret_cast<int32_t *>(p)[at] = int32_t(v); break;
    case PTSIM_DT_I16: reinterpret_cast<int16_t *>(p)[at] = int16_t(v); break;
    case PTSIM_DT_I8: reinterpret_cast<int8_t *>(p)[at] = int8_t(v); break;
    case PTSIM_DT_U8: reinterpret_cast<uint8_t *>(p)[at] = uint8_t(v); break;
  }
}

// Runs the program for element f into reg[] (registers are written once each, so every output's
// register holds its value when the program ends).
__device__ void itab_eval(const ItabArgs &g, int64_t f, int64_t *reg) {
#pragma unroll 1
  for (int i = 0; i < g.ncode; ++i) {
    const ptsim_iinsn &in = g.code[i];
    const int64_t a = reg[in.a & 31], b = reg[in.b & 31];
    int64_t v = 0;
    switch (in.op) {
      case PTSIM_I_LOAD: v = itab_load(g, in.c, itab_map(g.maps[in.a % PTSIM_ITAB_MAPS], f)); break;
      case PTSIM_I_LOADM: v = b ? itab_load(g, in.c, itab_map(g.maps[in.a % PTSIM_ITAB_MAPS], f)) : in.imm; break;
      case PTSIM_I_IDX: v = itab_map(g.maps[in.a % PTSIM_ITAB_MAPS], f); break;
      case PTSIM_I_LOADI: v = itab_load(g, in.c, a); break;
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
  }
}

struct ItabTile {
  int tx, tr;
  int64_t x, xi;           // global row, row within the launch
  bool live;               // x inside the launch
  int64_t s0, s1;          // this thread's segment of r
};

__device__ __forceinline__ ItabTile itab_tile(const ItabArgs &g) {
  ItabTile t;
  t.tx = int(threadIdx.x) % g.tx;
  t.tr = int(threadIdx.x) / g.tx;
  t.xi = int64_t(blockIdx.x) * g.tx + t.tx;
  t.x = g.row_begin + t.xi;
  t.live = t.x < g.row_end;
  const int64_t c0 = int64_t(blockIdx.y) * g.chunk_len;
  const int64_t c1 = min(g.cols, c0 + g.chunk_len);
  const int64_t per = (c1 - c0 + g.tr - 1) / g.tr;
  t.s0 = min(c1, c0 + t.tr * per);
  t.s1 = min(c1, t.s0 + per);
  return t;
}

// Split launches, first pass: each segment's and each chunk's totals of the accumulated outputs.
__global__ void __launch_bounds__(kItabThreads) itab_totals_kernel(const __grid_constant__ ItabArgs g) {
  __shared__ int64_t sh[kItabThreads * PTSIM_ITAB_OUTS];
  const ItabTile t = itab_tile(g);
  const int64_t nrows = g.row_end - g.row_begin;
  int64_t acc[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};
  int64_t reg[PTSIM_MAX_ICODE] = {};
  if (t.live)
    for (int64_t r = t.s0; r < t.s1; ++r) {
      itab_eval(g, t.x * g.cols + r, reg);
      for (int k = 0; k < g.nout; ++k)
        if (g.acc_of[k] >= 0) acc[g.acc_of[k]] += reg[g.out[k].reg & 31];
    }
  for (int j = 0; j < g.nacc; ++j) sh[threadIdx.x * PTSIM_ITAB_OUTS + j] = acc[j];
  if (t.live)
    for (int j = 0; j < g.nacc; ++j)
      g.seg[((int64_t(blockIdx.y) * g.tr + t.tr) * nrows + t.xi) * g.nacc + j] = acc[j];
  __syncthreads();
  if (t.tr == 0 && t.live)
    for (int j = 0; j < g.nacc; ++j) {
      int64_t s = 0;
      for (int q = 0; q < g.tr; ++q) s += sh[(q * g.tx + t.tx) * PTSIM_ITAB_OUTS + j];
      g.chunk[(int64_t(blockIdx.y) * nrows + t.xi) * g.nacc + j] = s;
    }
}

// The stores.  Unsplit: a first walk of the segment (when a running total is stored) gives the segment
// totals, scanned across the CTA's segments in shared memory.  Split: the totals come from the workspace.
__global__ void __launch_bounds__(kItabThreads) itab_kernel(const __grid_constant__ ItabArgs g) {
  __shared__ int64_t sh[kItabThreads * PTSIM_ITAB_OUTS];
  const ItabTile t = itab_tile(g);
  const int64_t nrows = g.row_end - g.row_begin;
  const bool split = g.chunks > 1;
  bool has_scan = false, has_sum = false;
  for (int k = 0; k < g.nout; ++k) {
    has_scan |= g.out[k].mode == PTSIM_ITAB_SCAN;
    has_sum |= g.out[k].mode == PTSIM_ITAB_SUM;
  }
  int64_t reg[PTSIM_MAX_ICODE] = {};
  int64_t base[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};   // total of every element before this segment
  int64_t row_total[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};
  if (split) {
    if (t.live) {
      for (int64_t c = 0; c < int64_t(g.chunks); ++c)
        for (int j = 0; j < g.nacc; ++j) {
          const int64_t v = g.chunk[(c * nrows + t.xi) * g.nacc + j];
          if (c < int64_t(blockIdx.y)) base[j] += v;
          row_total[j] += v;
        }
      for (int q = 0; q < t.tr; ++q)
        for (int j = 0; j < g.nacc; ++j) base[j] += g.seg[((int64_t(blockIdx.y) * g.tr + q) * nrows + t.xi) * g.nacc + j];
    }
  } else if (has_scan || has_sum) {
    int64_t acc[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};
    if (t.live && has_scan)
      for (int64_t r = t.s0; r < t.s1; ++r) {
        itab_eval(g, t.x * g.cols + r, reg);
        for (int k = 0; k < g.nout; ++k)
          if (g.acc_of[k] >= 0) acc[g.acc_of[k]] += reg[g.out[k].reg & 31];
      }
    if (has_scan) {
      for (int j = 0; j < g.nacc; ++j) sh[threadIdx.x * PTSIM_ITAB_OUTS + j] = acc[j];
      __syncthreads();
      for (int q = 0; q < g.tr; ++q)
        for (int j = 0; j < g.nacc; ++j) {
          const int64_t v = sh[(q * g.tx + t.tx) * PTSIM_ITAB_OUTS + j];
          if (q < t.tr) base[j] += v;
          row_total[j] += v;
        }
    }
  }
  int64_t run[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};
  if (t.live)
    for (int64_t r = t.s0; r < t.s1; ++r) {
      const int64_t f = t.x * g.cols + r;
      itab_eval(g, f, reg);
      for (int k = 0; k < g.nout; ++k) {
        const ptsim_itab_out &o = g.out[k];
        const int64_t v = reg[o.reg & 31];
        if (o.mode == PTSIM_ITAB_ELEM) {
          itab_store(g, o.arg, itab_map(g.maps[o.map % PTSIM_ITAB_MAPS], f), v);
        } else {
          const int j = g.acc_of[k];
          run[j] += v;
          if (o.mode == PTSIM_ITAB_SCAN) itab_store(g, o.arg, itab_map(g.maps[o.map % PTSIM_ITAB_MAPS], f), base[j] + run[j]);
        }
      }
    }
  if (!has_sum) return;
  if (!split && !has_scan) {   // the row totals are this pass's segment totals, summed across the CTA
    for (int j = 0; j < g.nacc; ++j) sh[threadIdx.x * PTSIM_ITAB_OUTS + j] = run[j];
    __syncthreads();
    for (int q = 0; q < g.tr; ++q)
      for (int j = 0; j < g.nacc; ++j) row_total[j] += sh[(q * g.tx + t.tx) * PTSIM_ITAB_OUTS + j];
  }
  if (t.live && t.tr == 0 && blockIdx.y == 0)
    for (int k = 0; k < g.nout; ++k)
      if (g.out[k].mode == PTSIM_ITAB_SUM)
        itab_store(g, g.out[k].arg, itab_map(g.maps[g.out[k].map % PTSIM_ITAB_MAPS], t.x * g.cols), row_total[g.acc_of[k]]);
}

struct ItabPlan {
  int tx, tr, chunks;
  int64_t chunk_len, xblocks;
};

// Rows per CTA up to 32, the rest of the 256 threads on segments; the r range split so about two CTAs
// per SM run, each thread with at least 16 columns, when the rows alone give too few CTAs.
static ItabPlan plan_itab(int64_t nrows, int64_t cols, int sm_count) {
  ItabPlan p;
  p.tx = 1;
  while (p.tx < 32 && p.tx < nrows) p.tx *= 2;
  p.tr = kItabThreads / p.tx;
  p.xblocks = (nrows + p.tx - 1) / p.tx;
  const int64_t want = (2 * int64_t(sm_count)) / (p.xblocks > 0 ? p.xblocks : 1);
  const int64_t by_len = cols / (int64_t(p.tr) * 16);
  int64_t chunks = want < by_len ? want : by_len;
  if (chunks < 2) chunks = 1;
  p.chunks = int(chunks);
  p.chunk_len = (cols + chunks - 1) / chunks;
  return p;
}

static int itab_naccs(const ptsim_itab_params &q) {
  int n = 0;
  for (int k = 0; k < q.nout; ++k) n += q.out[k].mode != PTSIM_ITAB_ELEM;
  return n;
}

// Workspace for any launch of the descriptor: a split launch has chunks * xblocks <= 2 * sm_count CTAs of
// 256 segments and 32 rows each.
int64_t itab_workspace(const ptsim_desc &d, int sm_count) {
  const int nacc = itab_naccs(d.p.itab);
  if (nacc == 0) return 0;
  return (2 * int64_t(sm_count) * kItabThreads + 2 * int64_t(sm_count) * 32) * nacc * int64_t(sizeof(int64_t));
}

int launch_itab(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                const LaunchCtx &c) {
  const ptsim_itab_params &q = d.p.itab;
  ItabArgs g;
  memset(&g, 0, sizeof(g));
  for (int a = 0; a < d.nargs; ++a) {
    g.arg[a] = ptrs[a];
    g.numel[a] = d.arg_numel[a];
    g.dt[a] = d.arg_dtype[a];
  }
  g.rows = q.rows;
  g.cols = q.cols;
  g.row_begin = lo;
  g.row_end = hi;
  g.ncode = q.ncode;
  g.nout = q.nout;
  int nacc = 0;
  for (int k = 0; k < q.nout; ++k) g.acc_of[k] = q.out[k].mode == PTSIM_ITAB_ELEM ? -1 : nacc++;
  g.nacc = nacc;
  memcpy(g.maps, q.maps, sizeof(g.maps));
  memcpy(g.out, q.out, sizeof(g.out));
  memcpy(g.code, q.code, sizeof(g.code));
  const ItabPlan p = plan_itab(hi - lo, q.cols, c.sm_count);
  g.tx = p.tx;
  g.tr = p.tr;
  g.chunks = nacc > 0 ? p.chunks : 1;
  g.chunk_len = g.chunks > 1 ? p.chunk_len : q.cols;
  if (g.chunks > 1 && p.xblocks * g.chunks > 2 * int64_t(c.sm_count)) g.chunks = 1, g.chunk_len = q.cols;
  if (g.chunks > 1) {
    const int64_t seg_n = int64_t(g.chunks) * g.tr * (hi - lo) * nacc;
    const int64_t chunk_n = int64_t(g.chunks) * (hi - lo) * nacc;
    if (ws == nullptr || int64_t(ws_bytes) < (seg_n + chunk_n) * int64_t(sizeof(int64_t)))
      return fail(PTSIM_E_RESOURCE, "integer table launch needs %lld bytes of workspace, given %zu",
                  (long long)((seg_n + chunk_n) * int64_t(sizeof(int64_t))), ws_bytes);
    g.seg = reinterpret_cast<int64_t *>(ws);
    g.chunk = g.seg + seg_n;
  }
  const dim3 grid(unsigned(p.xblocks), unsigned(g.chunks));
  if (g.chunks > 1) itab_totals_kernel<<<grid, kItabThreads, 0, c.stream>>>(g);
  itab_kernel<<<grid, kItabThreads, 0, c.stream>>>(g);
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

}  // namespace ptsim
