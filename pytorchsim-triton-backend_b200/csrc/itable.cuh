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
constexpr int kItabCtasPerSm = 4;   // split launches: chunks * row blocks <= this * SMs

// A map over f = x * cols + r split into a part of the row x (added once per thread) and digits of the
// column r, evaluated in 32 bits: (f / div) % mod is (x / (div / cols)) % mod when cols divides div, and
// (r / div) % mod when div divides cols and mod divides cols / div (with no mod, x * (cols / div) joins the
// row part).  `general` maps (any other digit, or cols past 2^31) run on f itself.
struct ItabMapX {
  int32_t general, nx, nr, pad0;
  int64_t xdiv[PTSIM_MAX_DIGITS], xmod[PTSIM_MAX_DIGITS], xstride[PTSIM_MAX_DIGITS];  // xmod 0: none
  int32_t rdiv[PTSIM_MAX_DIGITS], rmod[PTSIM_MAX_DIGITS];                              // rmod 0: none
  int64_t rstride[PTSIM_MAX_DIGITS];
};

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
  ItabMapX mx[PTSIM_ITAB_MAPS];
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

// The row parts of the maps for row x (once per thread).
__device__ __forceinline__ void itab_row_bases(const ItabArgs &g, int64_t x, int64_t *xb) {
  for (int m = 0; m < PTSIM_ITAB_MAPS; ++m) {
    const ItabMapX &q = g.mx[m];
    int64_t at = g.maps[m].offset;
    for (int d = 0; d < q.nx; ++d) {
      int64_t v = q.xdiv[d] == 1 ? x : x / q.xdiv[d];
      if (q.xmod[d] != 0) v %= q.xmod[d];
      at += v * q.xstride[d];
    }
    xb[m] = at;
  }
}

// Map m at element (x, r).
__device__ __forceinline__ int64_t itab_at(const ItabArgs &g, int m, const int64_t *xb, int64_t x, int64_t r) {
  const ItabMapX &q = g.mx[m];
  if (q.general) return itab_map(g.maps[m], x * g.cols + r);
  int64_t at = xb[m];
  for (int d = 0; d < q.nr; ++d) {
    uint32_t v = uint32_t(r);
    if (q.rdiv[d] != 1) v /= uint32_t(q.rdiv[d]);
    if (q.rmod[d] != 0) v %= uint32_t(q.rmod[d]);
    at += int64_t(v) * q.rstride[d];
  }
  return at;
}

// Runs the program for element (x, r) into reg[] (registers are written once each, so every output's
// register holds its value when the program ends).
__device__ void itab_eval(const ItabArgs &g, int64_t x, int64_t r, const int64_t *xb, int64_t *reg) {
#pragma unroll 1
  for (int i = 0; i < g.ncode; ++i) {
    const ptsim_iinsn &in = g.code[i];
    const int64_t a = reg[in.a & 31], b = reg[in.b & 31];
    int64_t v = 0;
    switch (in.op) {
      case PTSIM_I_LOAD: v = itab_load(g, in.c, itab_at(g, in.a % PTSIM_ITAB_MAPS, xb, x, r)); break;
      case PTSIM_I_LOADM: v = b ? itab_load(g, in.c, itab_at(g, in.a % PTSIM_ITAB_MAPS, xb, x, r)) : in.imm; break;
      case PTSIM_I_IDX: v = itab_at(g, in.a % PTSIM_ITAB_MAPS, xb, x, r); break;
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
  int64_t xb[PTSIM_ITAB_MAPS];
  if (t.live) {
    itab_row_bases(g, t.x, xb);
    for (int64_t r = t.s0; r < t.s1; ++r) {
      itab_eval(g, t.x, r, xb, reg);
      for (int k = 0; k < g.nout; ++k)
        if (g.acc_of[k] >= 0) acc[g.acc_of[k]] += reg[g.out[k].reg & 31];
    }
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
  int64_t xb[PTSIM_ITAB_MAPS];
  if (t.live) itab_row_bases(g, t.x, xb);
  int64_t base[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};   // total of every element before this segment
  int64_t row_total[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};
  if (split) {
    // The chunk totals of the row, split over the CTA's segment threads (thread tr takes chunks tr,
    // tr + TR, ...), summed in shared memory: the total of the chunks before this one, and the row's.
    __shared__ int64_t sb[kItabThreads * PTSIM_ITAB_OUTS];
    int64_t pb[PTSIM_ITAB_OUTS] = {0, 0, 0, 0}, pt[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};
    if (t.live) {
      for (int64_t c = t.tr; c < int64_t(g.chunks); c += g.tr)
        for (int j = 0; j < g.nacc; ++j) {
          const int64_t v = g.chunk[(c * nrows + t.xi) * g.nacc + j];
          if (c < int64_t(blockIdx.y)) pb[j] += v;
          pt[j] += v;
        }
      for (int q = 0; q < t.tr; ++q)
        for (int j = 0; j < g.nacc; ++j) base[j] += g.seg[((int64_t(blockIdx.y) * g.tr + q) * nrows + t.xi) * g.nacc + j];
    }
    for (int j = 0; j < g.nacc; ++j) {
      sh[threadIdx.x * PTSIM_ITAB_OUTS + j] = pb[j];
      sb[threadIdx.x * PTSIM_ITAB_OUTS + j] = pt[j];
    }
    __syncthreads();
    for (int q = 0; q < g.tr; ++q)
      for (int j = 0; j < g.nacc; ++j) {
        base[j] += sh[(q * g.tx + t.tx) * PTSIM_ITAB_OUTS + j];
        row_total[j] += sb[(q * g.tx + t.tx) * PTSIM_ITAB_OUTS + j];
      }
  } else if (has_scan || has_sum) {
    int64_t acc[PTSIM_ITAB_OUTS] = {0, 0, 0, 0};
    if (t.live && has_scan)
      for (int64_t r = t.s0; r < t.s1; ++r) {
        itab_eval(g, t.x, r, xb, reg);
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
      itab_eval(g, t.x, r, xb, reg);
      for (int k = 0; k < g.nout; ++k) {
        const ptsim_itab_out &o = g.out[k];
        const int64_t v = reg[o.reg & 31];
        if (o.mode == PTSIM_ITAB_ELEM) {
          itab_store(g, o.arg, itab_at(g, o.map % PTSIM_ITAB_MAPS, xb, t.x, r), v);
        } else {
          const int j = g.acc_of[k];
          run[j] += v;
          if (o.mode == PTSIM_ITAB_SCAN) itab_store(g, o.arg, itab_at(g, o.map % PTSIM_ITAB_MAPS, xb, t.x, r), base[j] + run[j]);
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
        itab_store(g, g.out[k].arg, itab_at(g, g.out[k].map % PTSIM_ITAB_MAPS, xb, t.x, 0), row_total[g.acc_of[k]]);
}

// ---------------------------------------------------------------------------------------------------
// Direct kernels for two programs of the combine, chosen by the launcher when the descriptor's program is
// exactly one of them (PTSIM_FLAG_INTERPRET keeps the interpreter); same results, bounds reports included.
//
// One-hot counts (layer_op_combine_*/00_*): v(x, r) = (ids[r] == x), stored as the running total over r
// and / or the row total.  The routed rows are cut into chunks of G * 64: the first kernel counts each
// chunk's ids per expert in shared memory; the second gives each of its G row groups the counts of every
// earlier chunk and earlier group, then walks the group's 64 rows keeping one running count per expert
// thread (a warp writes 32 consecutive experts of a row: the [routed rows, experts] table is
// expert-contiguous).
// ---------------------------------------------------------------------------------------------------
constexpr int kOnehotSub = 64;         // routed rows per group
constexpr int kOnehotMaxRows = 1024;   // experts one CTA covers

struct OnehotArgs {
  const int64_t *ids;
  int64_t ids_numel, ids_off;
  int64_t lo, nx, cols;                // experts [lo, lo + nx), routed rows [0, cols)
  int32_t groups, xpad, chunk_len, has_scan, has_sum, scan_arg, sum_arg, pad0;
  void *scan_out, *sum_out;
  int32_t scan_dt, sum_dt;
  int64_t scan_numel, sum_numel;
  int64_t scan_off, scan_xs, scan_rs, sum_off, sum_xs;
  int64_t *counts;                     // [chunks][nx] per-chunk counts
};

__device__ __forceinline__ void store_int(void *p, int dt, int64_t numel, int64_t at, int64_t v) {
  if (at < 0 || at >= numel) {
    record_status(PTSIM_E_OOB);
    return;
  }
  switch (dt) {
    case PTSIM_DT_I64: reinterpret_cast<int64_t *>(p)[at] = v; break;
    case PTSIM_DT_I32: reinterpret_cast<int32_t *>(p)[at] = int32_t(v); break;
    case PTSIM_DT_I16: reinterpret_cast<int16_t *>(p)[at] = int16_t(v); break;
    case PTSIM_DT_I8: reinterpret_cast<int8_t *>(p)[at] = int8_t(v); break;
    case PTSIM_DT_U8: reinterpret_cast<uint8_t *>(p)[at] = uint8_t(v); break;
  }
}

__device__ __forceinline__ int64_t onehot_id(const OnehotArgs &a, int64_t r) {
  const int64_t at = a.ids_off + r;
  if (at < 0 || at >= a.ids_numel) {
    record_status(PTSIM_E_OOB);
    return 0;
  }
  return __ldg(a.ids + at);
}

// The scan kernel is launched as this one's programmatic dependent: released at the start here, it loads its
// chunk of ids while the histograms are still being counted, and waits (griddepcontrol.wait: this grid has
// finished and its stores are visible) only before it reads the chunk counts.
__global__ void __launch_bounds__(256) onehot_hist_kernel(const __grid_constant__ OnehotArgs a) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ int h[kOnehotMaxRows];
  for (int i = threadIdx.x; i < a.nx; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t r0 = int64_t(blockIdx.x) * a.chunk_len;
  const int64_t r1 = min(a.cols, r0 + a.chunk_len);
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    const int64_t e = onehot_id(a, r) - a.lo;
    if (e >= 0 && e < a.nx) atomicAdd(&h[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.nx; i += blockDim.x) a.counts[int64_t(blockIdx.x) * a.nx + i] = h[i];
}

__global__ void __launch_bounds__(1024) onehot_scan_kernel(const __grid_constant__ OnehotArgs a) {
  __shared__ int64_t s_ids[8 * kOnehotSub];
  __shared__ int64_t s_part[1024], s_tot[1024], s_sub[1024];
  const int xi = int(threadIdx.x) % a.xpad, grp = int(threadIdx.x) / a.xpad;
  const int64_t c = blockIdx.x, chunks = gridDim.x;
  const int64_t r0 = c * a.chunk_len, r1 = min(a.cols, r0 + a.chunk_len);
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) s_ids[r - r0] = onehot_id(a, r);
  asm volatile("griddepcontrol.wait;" ::: "memory");   // the histogram grid's counts (a no-op when launched plainly)
  const bool live = xi < a.nx;
  const int64_t x = a.lo + xi;
  int64_t pb = 0, pt = 0;
  if (live)   // this group's share of the chunk counts, eight loads in flight (integer sums: any order)
    for (int64_t q0 = grp; q0 < chunks; q0 += 8 * int64_t(a.groups)) {
      int64_t v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t q = q0 + int64_t(u) * a.groups;
        v[u] = q < chunks ? __ldcg(a.counts + q * a.nx + xi) : 0;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t q = q0 + int64_t(u) * a.groups;
        if (q < c) pb += v[u];
        pt += v[u];
      }
    }
  __syncthreads();
  const int64_t g0 = r0 + int64_t(grp) * kOnehotSub, g1 = min(r1, g0 + kOnehotSub);
  int64_t cnt = 0;
  if (live)
    for (int64_t r = g0; r < g1; ++r) cnt += s_ids[r - r0] == x;
  s_part[threadIdx.x] = pb;
  s_tot[threadIdx.x] = pt;
  s_sub[threadIdx.x] = cnt;
  __syncthreads();
  if (!live) return;
  int64_t run = 0, total = 0;
  for (int q = 0; q < a.groups; ++q) {
    run += s_part[q * a.xpad + xi] + (q < grp ? s_sub[q * a.xpad + xi] : 0);
    total += s_tot[q * a.xpad + xi];
  }
  if (a.has_scan) {
    int64_t at = a.scan_off + x * a.scan_xs + g0 * a.scan_rs;
    if (a.scan_dt == PTSIM_DT_I64)
      for (int64_t r = g0; r < g1; ++r, at += a.scan_rs) {
        run += s_ids[r - r0] == x;
        if (at < 0 || at >= a.scan_numel) { record_status(PTSIM_E_OOB); continue; }
        __stcs(reinterpret_cast<int64_t *>(a.scan_out) + at, run);
      }
    else
      for (int64_t r = g0; r < g1; ++r, at += a.scan_rs) {
        run += s_ids[r - r0] == x;
        store_int(a.scan_out, a.scan_dt, a.scan_numel, at, run);
      }
  }
  if (a.has_sum && c == 0 && grp == 0) store_int(a.sum_out, a.sum_dt, a.sum_numel, a.sum_off + x * a.sum_xs, total);
}

// Indexed select (layer_op_combine_*/02_*): out[x] = sum over r < cols of tab(x, r) * (ids(x) == r), which is
// tab(x, ids(x)) when 0 <= ids(x) < cols and 0 otherwise.  The launcher has checked that every tab(x, r) the
// program would read lies inside the table, so reading only the selected one reports nothing less.
struct SelectArgs {
  const int64_t *tab;
  const void *ids;
  int32_t ids_dt, out_dt;
  void *out;
  int64_t ids_numel, out_numel, lo, hi, cols;
  int64_t tab_off, tab_xs, tab_rs, ids_off, ids_xs, out_off, out_xs;
};

__global__ void __launch_bounds__(256) select_kernel(const __grid_constant__ SelectArgs a) {
  for (int64_t x = a.lo + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; x < a.hi; x += int64_t(gridDim.x) * blockDim.x) {
    const int64_t ia = a.ids_off + x * a.ids_xs;
    int64_t id = 0;
    if (ia < 0 || ia >= a.ids_numel) record_status(PTSIM_E_OOB);
    else id = a.ids_dt == PTSIM_DT_I64 ? reinterpret_cast<const int64_t *>(a.ids)[ia] : reinterpret_cast<const int32_t *>(a.ids)[ia];
    const int64_t v = (id >= 0 && id < a.cols) ? __ldg(a.tab + a.tab_off + x * a.tab_xs + id * a.tab_rs) : 0;
    store_int(a.out, a.out_dt, a.out_numel, a.out_off + x * a.out_xs, v);
  }
}

// Row groups of a one-hot CTA (about 512 threads: groups x experts rounded up to a warp).
static int onehot_groups(int64_t nx, int &xpad) {
  xpad = int((nx + 31) / 32 * 32);
  int g = 512 / xpad;
  return g < 1 ? 1 : (g > 8 ? 8 : g);
}

// Workspace of the one-hot path: per-chunk counts of every expert row (a launch of fewer rows has as many
// chunks or fewer: more groups per CTA, longer chunks).
static int64_t onehot_workspace(const ptsim_desc &d) {
  int xpad;
  const int g = onehot_groups(d.p.itab.rows, xpad);
  const int64_t chunk = int64_t(g) * kOnehotSub;
  return ((d.p.itab.cols + chunk - 1) / chunk) * d.p.itab.rows * int64_t(sizeof(int64_t));
}

struct ItabPlan {
  int tx, tr, chunks;
  int64_t chunk_len, xblocks;
};

// Rows per CTA up to 32, the rest of the 256 threads on segments; the r range split so about four CTAs
// per SM run, each thread with at least 16 columns, when the rows alone give too few CTAs.
static ItabPlan plan_itab(int64_t nrows, int64_t cols, int sm_count) {
  ItabPlan p;
  p.tx = 1;
  while (p.tx < 32 && p.tx < nrows) p.tx *= 2;
  p.tr = kItabThreads / p.tx;
  p.xblocks = (nrows + p.tx - 1) / p.tx;
  const int64_t want = (kItabCtasPerSm * int64_t(sm_count)) / (p.xblocks > 0 ? p.xblocks : 1);
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

// Workspace for any launch of the descriptor: a split launch has chunks * xblocks <= kItabCtasPerSm *
// sm_count CTAs of 256 segments and 32 rows each.
int64_t itab_workspace(const ptsim_desc &d, int sm_count) {
  const int nacc = itab_naccs(d.p.itab);
  if (nacc == 0) return 0;
  const int64_t ctas = kItabCtasPerSm * int64_t(sm_count);
  const int64_t generic = (ctas * kItabThreads + ctas * 32) * nacc * int64_t(sizeof(int64_t));
  const int64_t onehot = d.p.itab.rows <= kOnehotMaxRows ? onehot_workspace(d) : 0;
  return generic > onehot ? generic : onehot;
}

// The row / column split of map m (ItabMapX) for a [rows, cols] space.
static void split_map(const ptsim_map &m, int64_t cols, ItabMapX &q) {
  memset(&q, 0, sizeof(q));
  if (cols >= (int64_t(1) << 31)) {
    q.general = 1;
    return;
  }
  for (int d = 0; d < m.ndigit; ++d) {
    const int64_t div = m.div[d], mod = m.mod[d], stride = m.stride[d];
    const bool no_mod = mod >= (int64_t(1) << 62);
    if (div % cols == 0) {
      q.xdiv[q.nx] = div / cols;
      q.xmod[q.nx] = no_mod ? 0 : mod;
      q.xstride[q.nx++] = stride;
    } else if (cols % div == 0 && no_mod) {         // x * (cols / div) + r / div
      q.xdiv[q.nx] = 1;
      q.xmod[q.nx] = 0;
      q.xstride[q.nx++] = (cols / div) * stride;
      q.rdiv[q.nr] = int32_t(div);
      q.rmod[q.nr] = 0;
      q.rstride[q.nr++] = stride;
    } else if (cols % div == 0 && (cols / div) % mod == 0) {
      q.rdiv[q.nr] = int32_t(div);
      q.rmod[q.nr] = mod >= cols / div ? 0 : int32_t(mod);   // r / div < cols / div: a mod past it is none
      q.rstride[q.nr++] = stride;
    } else {
      q.general = 1;
      return;
    }
  }
}

// Map m as off + x * xs + r * rs (one plain digit per coordinate at most), or false.
static bool affine_map(const ptsim_map &m, const ItabMapX &q, int64_t &off, int64_t &xs, int64_t &rs) {
  if (q.general || q.nx > 1 || q.nr > 1) return false;
  if (q.nx == 1 && (q.xdiv[0] != 1 || q.xmod[0] != 0)) return false;
  if (q.nr == 1 && (q.rdiv[0] != 1 || q.rmod[0] != 0)) return false;
  off = m.offset;
  xs = q.nx ? q.xstride[0] : 0;
  rs = q.nr ? q.rstride[0] : 0;
  return true;
}

static bool is_int_dt(int dt) {
  return dt == PTSIM_DT_I64 || dt == PTSIM_DT_I32 || dt == PTSIM_DT_I16 || dt == PTSIM_DT_I8 || dt == PTSIM_DT_U8;
}

// The combine's 00 program: LOAD ids at r, IDX x, EQ; outputs its running total and / or row total.
static bool match_onehot(const ptsim_desc &d, const ItabMapX *mx, int64_t nx, OnehotArgs &a) {
  const ptsim_itab_params &q = d.p.itab;
  if (q.ncode != 3 || nx > kOnehotMaxRows) return false;
  const ptsim_iinsn *c = q.code;
  if (c[0].op != PTSIM_I_LOAD || c[1].op != PTSIM_I_IDX || c[2].op != PTSIM_I_EQ || c[0].dst != 0 || c[1].dst != 1 ||
      c[2].dst != 2 || !((c[2].a == 0 && c[2].b == 1) || (c[2].a == 1 && c[2].b == 0)))
    return false;
  int64_t off, xs, rs;
  const int mr = c[0].a % PTSIM_ITAB_MAPS, mi = c[1].a % PTSIM_ITAB_MAPS;
  if (!affine_map(q.maps[mr], mx[mr], off, xs, rs) || xs != 0 || rs != 1 || d.arg_dtype[c[0].c] != PTSIM_DT_I64) return false;
  a.ids_off = off;
  a.ids_numel = d.arg_numel[c[0].c];
  if (!affine_map(q.maps[mi], mx[mi], off, xs, rs) || off != 0 || xs != 1 || rs != 0) return false;
  a.has_scan = a.has_sum = 0;
  for (int k = 0; k < q.nout; ++k) {
    const ptsim_itab_out &o = q.out[k];
    const int m = o.map % PTSIM_ITAB_MAPS;
    if (o.reg != 2 || !is_int_dt(d.arg_dtype[o.arg]) || !affine_map(q.maps[m], mx[m], off, xs, rs)) return false;
    if (o.mode == PTSIM_ITAB_SCAN && !a.has_scan) {
      a.has_scan = 1;
      a.scan_dt = d.arg_dtype[o.arg];
      a.scan_numel = d.arg_numel[o.arg];
      a.scan_off = off, a.scan_xs = xs, a.scan_rs = rs;
      a.scan_arg = o.arg;
    } else if (o.mode == PTSIM_ITAB_SUM && !a.has_sum) {
      a.has_sum = 1;
      a.sum_dt = d.arg_dtype[o.arg];
      a.sum_numel = d.arg_numel[o.arg];
      a.sum_off = off, a.sum_xs = xs;
      a.sum_arg = o.arg;
    } else {
      return false;
    }
  }
  return true;
}

// The combine's 02 program: LOAD tab at (x, r), LOAD ids at x, IDX r, EQ, MUL; one row-total output.
static bool match_select(const ptsim_desc &d, const ItabMapX *mx, int64_t lo, int64_t hi, SelectArgs &a) {
  const ptsim_itab_params &q = d.p.itab;
  if (q.ncode != 5 || q.nout != 1 || q.out[0].mode != PTSIM_ITAB_SUM || q.out[0].reg != 4) return false;
  const ptsim_iinsn *c = q.code;
  for (int i = 0; i < 5; ++i)
    if (c[i].dst != i) return false;
  if (c[0].op != PTSIM_I_LOAD || c[1].op != PTSIM_I_LOAD || c[2].op != PTSIM_I_IDX || c[3].op != PTSIM_I_EQ ||
      c[4].op != PTSIM_I_MUL || !((c[3].a == 1 && c[3].b == 2) || (c[3].a == 2 && c[3].b == 1)) ||
      !((c[4].a == 0 && c[4].b == 3) || (c[4].a == 3 && c[4].b == 0)))
    return false;
  const int mt = c[0].a % PTSIM_ITAB_MAPS, mi = c[1].a % PTSIM_ITAB_MAPS, mr = c[2].a % PTSIM_ITAB_MAPS;
  const int mo = q.out[0].map % PTSIM_ITAB_MAPS;
  int64_t off, xs, rs;
  if (!affine_map(q.maps[mr], mx[mr], off, xs, rs) || off != 0 || xs != 0 || rs != 1) return false;
  if (!affine_map(q.maps[mt], mx[mt], a.tab_off, a.tab_xs, a.tab_rs) || a.tab_xs < 0 || a.tab_rs < 0) return false;
  if (!affine_map(q.maps[mi], mx[mi], a.ids_off, a.ids_xs, rs) || rs != 0) return false;
  if (!affine_map(q.maps[mo], mx[mo], a.out_off, a.out_xs, rs) || rs != 0) return false;
  if (d.arg_dtype[c[0].c] != PTSIM_DT_I64 || (d.arg_dtype[c[1].c] != PTSIM_DT_I64 && d.arg_dtype[c[1].c] != PTSIM_DT_I32) ||
      !is_int_dt(d.arg_dtype[q.out[0].arg]))
    return false;
  // every element the program reads of the table lies inside it (else the interpreter reports it)
  const int64_t first = a.tab_off + lo * a.tab_xs, last = a.tab_off + (hi - 1) * a.tab_xs + (q.cols - 1) * a.tab_rs;
  if (first < 0 || last >= d.arg_numel[c[0].c]) return false;
  a.ids_dt = d.arg_dtype[c[1].c];
  a.ids_numel = d.arg_numel[c[1].c];
  a.out_dt = d.arg_dtype[q.out[0].arg];
  a.out_numel = d.arg_numel[q.out[0].arg];
  a.lo = lo, a.hi = hi, a.cols = q.cols;
  return true;
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
  for (int m = 0; m < PTSIM_ITAB_MAPS; ++m) split_map(q.maps[m], q.cols, g.mx[m]);
  memcpy(g.out, q.out, sizeof(g.out));
  if (!(d.flags & PTSIM_FLAG_INTERPRET)) {
    SelectArgs sa;
    OnehotArgs oa;
    memset(&sa, 0, sizeof(sa));
    memset(&oa, 0, sizeof(oa));
    if (match_select(d, g.mx, lo, hi, sa)) {
      sa.tab = reinterpret_cast<const int64_t *>(ptrs[q.code[0].c]);
      sa.ids = ptrs[q.code[1].c];
      sa.out = ptrs[q.out[0].arg];
      int64_t blocks = (hi - lo + 255) / 256;
      if (blocks > int64_t(c.sm_count) * 8) blocks = int64_t(c.sm_count) * 8;
      select_kernel<<<unsigned(blocks), 256, 0, c.stream>>>(sa);
      PTSIM_CUDA(cudaGetLastError());
      return PTSIM_OK;
    }
    if (match_onehot(d, g.mx, hi - lo, oa)) {
      oa.ids = reinterpret_cast<const int64_t *>(ptrs[q.code[0].c]);
      oa.scan_out = oa.has_scan ? ptrs[oa.scan_arg] : nullptr;
      oa.sum_out = oa.has_sum ? ptrs[oa.sum_arg] : nullptr;
      oa.lo = lo, oa.nx = hi - lo, oa.cols = q.cols;
      oa.groups = onehot_groups(oa.nx, oa.xpad);
      oa.chunk_len = oa.groups * kOnehotSub;
      const int64_t chunks = (q.cols + oa.chunk_len - 1) / oa.chunk_len;
      const int64_t need = chunks * oa.nx * int64_t(sizeof(int64_t));
      if (ws == nullptr || int64_t(ws_bytes) < need)
        return fail(PTSIM_E_RESOURCE, "integer table launch needs %lld bytes of workspace, given %zu", (long long)need, ws_bytes);
      oa.counts = reinterpret_cast<int64_t *>(ws);
      onehot_hist_kernel<<<unsigned(chunks), 256, 0, c.stream>>>(oa);
      PTSIM_CUDA(cudaGetLastError());
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(unsigned(chunks), 1, 1);
      cfg.blockDim = dim3(unsigned(oa.groups * oa.xpad), 1, 1);
      cfg.stream = c.stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      PTSIM_CUDA(cudaLaunchKernelEx(&cfg, onehot_scan_kernel, oa));
      return PTSIM_OK;
    }
  }
  memcpy(g.code, q.code, sizeof(g.code));
  const ItabPlan p = plan_itab(hi - lo, q.cols, c.sm_count);
  g.tx = p.tx;
  g.tr = p.tr;
  g.chunks = nacc > 0 ? p.chunks : 1;
  g.chunk_len = g.chunks > 1 ? p.chunk_len : q.cols;
  if (g.chunks > 1 && p.xblocks * g.chunks > kItabCtasPerSm * int64_t(c.sm_count)) g.chunks = 1, g.chunk_len = q.cols;
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
