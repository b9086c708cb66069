// ELEMENTWISE tile programs: DMA loads at affine index maps, a short vector-unit program in fp32
// registers, one DMA store.  This is what the NPU runs for every Inductor pointwise kernel of the
// validation bundle (vector_add1_*, the Qwen3 layer's relayout copies 05/07 and SiLU-mul 10, tests/cases
// smoke/add.py): per program, MVIN of each operand box (targets/tpu/lower_dma.py:466-492), RVV/EUP ops
// (passes/utils/math_ops.py:10-16, lower_vector_functions.py), MVOUT of the result (lower_dma.py:17).
//
// B200 mapping: the flat index space [begin, end) of the store is cut into groups of 8 consecutive
// indices, one group per thread per grid-stride step.  An operand whose innermost index digit is
// contiguous is fetched with one 16-byte (bf16) or two 16-byte (fp32) vector loads per group; any
// other map gathers element by element.  The program is decoded once per group (uniform across the
// warp), so the per-element cost is the arithmetic itself.  A pure copy moves raw bits (bit exact).
#pragma once
#include "common.cuh"

namespace ptsim {

// An index map in 32-bit form, for launches whose flat index space and tensors stay below 2^31
// elements: each digit's division by an invariant divisor d is a multiply-high and a shift,
// q = (umulhi(n, m) + n) >> s with s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1 (Granlund and
// Montgomery, "Division by invariant integers using multiplication", PLDI 1994; exact for n < 2^31), and
// a digit that cannot wrap inside the launch skips its modulo.
struct FastMap {
  int32_t ndigit;
  uint32_t offset;
  uint32_t wrap;  // bit d: digit d can reach its modulus inside the launch
  uint32_t div_m[PTSIM_MAX_DIGITS], div_s[PTSIM_MAX_DIGITS];
  uint32_t mod[PTSIM_MAX_DIGITS], mod_m[PTSIM_MAX_DIGITS], mod_s[PTSIM_MAX_DIGITS];
  uint32_t stride[PTSIM_MAX_DIGITS];
};

struct EwLaunch {
  ptsim_ew_params p;
  const void *ptr[PTSIM_MAX_ARGS];
  int64_t numel[PTSIM_MAX_ARGS];
  int32_t dtype[PTSIM_MAX_ARGS];
  int32_t vec[PTSIM_MAX_MAPS];  // 1: the map is contiguous over every aligned group of 8 indices
  int64_t begin, end;
  int32_t idx32;                // 1: every index fits 31 bits; fmap[] holds the maps in 32-bit form
  FastMap fmap[PTSIM_MAX_MAPS];
};

__device__ __forceinline__ uint32_t fast_div(uint32_t n, uint32_t m, uint32_t s) { return (__umulhi(n, m) + n) >> s; }

__device__ __forceinline__ uint32_t fast_index(const FastMap &m, uint32_t i) {
  uint32_t idx = m.offset;
#pragma unroll
  for (int d = 0; d < PTSIM_MAX_DIGITS; ++d)
    if (d < m.ndigit) {
      uint32_t q = fast_div(i, m.div_m[d], m.div_s[d]);
      if ((m.wrap >> d) & 1u) q -= fast_div(q, m.mod_m[d], m.mod_s[d]) * m.mod[d];
      idx += q * m.stride[d];
    }
  return idx;
}

__device__ __forceinline__ int64_t map_index(const ptsim_map &m, int64_t i) {
  int64_t idx = m.offset;
#pragma unroll
  for (int d = 0; d < PTSIM_MAX_DIGITS; ++d)
    if (d < m.ndigit) idx += ((i / m.div[d]) % m.mod[d]) * m.stride[d];
  return idx;
}

// Element index of flat index i through map mi of the launch.
__device__ __forceinline__ int64_t ew_index(const EwLaunch &L, int mi, int64_t i) {
  return L.idx32 ? int64_t(fast_index(L.fmap[mi], uint32_t(i))) : map_index(L.p.map[mi], i);
}

__device__ __forceinline__ float load_elem(const void *p, int dt, int64_t idx) {
  switch (dt) {
    case PTSIM_DT_F32: return __ldg(reinterpret_cast<const float *>(p) + idx);
    case PTSIM_DT_BF16: return bf16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short *>(p) + idx));
    case PTSIM_DT_F16: return __half2float(__ldg(reinterpret_cast<const __half *>(p) + idx));
    case PTSIM_DT_I32: return float(__ldg(reinterpret_cast<const int *>(p) + idx));
    case PTSIM_DT_I64: return float(__ldg(reinterpret_cast<const long long *>(p) + idx));
    case PTSIM_DT_I16: return float(__ldg(reinterpret_cast<const short *>(p) + idx));
    case PTSIM_DT_I8: return float(reinterpret_cast<const signed char *>(p)[idx]);
    case PTSIM_DT_U8: return float(reinterpret_cast<const unsigned char *>(p)[idx]);
    case PTSIM_DT_F64: return float(__ldg(reinterpret_cast<const double *>(p) + idx));
  }
  return 0.f;
}

__device__ __forceinline__ void store_elem(void *p, int dt, int64_t idx, float v) {
  switch (dt) {
    case PTSIM_DT_F32: reinterpret_cast<float *>(p)[idx] = v; break;
    case PTSIM_DT_BF16: reinterpret_cast<unsigned short *>(p)[idx] = f32_to_bf16_bits(v); break;
    case PTSIM_DT_F16: reinterpret_cast<__half *>(p)[idx] = __float2half_rn(v); break;
    case PTSIM_DT_I32: reinterpret_cast<int *>(p)[idx] = int(v); break;
    case PTSIM_DT_I64: reinterpret_cast<long long *>(p)[idx] = (long long)(v); break;
    case PTSIM_DT_I16: reinterpret_cast<short *>(p)[idx] = short(v); break;
    case PTSIM_DT_I8: reinterpret_cast<signed char *>(p)[idx] = (signed char)(v); break;
    case PTSIM_DT_U8: reinterpret_cast<unsigned char *>(p)[idx] = (unsigned char)(v); break;
    case PTSIM_DT_F64: reinterpret_cast<double *>(p)[idx] = double(v); break;
  }
}

// 8 operand values of group i0 (n valid) through map m.
__device__ __forceinline__ void load8(const EwLaunch &L, int mi, int64_t i0, int n, float v[8]) {
  const ptsim_map &m = L.p.map[mi];
  const void *p = L.ptr[m.arg];
  const int dt = L.dtype[m.arg];
  if (n == 8 && L.vec[mi]) {
    const int64_t base = ew_index(L, mi, i0);
    if (base < 0 || base + 8 > L.numel[m.arg]) { record_status(PTSIM_E_OOB); for (int k = 0; k < 8; ++k) v[k] = 0.f; return; }
    if (dt == PTSIM_DT_BF16) {
      uint4 w = __ldg(reinterpret_cast<const uint4 *>(reinterpret_cast<const unsigned short *>(p) + base));
      v[0] = lo_bf16(w.x); v[1] = hi_bf16(w.x); v[2] = lo_bf16(w.y); v[3] = hi_bf16(w.y);
      v[4] = lo_bf16(w.z); v[5] = hi_bf16(w.z); v[6] = lo_bf16(w.w); v[7] = hi_bf16(w.w);
      return;
    }
    if (dt == PTSIM_DT_F32) {
      const float4 *q = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + base);
      float4 a = __ldg(q), b = __ldg(q + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    v[k] = 0.f;
    if (k < n) {
      const int64_t idx = ew_index(L, mi, i0 + k);
      if (idx < 0 || idx >= L.numel[m.arg]) { record_status(PTSIM_E_OOB); continue; }
      v[k] = load_elem(p, dt, idx);
    }
  }
}

__device__ __forceinline__ void store8(const EwLaunch &L, int64_t i0, int n, const float v[8]) {
  const ptsim_map &m = L.p.map[L.p.store_map];
  void *p = const_cast<void *>(L.ptr[m.arg]);
  const int dt = L.dtype[m.arg];
  if (n == 8 && L.vec[L.p.store_map]) {
    const int64_t base = ew_index(L, L.p.store_map, i0);
    if (base < 0 || base + 8 > L.numel[m.arg]) { record_status(PTSIM_E_OOB); return; }
    if (dt == PTSIM_DT_BF16) {
      uint4 w;
      w.x = pack_bf16x2(v[0], v[1]); w.y = pack_bf16x2(v[2], v[3]);
      w.z = pack_bf16x2(v[4], v[5]); w.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4 *>(reinterpret_cast<unsigned short *>(p) + base) = w;
      return;
    }
    if (dt == PTSIM_DT_F32) {
      float4 *q = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p) + base);
      q[0] = make_float4(v[0], v[1], v[2], v[3]);
      q[1] = make_float4(v[4], v[5], v[6], v[7]);
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (k < n) {
      const int64_t idx = ew_index(L, L.p.store_map, i0 + k);
      if (idx < 0 || idx >= L.numel[m.arg]) { record_status(PTSIM_E_OOB); continue; }
      store_elem(p, dt, idx, v[k]);
    }
  }
}

// Register file access with static indices only, so the NREG x 8 register file stays in registers
// (a register index past NREG cannot occur: the host picks NREG above the program's highest register).
template <int NREG>
__device__ __forceinline__ void reg_read(const float (&r)[NREG][8], int i, float v[8]) {
#pragma unroll
  for (int c = 0; c < NREG; ++c)
    if (i == c) {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = r[c][k];
    }
}

template <int NREG>
__device__ __forceinline__ void reg_write(float (&r)[NREG][8], int i, const float v[8]) {
#pragma unroll
  for (int c = 0; c < NREG; ++c)
    if (i == c) {
#pragma unroll
      for (int k = 0; k < 8; ++k) r[c][k] = v[k];
    }
}

template <int NREG>
__global__ void __launch_bounds__(256) ew_program_kernel(const __grid_constant__ EwLaunch L) {
  pdl_enter();
  const int64_t groups = ceil_div(L.end - L.begin, 8);
  float r[NREG][8];
#pragma unroll
  for (int a = 0; a < NREG; ++a)
#pragma unroll
    for (int k = 0; k < 8; ++k) r[a][k] = 0.f;
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i0 = L.begin + g * 8;
    const int n = int((L.end - i0) < 8 ? (L.end - i0) : 8);
    for (int pc = 0; pc < L.p.ncode; ++pc) {
      const ptsim_insn in = L.p.code[pc];
      float x[8], y[8];
      switch (in.op) {
        case PTSIM_OP_LOAD: load8(L, in.a, i0, n, x); reg_write<NREG>(r, in.dst, x); break;
        case PTSIM_OP_CONST:
#pragma unroll
          for (int k = 0; k < 8; ++k) x[k] = in.imm;
          reg_write<NREG>(r, in.dst, x);
          break;
        case PTSIM_OP_STORE: reg_read<NREG>(r, in.a, x); store8(L, i0, n, x); break;
        default: {
          reg_read<NREG>(r, in.a, x);
          reg_read<NREG>(r, in.b, y);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            float a = x[k], b = y[k], o = 0.f;
            switch (in.op) {
              case PTSIM_OP_ADD: o = __fadd_rn(a, b); break;
              case PTSIM_OP_SUB: o = __fsub_rn(a, b); break;
              case PTSIM_OP_MUL: o = __fmul_rn(a, b); break;
              case PTSIM_OP_DIV: o = __fdiv_rn(a, b); break;
              case PTSIM_OP_NEG: o = -a; break;
              case PTSIM_OP_EXP: o = npu_exp(a); break;
              case PTSIM_OP_RSQRT: o = rsqrtf(a); break;
              case PTSIM_OP_SQRT: o = __fsqrt_rn(a); break;
              case PTSIM_OP_MAX: o = nan_max(a, b); break;
              case PTSIM_OP_MIN: o = nan_min(a, b); break;
              case PTSIM_OP_RBF16: o = bf16_bits_to_f32(f32_to_bf16_bits(a)); break;
              case PTSIM_OP_ABS: o = fabsf(a); break;
            }
            x[k] = o;
          }
          reg_write<NREG>(r, in.dst, x);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// The program shapes the validation configurations run, unrolled instead of interpreted (no per-op
// dispatch, no register-file selects).  Each performs the interpreter's operations in the same order,
// so the results are the same bits:
//   EW_BINOP     load a; load b; c = a op b; store c               (vector add, smoke add)
//   EW_SCALAR    load a; const k; c = a op k (or k op a); store c  (vector_add1: x + 1)
//   EW_SILU_MUL  load g; t = exp(-g); s = t + 1; q = g / s; load u; o = q * u; store o  (Qwen3 10)
// The host matches a descriptor's code against these shapes exactly (registers, operands, constant);
// anything else runs on the interpreter.
// ---------------------------------------------------------------------------------------------------
enum { EW_VM = 0, EW_BINOP = 1, EW_SCALAR = 2, EW_SILU_MUL = 3 };

struct EwPattern {
  int32_t kind;
  int32_t op;           // PTSIM_OP_* of the binary operation (BINOP, SCALAR)
  int32_t map_a, map_b; // BINOP: a op b; SCALAR: map_a is the tensor operand; SILU_MUL: gate, up
  int32_t const_first;  // SCALAR: the constant is the left operand
  float imm;
};

template <int OP>
__device__ __forceinline__ float ew_op(float a, float b) {
  if constexpr (OP == PTSIM_OP_ADD) return __fadd_rn(a, b);
  else if constexpr (OP == PTSIM_OP_SUB) return __fsub_rn(a, b);
  else if constexpr (OP == PTSIM_OP_MUL) return __fmul_rn(a, b);
  else if constexpr (OP == PTSIM_OP_DIV) return __fdiv_rn(a, b);
  else if constexpr (OP == PTSIM_OP_MAX) return nan_max(a, b);
  else return nan_min(a, b);
}

template <int OP>
__device__ __forceinline__ void ew_binop8(const float a[8], const float b[8], float o[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = ew_op<OP>(a[k], b[k]);
}

__device__ __forceinline__ void ew_dispatch8(int op, const float a[8], const float b[8], float o[8]) {
  switch (op) {
    case PTSIM_OP_ADD: ew_binop8<PTSIM_OP_ADD>(a, b, o); break;
    case PTSIM_OP_SUB: ew_binop8<PTSIM_OP_SUB>(a, b, o); break;
    case PTSIM_OP_MUL: ew_binop8<PTSIM_OP_MUL>(a, b, o); break;
    case PTSIM_OP_DIV: ew_binop8<PTSIM_OP_DIV>(a, b, o); break;
    case PTSIM_OP_MAX: ew_binop8<PTSIM_OP_MAX>(a, b, o); break;
    default: ew_binop8<PTSIM_OP_MIN>(a, b, o); break;
  }
}

// NG groups of 8 per thread per step, all loads issued before any arithmetic (more bytes in flight per
// SM); group u of a block's step is u * blockDim + threadIdx, so every load instruction of a warp is one
// contiguous run.
template <int KIND, int NG>
__global__ void __launch_bounds__(256) ew_pattern_kernel(const __grid_constant__ EwLaunch L, const EwPattern P) {
  pdl_enter();
  const int64_t groups = ceil_div(L.end - L.begin, 8);
  const int64_t step = int64_t(gridDim.x) * blockDim.x * NG;
  for (int64_t g0 = int64_t(blockIdx.x) * blockDim.x * NG + threadIdx.x; g0 < groups; g0 += step) {
    float a[NG][8], b[NG][8];
#pragma unroll
    for (int u = 0; u < NG; ++u) {
      const int64_t g = g0 + int64_t(u) * blockDim.x;
      if (g < groups) {
        const int64_t i0 = L.begin + g * 8;
        const int n = int((L.end - i0) < 8 ? (L.end - i0) : 8);
        load8(L, P.map_a, i0, n, a[u]);
        if constexpr (KIND != EW_SCALAR) load8(L, P.map_b, i0, n, b[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < NG; ++u) {
      const int64_t g = g0 + int64_t(u) * blockDim.x;
      if (g >= groups) break;
      const int64_t i0 = L.begin + g * 8;
      const int n = int((L.end - i0) < 8 ? (L.end - i0) : 8);
      float o[8];
      if constexpr (KIND == EW_BINOP) {
        ew_dispatch8(P.op, a[u], b[u], o);
      } else if constexpr (KIND == EW_SCALAR) {
#pragma unroll
        for (int k = 0; k < 8; ++k) b[u][k] = P.imm;
        if (P.const_first) ew_dispatch8(P.op, b[u], a[u], o);
        else ew_dispatch8(P.op, a[u], b[u], o);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float t = npu_exp(-a[u][k]);
          const float q = __fdiv_rn(a[u][k], __fadd_rn(t, 1.0f));
          o[k] = __fmul_rn(q, b[u][k]);
        }
      }
      store8(L, i0, n, o);
    }
  }
}

// Vector path of the same shapes: every map of the program contiguous and 16-byte aligned over each group
// of 8, all tensors of one dtype (bf16 or fp32), every index below 2^31.  The kernel gets its own small
// parameter block with the operands' pointers, 32-bit maps and bounds resolved on the host, so it reads
// only fixed parameter offsets.  Groups stay packed in registers until the arithmetic (4 registers per
// bf16 group, 8 per fp32 group); a block of 256 threads takes 256 x NG consecutive groups, all loads
// issued before any arithmetic, and the grid has one block per such run so the scheduler keeps every SM
// full (as the row-per-CTA kernel does).  The ragged last group, if any, is finished element by element.
struct EwVec {
  const void *a, *b;
  void *o;
  FastMap ma, mb, mo;
  uint32_t na, nb, no;     // tensor sizes (elements) for the bounds checks
  uint32_t begin, end;     // flat index range of the launch
  int32_t op, const_first;
  float imm;
};

template <int DT>
struct RawGroup {
  uint4 w[DT == PTSIM_DT_F32 ? 2 : 1];
};

template <int DT>
__device__ __forceinline__ bool raw_load(const void *p, const FastMap &m, uint32_t n, uint32_t i0, RawGroup<DT> &r) {
  const uint32_t base = fast_index(m, i0);
  if (base + 8 > n) {
    record_status(PTSIM_E_OOB);
    return false;
  }
  const uint4 *q = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(p) + size_t(base) * (DT == PTSIM_DT_F32 ? 4 : 2));
  r.w[0] = __ldcs(q);
  if constexpr (DT == PTSIM_DT_F32) r.w[1] = __ldcs(q + 1);
  return true;
}

template <int DT>
__device__ __forceinline__ void raw_unpack(const RawGroup<DT> &r, float v[8]) {
  if constexpr (DT == PTSIM_DT_F32) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      v[4 * h] = __uint_as_float(r.w[h].x);
      v[4 * h + 1] = __uint_as_float(r.w[h].y);
      v[4 * h + 2] = __uint_as_float(r.w[h].z);
      v[4 * h + 3] = __uint_as_float(r.w[h].w);
    }
  } else {
    const uint32_t ws[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = lo_bf16(ws[j]);
      v[2 * j + 1] = hi_bf16(ws[j]);
    }
  }
}

template <int DT>
__device__ __forceinline__ void raw_store(const EwVec &V, uint32_t i0, const float v[8]) {
  const uint32_t base = fast_index(V.mo, i0);
  if (base + 8 > V.no) {
    record_status(PTSIM_E_OOB);
    return;
  }
  uint4 *q = reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(V.o) + size_t(base) * (DT == PTSIM_DT_F32 ? 4 : 2));
  if constexpr (DT == PTSIM_DT_F32) {
    __stcs(q, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3])));
    __stcs(q + 1, make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]), __float_as_uint(v[7])));
  } else {
    __stcs(q, make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7])));
  }
}

template <int KIND>
__device__ __forceinline__ void vpattern_math(const EwVec &V, float x[8], float y[8], float o[8]) {
  if constexpr (KIND == EW_BINOP) {
    ew_dispatch8(V.op, x, y, o);
  } else if constexpr (KIND == EW_SCALAR) {
#pragma unroll
    for (int k = 0; k < 8; ++k) y[k] = V.imm;
    if (V.const_first) ew_dispatch8(V.op, y, x, o);
    else ew_dispatch8(V.op, x, y, o);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float t = npu_exp(-x[k]);
      const float q = __fdiv_rn(x[k], __fadd_rn(t, 1.0f));
      o[k] = __fmul_rn(q, y[k]);
    }
  }
}

template <int KIND, int NG, int DT>
__global__ void __launch_bounds__(256, DT == PTSIM_DT_F32 ? 5 : 8) ew_vpattern_kernel(const __grid_constant__ EwVec V) {
  pdl_enter();
  const uint32_t full = (V.end - V.begin) / 8;   // groups of 8 inside the launch
  const uint32_t g0 = blockIdx.x * blockDim.x * NG + threadIdx.x;
  RawGroup<DT> a[NG], b[NG];
  bool ok[NG];
#pragma unroll
  for (int u = 0; u < NG; ++u) {
    const uint32_t g = g0 + u * blockDim.x;
    ok[u] = g < full;
    if (ok[u]) {
      const uint32_t i0 = V.begin + g * 8;
      ok[u] = raw_load<DT>(V.a, V.ma, V.na, i0, a[u]);
      if constexpr (KIND != EW_SCALAR) ok[u] = raw_load<DT>(V.b, V.mb, V.nb, i0, b[u]) && ok[u];
    }
  }
#pragma unroll
  for (int u = 0; u < NG; ++u) {
    if (!ok[u]) continue;
    float x[8], y[8], o[8];
    raw_unpack<DT>(a[u], x);
    if constexpr (KIND != EW_SCALAR) raw_unpack<DT>(b[u], y);
    vpattern_math<KIND>(V, x, y, o);
    raw_store<DT>(V, V.begin + (g0 + u * blockDim.x) * 8, o);
  }
  // The ragged last group, element by element.
  if (blockIdx.x == 0 && threadIdx.x == 0 && V.begin + full * 8 < V.end) {
    const uint32_t i0 = V.begin + full * 8, n = V.end - i0;
    float x[8], y[8], o[8];
    for (int k = 0; k < 8; ++k) {
      x[k] = y[k] = 0.f;
      if (uint32_t(k) >= n) continue;
      const uint32_t ia = fast_index(V.ma, i0 + k), ib = KIND != EW_SCALAR ? fast_index(V.mb, i0 + k) : 0;
      if (ia >= V.na || (KIND != EW_SCALAR && ib >= V.nb)) { record_status(PTSIM_E_OOB); continue; }
      x[k] = load_elem(V.a, DT, ia);
      if (KIND != EW_SCALAR) y[k] = load_elem(V.b, DT, ib);
    }
    vpattern_math<KIND>(V, x, y, o);
    for (int k = 0; k < 8; ++k) {
      if (uint32_t(k) >= n) continue;
      const uint32_t io = fast_index(V.mo, i0 + k);
      if (io >= V.no) { record_status(PTSIM_E_OOB); continue; }
      store_elem(V.o, DT, io, o[k]);
    }
  }
}

// Which unrolled shape runs descriptor program p (EW_VM: none).
static EwPattern match_pattern(const ptsim_ew_params &p) {
  EwPattern P;
  memset(&P, 0, sizeof(P));
  P.kind = EW_VM;
  const ptsim_insn *c = p.code;
  auto binop = [](int op) {
    return op == PTSIM_OP_ADD || op == PTSIM_OP_SUB || op == PTSIM_OP_MUL || op == PTSIM_OP_DIV ||
           op == PTSIM_OP_MAX || op == PTSIM_OP_MIN;
  };
  auto map_ok = [&](int m) { return m >= 0 && m < p.nmap && m != p.store_map; };
  if (p.ncode == 4 && c[0].op == PTSIM_OP_LOAD && c[3].op == PTSIM_OP_STORE && binop(c[2].op) && c[3].a == c[2].dst &&
      map_ok(c[0].a)) {
    const int ra = c[0].dst;
    if (c[1].op == PTSIM_OP_LOAD && map_ok(c[1].a) && c[1].dst != ra) {
      const int rb = c[1].dst;
      if (c[2].a == ra && c[2].b == rb) { P.kind = EW_BINOP; P.map_a = c[0].a; P.map_b = c[1].a; }
      else if (c[2].a == rb && c[2].b == ra) { P.kind = EW_BINOP; P.map_a = c[1].a; P.map_b = c[0].a; }
      P.op = c[2].op;
    } else if (c[1].op == PTSIM_OP_CONST && c[1].dst != ra) {
      const int rk = c[1].dst;
      if ((c[2].a == ra && c[2].b == rk) || (c[2].a == rk && c[2].b == ra)) {
        P.kind = EW_SCALAR;
        P.map_a = c[0].a;
        P.const_first = c[2].a == rk;
        P.imm = c[1].imm;
        P.op = c[2].op;
      }
    }
  }
  if (p.ncode == 9) {
    const int rg = c[0].dst;
    const bool ok = c[0].op == PTSIM_OP_LOAD && map_ok(c[0].a) &&
                    c[1].op == PTSIM_OP_NEG && c[1].a == rg && c[1].dst != rg &&
                    c[2].op == PTSIM_OP_EXP && c[2].a == c[1].dst && c[2].dst != rg &&
                    c[3].op == PTSIM_OP_CONST && c[3].imm == 1.0f && c[3].dst != rg && c[3].dst != c[2].dst &&
                    c[4].op == PTSIM_OP_ADD && c[4].dst != rg &&
                    ((c[4].a == c[2].dst && c[4].b == c[3].dst) || (c[4].a == c[3].dst && c[4].b == c[2].dst)) &&
                    c[5].op == PTSIM_OP_DIV && c[5].a == rg && c[5].b == c[4].dst &&
                    c[6].op == PTSIM_OP_LOAD && map_ok(c[6].a) && c[6].dst != c[5].dst &&
                    c[7].op == PTSIM_OP_MUL &&
                    ((c[7].a == c[5].dst && c[7].b == c[6].dst) || (c[7].a == c[6].dst && c[7].b == c[5].dst)) &&
                    c[8].op == PTSIM_OP_STORE && c[8].a == c[7].dst;
    if (ok) {
      P.kind = EW_SILU_MUL;
      P.map_a = c[0].a;
      P.map_b = c[6].a;
    }
  }
  return P;
}

// Pure copy: the loaded element's bytes go to the store unchanged (bit exact for every dtype).
template <int ESIZE>
__global__ void __launch_bounds__(256) ew_copy_kernel(const __grid_constant__ EwLaunch L) {
  pdl_enter();
  using T = typename std::conditional<ESIZE == 1, uint8_t,
            typename std::conditional<ESIZE == 2, uint16_t,
            typename std::conditional<ESIZE == 4, uint32_t, uint64_t>::type>::type>::type;
  const ptsim_map &src = L.p.map[0];
  const ptsim_map &dst = L.p.map[L.p.store_map];
  const T *sp = reinterpret_cast<const T *>(L.ptr[src.arg]);
  T *dp = reinterpret_cast<T *>(const_cast<void *>(L.ptr[dst.arg]));
  const int64_t groups = ceil_div(L.end - L.begin, 8);
  const bool vs = L.vec[0] && ESIZE == 2, vd = L.vec[L.p.store_map] && ESIZE == 2;
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i0 = L.begin + g * 8;
    const int n = int((L.end - i0) < 8 ? (L.end - i0) : 8);
    T v[8];
    if (n == 8 && vs) {
      const int64_t b = ew_index(L, 0, i0);
      if (b < 0 || b + 8 > L.numel[src.arg]) { record_status(PTSIM_E_OOB); continue; }
      *reinterpret_cast<uint4 *>(v) = __ldg(reinterpret_cast<const uint4 *>(sp + b));
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[k] = 0;
        if (k < n) {
          const int64_t idx = ew_index(L, 0, i0 + k);
          if (idx < 0 || idx >= L.numel[src.arg]) { record_status(PTSIM_E_OOB); continue; }
          v[k] = sp[idx];
        }
      }
    }
    if (n == 8 && vd) {
      const int64_t b = ew_index(L, L.p.store_map, i0);
      if (b < 0 || b + 8 > L.numel[dst.arg]) { record_status(PTSIM_E_OOB); continue; }
      *reinterpret_cast<uint4 *>(dp + b) = *reinterpret_cast<uint4 *>(v);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k < n) {
          const int64_t idx = ew_index(L, L.p.store_map, i0 + k);
          if (idx < 0 || idx >= L.numel[dst.arg]) { record_status(PTSIM_E_OOB); continue; }
          dp[idx] = v[k];
        }
      }
    }
  }
}

// Whether map m addresses 8 consecutive elements from a 16-byte aligned start for every group of 8
// flat indices that starts at a multiple of 8.
static bool map_vectorizable(const ptsim_map &m, int dt, const void *ptr) {
  if (m.ndigit < 1) return false;
  if (m.div[0] != 1 || m.stride[0] != 1 || m.mod[0] % 8 != 0) return false;
  for (int d = 1; d < m.ndigit; ++d) {
    if (m.div[d] % 8 != 0) return false;                       // higher digits constant over a group
    if ((m.stride[d] * dtype_size(dt)) % 16 != 0) return false; // each group starts 16-byte aligned
  }
  if ((m.offset * dtype_size(dt)) % 16 != 0) return false;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return false;
  return dt == PTSIM_DT_BF16 || dt == PTSIM_DT_F32 || (dt == PTSIM_DT_F16);
}

// Multiply-high reciprocal of divisor d (see FastMap).
static void fast_divisor(uint32_t d, uint32_t *m, uint32_t *s) {
  uint32_t sh = 0;
  while ((uint64_t(1) << sh) < d) ++sh;
  *s = sh;
  *m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << sh) - d)) / d + 1);
}

// Fill L.fmap and set L.idx32 when every flat index, offset, stride and tensor fits 31 bits.
static void build_fast_maps(EwLaunch &L) {
  const int64_t lim = int64_t(1) << 31;
  L.idx32 = 0;
  if (L.end + 8 > lim) return;
  for (int a = 0; a < PTSIM_MAX_ARGS; ++a)
    if (L.numel[a] >= lim) return;
  for (int mi = 0; mi < L.p.nmap; ++mi) {
    const ptsim_map &m = L.p.map[mi];
    FastMap &f = L.fmap[mi];
    memset(&f, 0, sizeof(f));
    if (m.offset < 0 || m.offset >= lim || m.ndigit < 0 || m.ndigit > PTSIM_MAX_DIGITS) return;
    f.ndigit = m.ndigit;
    f.offset = uint32_t(m.offset);
    int64_t reach = m.offset;   // largest index the map produces inside the launch
    for (int d = 0; d < m.ndigit; ++d) {
      if (m.div[d] < 1 || m.div[d] >= lim || m.mod[d] < 1 || m.stride[d] < 0 || m.stride[d] >= lim) return;
      fast_divisor(uint32_t(m.div[d]), &f.div_m[d], &f.div_s[d]);
      // The digit's quotient over the launch is at most (end - 1) / div; no modulo when that stays
      // below the modulus.
      const int64_t top = (L.end - 1) / m.div[d];
      reach += (top < m.mod[d] - 1 ? top : m.mod[d] - 1) * m.stride[d];
      if (reach >= lim) return;
      if (top >= m.mod[d]) {
        if (m.mod[d] >= lim) return;
        f.wrap |= 1u << d;
        f.mod[d] = uint32_t(m.mod[d]);
        fast_divisor(f.mod[d], &f.mod_m[d], &f.mod_s[d]);
      }
      f.stride[d] = uint32_t(m.stride[d]);
    }
  }
  L.idx32 = 1;
}

int launch_elementwise(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c) {
  EwLaunch L;
  memset(&L, 0, sizeof(L));
  L.p = d.p.ew;
  for (int a = 0; a < d.nargs; ++a) {
    L.ptr[a] = ptrs[a];
    L.numel[a] = d.arg_numel[a];
    L.dtype[a] = d.arg_dtype[a];
  }
  L.begin = lo * d.unit_size;
  L.end = hi * d.unit_size < d.p.ew.numel ? hi * d.unit_size : d.p.ew.numel;
  if (L.end <= L.begin) return PTSIM_OK;
  const bool aligned = (L.begin % 8) == 0;
  build_fast_maps(L);
  for (int m = 0; m < L.p.nmap; ++m) {
    const int dt = d.arg_dtype[L.p.map[m].arg];
    L.vec[m] = aligned && map_vectorizable(L.p.map[m], dt, ptrs[L.p.map[m].arg]) ? 1 : 0;
    if (dt == PTSIM_DT_F16 && L.vec[m] && !L.p.pure_copy) L.vec[m] = 0;  // fp16 vector path: copy only
  }
  const int64_t groups = ceil_div(L.end - L.begin, 8);
  const int threads = 256;
  int64_t blocks = ceil_div(groups, threads);
  const int64_t cap = int64_t(c.sm_count) * 8;
  if (blocks > cap) blocks = cap;
  if (L.p.pure_copy) {
    const int es = dtype_size(d.arg_dtype[L.p.map[0].arg]);
    switch (es) {
      case 1: PTSIM_CUDA(launch_pdl(ew_copy_kernel<1>, dim3(unsigned(blocks)), dim3(threads), 0, c.stream, L)); break;
      case 2: PTSIM_CUDA(launch_pdl(ew_copy_kernel<2>, dim3(unsigned(blocks)), dim3(threads), 0, c.stream, L)); break;
      case 4: PTSIM_CUDA(launch_pdl(ew_copy_kernel<4>, dim3(unsigned(blocks)), dim3(threads), 0, c.stream, L)); break;
      case 8: PTSIM_CUDA(launch_pdl(ew_copy_kernel<8>, dim3(unsigned(blocks)), dim3(threads), 0, c.stream, L)); break;
      default: return fail(PTSIM_E_DESC, "elementwise copy of a %d-byte element", es);
    }
  } else if (const EwPattern P = match_pattern(L.p); P.kind != EW_VM) {
    // Vector path when every map of the shape is contiguous and aligned, all tensors share one dtype and
    // every index fits 31 bits.
    const int dt = d.arg_dtype[L.p.map[P.map_a].arg];
    bool vec = L.idx32 && (dt == PTSIM_DT_BF16 || dt == PTSIM_DT_F32) && L.vec[P.map_a] && L.vec[L.p.store_map] &&
               d.arg_dtype[L.p.map[L.p.store_map].arg] == dt;
    if (P.kind != EW_SCALAR) vec = vec && L.vec[P.map_b] && d.arg_dtype[L.p.map[P.map_b].arg] == dt;
    if (vec) {
      EwVec V;
      memset(&V, 0, sizeof(V));
      const int aa = L.p.map[P.map_a].arg, oa = L.p.map[L.p.store_map].arg;
      const int ba = P.kind != EW_SCALAR ? L.p.map[P.map_b].arg : aa;
      V.a = ptrs[aa];
      V.b = ptrs[ba];
      V.o = ptrs[oa];
      V.ma = L.fmap[P.map_a];
      V.mb = P.kind != EW_SCALAR ? L.fmap[P.map_b] : L.fmap[P.map_a];
      V.mo = L.fmap[L.p.store_map];
      V.na = uint32_t(d.arg_numel[aa]);
      V.nb = uint32_t(d.arg_numel[ba]);
      V.no = uint32_t(d.arg_numel[oa]);
      V.begin = uint32_t(L.begin);
      V.end = uint32_t(L.end);
      V.op = P.op;
      V.const_first = P.const_first;
      V.imm = P.imm;
      constexpr int ng = 2;
      const int64_t pb = ceil_div(groups, int64_t(threads) * ng);
      const unsigned gb = unsigned(pb < 1 ? 1 : pb);
      if (dt == PTSIM_DT_BF16) {
        if (P.kind == EW_BINOP) PTSIM_CUDA(launch_pdl(ew_vpattern_kernel<EW_BINOP, ng, PTSIM_DT_BF16>, dim3(gb), dim3(threads), 0, c.stream, V));
        else if (P.kind == EW_SCALAR) PTSIM_CUDA(launch_pdl(ew_vpattern_kernel<EW_SCALAR, ng, PTSIM_DT_BF16>, dim3(gb), dim3(threads), 0, c.stream, V));
        else PTSIM_CUDA(launch_pdl(ew_vpattern_kernel<EW_SILU_MUL, ng, PTSIM_DT_BF16>, dim3(gb), dim3(threads), 0, c.stream, V));
      } else {
        if (P.kind == EW_BINOP) PTSIM_CUDA(launch_pdl(ew_vpattern_kernel<EW_BINOP, ng, PTSIM_DT_F32>, dim3(gb), dim3(threads), 0, c.stream, V));
        else if (P.kind == EW_SCALAR) PTSIM_CUDA(launch_pdl(ew_vpattern_kernel<EW_SCALAR, ng, PTSIM_DT_F32>, dim3(gb), dim3(threads), 0, c.stream, V));
        else PTSIM_CUDA(launch_pdl(ew_vpattern_kernel<EW_SILU_MUL, ng, PTSIM_DT_F32>, dim3(gb), dim3(threads), 0, c.stream, V));
      }
    } else {
      int64_t pb = ceil_div(groups, int64_t(threads) * 2);
      if (pb > cap) pb = cap;
      if (P.kind == EW_BINOP) PTSIM_CUDA(launch_pdl(ew_pattern_kernel<EW_BINOP, 2>, dim3(unsigned(pb)), dim3(threads), 0, c.stream, L, P));
      else if (P.kind == EW_SCALAR) PTSIM_CUDA(launch_pdl(ew_pattern_kernel<EW_SCALAR, 2>, dim3(unsigned(pb)), dim3(threads), 0, c.stream, L, P));
      else PTSIM_CUDA(launch_pdl(ew_pattern_kernel<EW_SILU_MUL, 2>, dim3(unsigned(pb)), dim3(threads), 0, c.stream, L, P));
    }
  } else {
    int top = 0;
    for (int i = 0; i < L.p.ncode; ++i) {
      const ptsim_insn &in = L.p.code[i];
      top = in.dst > top ? in.dst : top;
      if (in.op != PTSIM_OP_LOAD && in.op != PTSIM_OP_CONST) {
        top = in.a > top ? in.a : top;
        top = in.b > top ? in.b : top;
      }
    }
    if (top < 2) PTSIM_CUDA(launch_pdl(ew_program_kernel<2>, dim3(unsigned(blocks)), dim3(threads), 0, c.stream, L));
    else if (top < 4) PTSIM_CUDA(launch_pdl(ew_program_kernel<4>, dim3(unsigned(blocks)), dim3(threads), 0, c.stream, L));
    else PTSIM_CUDA(launch_pdl(ew_program_kernel<8>, dim3(unsigned(blocks)), dim3(threads), 0, c.stream, L));
  }
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

}  // namespace ptsim
