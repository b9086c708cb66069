// Fused vector programs (ptsim_vprog): the small fp32 programs a descriptor attaches to a kernel's operand
// or result -- the M = 1 matmul's vector (an RMSNorm x * rsqrt(ss / n + eps) * w, a SiLU gate times its up
// half) and its output (the dot product plus residual rows), a whole-tensor reduction's operand (a square,
// a residual sum squared).  They run per index with the elementwise program's op semantics.
#pragma once
#include "common.cuh"

namespace ptsim {

// The launch's arguments as the programs read them.
struct VArgs {
  const void *ptr[PTSIM_MAX_ARGS];
  int64_t numel[PTSIM_MAX_ARGS];
  int32_t dt[PTSIM_MAX_ARGS];
};

inline void vargs_fill(VArgs &t, const ptsim_desc &d, void *const *ptrs) {
  memset(&t, 0, sizeof(t));
  for (int a = 0; a < d.nargs; ++a) {
    t.ptr[a] = ptrs[a];
    t.numel[a] = d.arg_numel[a];
    t.dt[a] = d.arg_dtype[a];
  }
}

__device__ __forceinline__ float vprog_load(const VArgs &t, const ptsim_vload &l, int64_t i) {
  const int a = l.arg;
  const int64_t at = l.offset + i * l.stride;
  if (a < 0 || a >= PTSIM_MAX_ARGS || at < 0 || at >= t.numel[a]) {
    record_status(PTSIM_E_OOB);
    return 0.f;
  }
  switch (t.dt[a]) {
    case PTSIM_DT_F32: return reinterpret_cast<const float *>(t.ptr[a])[at];
    case PTSIM_DT_BF16: return bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(t.ptr[a])[at]);
    case PTSIM_DT_F16: return __half2float(reinterpret_cast<const __half *>(t.ptr[a])[at]);
  }
  record_status(PTSIM_E_OOB);
  return 0.f;
}

// The program over its loaded values pre[] (load slot l's element for this index; r7 = `in` when it starts).
__device__ __forceinline__ float vprog_run(const ptsim_vprog &p, const float (&pre)[PTSIM_VPROG_LOADS], float in) {
  float r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, in};
  float o = in;
  for (int k = 0; k < p.ncode; ++k) {
    const ptsim_insn &c = p.code[k];
    const float a = r[c.a & 7], b = r[c.b & 7];
    switch (c.op) {
      case PTSIM_OP_LOAD: o = pre[c.a % PTSIM_VPROG_LOADS]; break;
      case PTSIM_OP_CONST: o = c.imm; break;
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
    r[c.dst & 7] = o;
  }
  return o;
}

// The program's value at index i.  Every LOAD runs unconditionally, so all of them are issued before the
// program runs: one memory round trip per evaluation, not one per load.
__device__ __forceinline__ float vprog_eval(const ptsim_vprog &p, const VArgs &t, int64_t i, float in) {
  float pre[PTSIM_VPROG_LOADS];
#pragma unroll
  for (int l = 0; l < PTSIM_VPROG_LOADS; ++l) pre[l] = l < p.nload ? vprog_load(t, p.load[l], i) : 0.f;
  return vprog_run(p, pre, in);
}

// B indices at once: the loads of all of them in flight together, then the B programs.
template <int B>
__device__ __forceinline__ void vprog_eval_batch(const ptsim_vprog &p, const VArgs &t, const int64_t (&idx)[B],
                                                 const bool (&live)[B], float (&out)[B]) {
  float pre[B][PTSIM_VPROG_LOADS];
#pragma unroll
  for (int j = 0; j < B; ++j)
#pragma unroll
    for (int l = 0; l < PTSIM_VPROG_LOADS; ++l) pre[j][l] = (live[j] && l < p.nload) ? vprog_load(t, p.load[l], idx[j]) : 0.f;
#pragma unroll
  for (int j = 0; j < B; ++j) out[j] = live[j] ? vprog_run(p, pre[j], 0.f) : 0.f;
}

}  // namespace ptsim
