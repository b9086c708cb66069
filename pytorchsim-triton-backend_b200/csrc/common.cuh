// Shared device/host helpers of the B200 executor: element conversions with the NPU's rounding rules,
// the per-device status word kernels report failures through, and bounded waits.
#pragma once

#include <atomic>
#include <utility>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/ptsim_b200.h"

namespace ptsim {

// ---------------------------------------------------------------------------------------------------
// Status word.  A kernel that detects an out-of-bounds index or a wait that never completes records a
// PTSIM_E_* code here (first one wins) and returns; the host reads and clears it in ptsim_sync.  This is
// the GPU analogue of the reference's Spike trap exit codes (runtime/spike.py:12).
// ---------------------------------------------------------------------------------------------------
__device__ int g_status = 0;  // one translation unit: defined here

__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_status, 0, code); }

// Iteration cap of every spin-wait on an mbarrier or flag: far above any legitimate wait of these
// kernels (a few microseconds), far below a watchdog.  A wait that reaches it records PTSIM_E_TIMEOUT.
constexpr uint32_t kSpinLimit = 1u << 26;
// Wall-time limit of every such wait (microseconds), and the limit a launch with PTSIM_FLAG_TEST_STALL
// uses instead, so a test that withholds a hand-off sees the timeout and the unwind within milliseconds.
constexpr uint32_t kWaitUs = 2000000u;
constexpr uint32_t kTestWaitUs = 1000u;

// ---------------------------------------------------------------------------------------------------
// bf16 <-> fp32.  Widening is exact (bits << 16).  Narrowing rounds to nearest, ties to even, and keeps
// NaN a quiet NaN: the NPU's misc.pack (PyTorchSimTpuOps.td:46-50) and torch's .to(bfloat16).
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Two packed bf16 (lo in bits 0-15) from two floats, RNE.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ float lo_bf16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// exp as the EUP computes it: 2^(x * log2(e)) (targets/tpu/lower_vector_functions.py:310-329).
__device__ __forceinline__ float npu_exp(float x) { return exp2f(x * 1.4426950408889634f); }

// 2^x on the special-function unit (one MUFU op; denormal results flush to zero, which the downstream
// bf16 rounding of a softmax probability would also produce).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// NaN-propagating max/min (the vmax/vmin rule of PyTorchSimTpuOps.td:64-74; tl.PropagateNan.ALL).
// max.NaN / min.NaN return the canonical NaN when either operand is NaN (one instruction on sm_80+).
__device__ __forceinline__ float nan_max(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float nan_min(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Programmatic dependent launch.  Kernels launched with launch_pdl may be scheduled while the kernel before
// them in the stream is still running: each first waits for that kernel to finish and its memory to be
// visible (griddepcontrol.wait, before any global access, so reads after writes and writes after reads of
// the previous kernel stay ordered), then lets the kernel after it be scheduled (launch_dependents).  What
// overlaps is the next launch's scheduling and start-up with this kernel's tail.  Both instructions are
// no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Element size in bytes of a PTSIM_DT_* type.
__host__ __device__ __forceinline__ int dtype_size(int dt) {
  switch (dt) {
    case PTSIM_DT_F32: case PTSIM_DT_I32: return 4;
    case PTSIM_DT_BF16: case PTSIM_DT_F16: case PTSIM_DT_I16: return 2;
    case PTSIM_DT_I64: case PTSIM_DT_F64: return 8;
    case PTSIM_DT_I8: case PTSIM_DT_U8: return 1;
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------------
// Host-side launch helpers.
// ---------------------------------------------------------------------------------------------------
struct LaunchCtx {
  cudaStream_t stream;
  int device;
  int sm_count;
};

// Sets the thread's last error message (printf-style) and returns `code`.
int fail(int code, const char *fmt, ...);

// Checks a CUDA call's result; on failure records the message and returns PTSIM_E_CUDA.
// Raise a kernel's dynamic shared memory limit once per device (the attribute is per function and
// device; setting it on every launch costs a driver round trip in front of each launch).
template <auto Kern>
inline cudaError_t smem_limit_once(int bytes, int device) {
  static std::atomic<uint64_t> done{0};   // one per kernel function (Kern is a template argument)
  const uint64_t bit = (device >= 0 && device < 64) ? (uint64_t(1) << device) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Launch `kern` on `stream` with programmatic stream serialization (see pdl_enter); the kernel must call
// pdl_enter() before it touches global memory.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

#define PTSIM_CUDA(call)                                                                   \
  do {                                                                                     \
    cudaError_t _e = (call);                                                               \
    if (_e != cudaSuccess)                                                                 \
      return ::ptsim::fail(PTSIM_E_CUDA, "%s failed: %s (%s:%d)", #call,                   \
                           cudaGetErrorString(_e), __FILE__, __LINE__);                    \
  } while (0)

// Per-kind launchers (each validates what only it knows and enqueues its kernels).
int launch_elementwise(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c);
int launch_rowops(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c);
int launch_qkrope(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c);
int launch_reduce(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                  const LaunchCtx &c);
// Where a row-parallel GEMM's output rows go when they are pushed to their owner ranks: `n` blocks of `rows`
// rows, block q's to ptr[q] (GemmArgs.owners in gemm.cuh).
struct GemmOwners {
  int n;
  int64_t rows;
  void *const *ptr;
};
int launch_gemm(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                const LaunchCtx &c, const GemmOwners *own = nullptr);
int64_t gemv_workspace(const ptsim_desc &d, int sm_count);
int reduce_workspace(int sm_count);
int launch_attention(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c);
int launch_decode(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                  const LaunchCtx &c);
int64_t decode_workspace(const ptsim_desc &d, int sm_count);
int launch_topk(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c);
int launch_sort(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                const LaunchCtx &c);
int64_t sort_workspace(const ptsim_desc &d);
int launch_gather_rows(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c);
int launch_grouped_gemm(const ptsim_desc &d, void *const *ptrs, const LaunchCtx &c);
int launch_gather_sum(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, const LaunchCtx &c);
int launch_itab(const ptsim_desc &d, void *const *ptrs, int64_t lo, int64_t hi, void *ws, size_t ws_bytes,
                const LaunchCtx &c);
int64_t itab_workspace(const ptsim_desc &d, int sm_count);

}  // namespace ptsim
