// All-reduce of the tensor-parallel layer's row-parallel partial sums over NVLink peer memory (the collective
// after o_proj and after down of the Qwen3-shaped layer split over `nranks` GPUs; one process per GPU).
//
// Every rank's partial [rows, cols] (bf16, its GEMM's output) and output [rows, cols] live in buffers its peers
// have mapped (CUDA IPC).  Rank q owns rows [q R, (q + 1) R), R = rows / nranks: its CTAs read those rows of every
// rank's partial (peer loads over NVLink), add them in rank order 0, 1, ... in fp32 -- a fixed order, so every
// run gives the same bits, unlike a ring whose order depends on the rank -- round once to bf16 and store the
// rows into every rank's output (peer stores).  Data moved per rank: (n - 1) / n of the partial in and
// (n - 1) / n of the output out, the same as a two-shot all-reduce, with no copies through a staging buffer.
//
// Synchronisation, through a 256-byte signal block per rank that every rank has mapped:
//   words [0, 8)   ready[src]: the generation in which rank src's partial became complete;
//   word 8         this rank's generation (calls completed);
//   words [16, 18) done: CTAs (of every rank) that finished storing into this rank's output in this call.
// A call's generation g is this rank's word 8 plus one.  CTA 0 announces the partial is complete (the GEMM before
// this kernel in the stream has finished) by writing g into ready[rank] of every rank; each CTA waits until
// every ready[src] of its own block has reached g before reading any partial.  After storing its rows each CTA
// fences (system scope) and adds one to every rank's done; CTA 0 then waits until its own done reaches
// nranks * gridDim.x (so every row of this rank's output has landed when the kernel ends), sets it back to zero
// and stores g as the rank's generation.  No peer adds to done for call g + 1 before this rank announces g + 1,
// so the reset loses no count, and calls of different shapes (grids) may share one signal block.  No host-side counter: the kernel can be replayed from a CUDA graph.  A rank's partial
// is not overwritten before every peer has read it: the peers' stores into this rank's output, which this
// rank's call waits for, come after their reads.  Every wait is bounded (kWaitUs); a wait that gives up records
// PTSIM_E_TIMEOUT and the CTA skips its rows.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace ptsim {

constexpr int kTpMaxRanks = 8;
constexpr int kTpThreads = 256;
constexpr int kTpSignalBytes = 256;

struct TpArArgs {
  const uint16_t *part[kTpMaxRanks];
  const uint16_t *stage;                             // the second half of a fused all-reduce (below), or null
  uint16_t *out[kTpMaxRanks];
  uint32_t *sig[kTpMaxRanks];
  int32_t nranks, rank;
  int64_t rows, cols;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys64(uint64_t *p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(uint64_t *p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spin until `done()` holds, for at most kWaitUs; false (and PTSIM_E_TIMEOUT recorded) when it gives up.
template <class Done>
__device__ __forceinline__ bool spin_until(Done &&done) {
  if (done()) return true;
  const uint64_t t0 = sm100::globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (done()) return true;
    if ((i & 63u) == 0 && (sm100::globaltimer_ns() - t0 > uint64_t(kWaitUs) * 1000ull || i > kSpinLimit)) {
      record_status(PTSIM_E_TIMEOUT);
      return false;
    }
  }
}

// NR ranks; each thread keeps 16 / NR vectors' loads from every rank in flight (16 peer loads of 16 bytes), since
// a peer load over NVLink takes microseconds: the owned rows are one run of 16-byte vectors, taken K at a time.
//
// STAGED: the second half of the all-reduce whose first half (the reduce-scatter) the row-parallel GEMM did in
// its epilogue, storing each row block into its owner rank's staging buffer (GemmArgs.owners in gemm.cuh).
// This rank's staging holds NR slots of its R owned rows, slot src written by rank src; the kernel sums them
// (local loads) instead of loading every rank's partial over NVLink.  A rank announces ready once its GEMM has
// ended (stream order; the GEMM's threads fenced their peer stores at system scope), so every slot of every
// staging is complete once all ready flags are up.  Rank src's next GEMM overwrites slot src of every staging
// only after its own call of this kernel ended, i.e. after every CTA of every rank had read its staging.
template <int NR, bool STAGED>
__global__ void __launch_bounds__(kTpThreads) tp_allreduce_kernel(const __grid_constant__ TpArArgs a) {
  constexpr int K = 16 / NR;
  __shared__ int ok_all;
  const int tid = threadIdx.x;
  uint32_t *mine = a.sig[a.rank];
  const uint32_t gen = *reinterpret_cast<volatile uint32_t *>(mine + 8) + 1u;
  if (blockIdx.x == 0 && tid < NR) {
    __threadfence_system();
    st_release_sys(a.sig[tid] + a.rank, gen);       // this rank's partial is complete
  }
  if (tid == 0) ok_all = 1;
  __syncthreads();
  if (tid < NR && !spin_until([&] { return int32_t(ld_acquire_sys(mine + tid) - gen) >= 0; })) atomicExch(&ok_all, 0);
  __syncthreads();
  if (ok_all != 0) {
    const int64_t R = a.rows / NR;
    const int64_t v0 = int64_t(a.rank) * R * (a.cols / 8), nv = R * (a.cols / 8);   // the owned vectors
    const int64_t stride = int64_t(gridDim.x) * kTpThreads;
    for (int64_t base = int64_t(blockIdx.x) * kTpThreads + tid; base < nv; base += stride * K) {
      uint4 w[K][NR];
#pragma unroll
      for (int k = 0; k < K; ++k)
#pragma unroll
        for (int src = 0; src < NR; ++src)
          if (base + k * stride < nv)
            w[k][src] = STAGED ? reinterpret_cast<const uint4 *>(a.stage)[src * nv + base + k * stride]
                               : reinterpret_cast<const uint4 *>(a.part[src])[v0 + base + k * stride];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (base + k * stride >= nv) break;
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
        for (int src = 0; src < NR; ++src) {
          const uint32_t ws[4] = {w[k][src].x, w[k][src].y, w[k][src].z, w[k][src].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * e] = __fadd_rn(acc[2 * e], lo_bf16(ws[e]));
            acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], hi_bf16(ws[e]));
          }
        }
        const uint4 o = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                                   pack_bf16x2(acc[6], acc[7]));
#pragma unroll
        for (int dst = 0; dst < NR; ++dst) reinterpret_cast<uint4 *>(a.out[dst])[v0 + base + k * stride] = o;
      }
    }
  }
  __threadfence_system();                            // this thread's stores, before the CTA's count
  __syncthreads();
  if (tid < NR) red_add_release_sys(reinterpret_cast<uint64_t *>(a.sig[tid] + 16), 1ull);
  if (blockIdx.x == 0 && tid == 0) {
    uint64_t *done = reinterpret_cast<uint64_t *>(mine + 16);
    const uint64_t want = uint64_t(NR) * uint64_t(gridDim.x);
    spin_until([&] { return ld_acquire_sys64(done) >= want; });
    st_relaxed_sys64(done, 0ull);
    *reinterpret_cast<volatile uint32_t *>(mine + 8) = gen;
  }
}

// The grid every rank launches (it must be the same on every rank: the done count depends on it): enough
// threads to keep every owned vector's loads in flight at once, at most 2 CTAs per SM of a 148-SM part.
inline int tp_allreduce_grid(int64_t rows, int64_t cols, int nranks) {
  const int64_t vecs = rows / nranks * (cols / 8);
  const int64_t per_cta = int64_t(kTpThreads) * (16 / nranks);
  int64_t g = (vecs + per_cta - 1) / per_cta;
  return int(g < 1 ? 1 : (g > 296 ? 296 : g));
}

// `stage` null: the all-reduce over the partials part[]; else the fused all-reduce's second half over this
// rank's staging (part unused).
inline int launch_tp_allreduce(void *const *part, const void *stage, void *const *out, void *const *sig, int nranks,
                               int rank, int64_t rows, int64_t cols, int dtype, cudaStream_t stream) {
  if ((nranks != 2 && nranks != 4 && nranks != 8) || rank < 0 || rank >= nranks)
    return fail(PTSIM_E_ARGS, "tensor-parallel all-reduce over %d ranks (rank %d); runs 2, 4 or 8", nranks, rank);
  if (dtype != PTSIM_DT_BF16) return fail(PTSIM_E_UNSUPPORTED, "the tensor-parallel all-reduce sums bf16 partials");
  if (rows % nranks != 0 || cols % 8 != 0 || rows < 1)
    return fail(PTSIM_E_UNSUPPORTED, "all-reduce of [%lld, %lld] over %d ranks: rows must divide, cols be a multiple of 8",
                (long long)rows, (long long)cols, nranks);
  TpArArgs a;
  memset(&a, 0, sizeof(a));
  for (int r = 0; r < nranks; ++r) {
    const void *pr = stage != nullptr ? stage : part[r];
    if (pr == nullptr || out[r] == nullptr || sig[r] == nullptr)
      return fail(PTSIM_E_ARGS, "all-reduce: a null pointer for rank %d", r);
    if (reinterpret_cast<uintptr_t>(pr) % 16 || reinterpret_cast<uintptr_t>(out[r]) % 16 ||
        reinterpret_cast<uintptr_t>(sig[r]) % 16)
      return fail(PTSIM_E_ARGS, "all-reduce: rank %d's buffers are not 16-byte aligned", r);
    if (stage == nullptr) a.part[r] = static_cast<const uint16_t *>(part[r]);
    a.out[r] = static_cast<uint16_t *>(out[r]);
    a.sig[r] = static_cast<uint32_t *>(sig[r]);
  }
  a.stage = static_cast<const uint16_t *>(stage);
  a.nranks = nranks;
  a.rank = rank;
  a.rows = rows;
  a.cols = cols;
  const unsigned grid = unsigned(tp_allreduce_grid(rows, cols, nranks));
  if (stage != nullptr) {
    if (nranks == 2) tp_allreduce_kernel<2, true><<<grid, kTpThreads, 0, stream>>>(a);
    else if (nranks == 4) tp_allreduce_kernel<4, true><<<grid, kTpThreads, 0, stream>>>(a);
    else tp_allreduce_kernel<8, true><<<grid, kTpThreads, 0, stream>>>(a);
  } else {
    if (nranks == 2) tp_allreduce_kernel<2, false><<<grid, kTpThreads, 0, stream>>>(a);
    else if (nranks == 4) tp_allreduce_kernel<4, false><<<grid, kTpThreads, 0, stream>>>(a);
    else tp_allreduce_kernel<8, false><<<grid, kTpThreads, 0, stream>>>(a);
  }
  PTSIM_CUDA(cudaGetLastError());
  return PTSIM_OK;
}

}  // namespace ptsim
