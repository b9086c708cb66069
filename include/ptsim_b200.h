/*
 * ptsim_b200.h -- the C ABI of the B200 functional executor for PyTorchSim-Triton-Backend tile programs.
 *
 * The reference executes a compiled kernel object by running Spike + the Coprocessor model over the
 * kernel's ELF, one process per program range:
 *   - argv assembly and process spawn:  pytorchsim_triton_compiler/runtime/spike.py:44-56, :100-120
 *   - the program loop inside the ELF:  pytorchsim_triton_compiler/codegen/wrapper.py:238-266
 *     (pid_x = f % gx, pid_y = (f / gx) % gy, pid_z = f / (gx * gy) for f in [lo, hi))
 *   - trap codes on failure:            pytorchsim_triton_compiler/runtime/spike.py:12 (200, 201)
 * This library replaces both: a launch descriptor (the "binary" the B200 lowering emits in place of the
 * ELF) plus caller-owned device pointers go in, and one sm_100a kernel (or a short fixed sequence of
 * them) runs the programs [lo, hi) of the launch on the caller's stream.
 *
 * Rules of the ABI:
 *   - plain C types only; every pointer is caller-owned; ptsim_launch allocates nothing;
 *   - every call returns 0 on success or a PTSIM_E_* code; ptsim_last_error() gives the message of the
 *     calling thread's last failure;
 *   - device-side failures (a bounds check, a bounded wait that gave up) are recorded in a per-device
 *     status word and returned by ptsim_sync(); a kernel that records one returns early, it never traps.
 */
#ifndef PTSIM_B200_H
#define PTSIM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PTSIM_ABI_VERSION 1
#define PTSIM_DESC_MAGIC 0x42535450u /* "PTSB" little endian */

/* Status codes.  200/201 keep the numbers of the reference's named Spike traps
 * (runtime/spike.py:12 TRAP_HINT = {200: INVALID_SPAD_ACCESS, 201: STACK_OVERFLOW}). */
#define PTSIM_OK 0
#define PTSIM_E_DESC 1          /* malformed or unsupported descriptor */
#define PTSIM_E_ARGS 2          /* pointer count, alignment, range or size mismatch */
#define PTSIM_E_CUDA 3          /* a CUDA runtime/driver call failed */
#define PTSIM_E_UNSUPPORTED 4   /* a shape this executor does not run (refused, never approximated) */
#define PTSIM_E_OOB 200         /* a device-side bounds check caught an access outside a tensor */
#define PTSIM_E_RESOURCE 201    /* shared memory / TMEM / workspace too small for the launch */
#define PTSIM_E_TIMEOUT 202     /* a bounded device-side wait gave up (pipeline stall) */

/* Descriptor kinds: one per tile-program class the lowering recognises. */
#define PTSIM_KIND_ELEMENTWISE 1   /* DMA loads at affine index maps + vector-unit ops + one DMA store */
#define PTSIM_KIND_ROW_SOFTMAX 2   /* row max (NaN-propagating), sum of exp, divide */
#define PTSIM_KIND_ROW_RMSNORM 3   /* row mean of squares, rsqrt(mean + eps), times weight */
#define PTSIM_KIND_QKNORM_ROPE 4   /* per-head RMSNorm over head_dim + rotary embedding + head-major store */
#define PTSIM_KIND_GEMM 5          /* C = A.B (+ residual), bf16 inputs, fp32 accumulate, cast on store */
#define PTSIM_KIND_ATTN_PREFILL 6  /* causal GQA flash attention forward, fp32 online softmax */
#define PTSIM_KIND_REDUCE_ALL 7    /* a whole-tensor sum or max to one fp32 value */
#define PTSIM_KIND_ATTN_DECODE 8   /* one-token GQA attention: per KV head, G query rows over S keys */
#define PTSIM_KIND_ROW_DIVSUM 9    /* each row divided by its sum (the MoE router's top-k weight normalisation) */
#define PTSIM_KIND_TOPK 10         /* per row, the K largest (or smallest) values and their column indices */
#define PTSIM_KIND_SORT 11         /* per row, a stable sort of the keys: sorted values and source indices */
#define PTSIM_KIND_GATHER_ROWS 12  /* out[r, :] = table[t(r), :], t an integer program of an index loaded per row */
#define PTSIM_KIND_GROUPED_GEMM 13 /* per listed group g: C[rows of g] = A[rows of g] . B[g] (the MoE expert matmul) */
#define PTSIM_KIND_GATHER_SUM 14   /* out[r, :] = sum over k of w(r, k) * table[t(r, k), :] (the MoE combine) */
#define PTSIM_KIND_INT_TABLE 15    /* an int64 program over [rows, cols] stored per element, summed or scanned along a row */
#define PTSIM_KIND_ROW_SUM 16      /* out[r] = fp32 sum of row r (the MoE layer's per-token weight sums) */

/* Element types of tensor arguments (kernel.json dtype names, contract/kernel_object.py:43-56). */
#define PTSIM_DT_F32 0
#define PTSIM_DT_BF16 1
#define PTSIM_DT_F16 2
#define PTSIM_DT_I32 3
#define PTSIM_DT_I64 4
#define PTSIM_DT_I16 5
#define PTSIM_DT_I8 6
#define PTSIM_DT_U8 7
#define PTSIM_DT_F64 8

/* Vector-unit opcodes of an ELEMENTWISE program (fp32 registers, IEEE round-to-nearest). */
#define PTSIM_OP_LOAD 1    /* r[dst] = widen(arg[map a][index])                        (DMA MVIN) */
#define PTSIM_OP_CONST 2   /* r[dst] = imm */
#define PTSIM_OP_ADD 3
#define PTSIM_OP_SUB 4
#define PTSIM_OP_MUL 5
#define PTSIM_OP_DIV 6
#define PTSIM_OP_NEG 7
#define PTSIM_OP_EXP 8     /* 2^(x * log2 e), as the EUP computes exp (lower_vector_functions.py:310) */
#define PTSIM_OP_RSQRT 9
#define PTSIM_OP_SQRT 10
#define PTSIM_OP_MAX 11    /* NaN-propagating maximum (PyTorchSimTpuOps.td:70-74) */
#define PTSIM_OP_MIN 12    /* NaN-propagating minimum */
#define PTSIM_OP_RBF16 13  /* round to bf16 (RNE) and widen back: an explicit .to(bfloat16) */
#define PTSIM_OP_ABS 14
#define PTSIM_OP_STORE 15  /* arg[store map][index] = narrow(r[a])                        (DMA MVOUT) */

/* REDUCE_ALL operations. */
#define PTSIM_RED_SUM 0
#define PTSIM_RED_MAX 1

#define PTSIM_MAX_ARGS 16
#define PTSIM_MAX_MAPS 8
#define PTSIM_MAX_DIGITS 4
#define PTSIM_MAX_CODE 32
#define PTSIM_MAX_REGS 8

/* One DMA transfer's index map (the 4-D strided box of pytorchsim.transfer, PyTorchSimOps.td:20-72):
 * element offset in tensor `arg` of flat launch index i = offset + sum_d ((i / div[d]) % mod[d]) * stride[d]. */
typedef struct ptsim_map {
  int32_t arg;
  int32_t ndigit;
  int64_t offset;
  int64_t div[PTSIM_MAX_DIGITS];
  int64_t mod[PTSIM_MAX_DIGITS];
  int64_t stride[PTSIM_MAX_DIGITS];
} ptsim_map;

typedef struct ptsim_insn {
  uint8_t op, dst, a, b;
  float imm;
} ptsim_insn;

typedef struct ptsim_ew_params {
  int64_t numel;          /* flat index space of the store */
  int32_t nmap, ncode;
  int32_t store_map;      /* index into map[] of the store */
  int32_t pure_copy;      /* 1: one load stored unchanged to the same dtype -> byte copy (bit exact) */
  ptsim_map map[PTSIM_MAX_MAPS];
  ptsim_insn code[PTSIM_MAX_CODE];
} ptsim_ew_params;

typedef struct ptsim_row_params {
  int64_t rows, cols;
  int64_t in_row_stride, out_row_stride;
  int32_t in_arg, out_arg, weight_arg;      /* weight_arg -1 when absent */
  int32_t res_arg_p1;     /* ROW_RMSNORM: 1 + the argument of a residual row (same row stride) added to the input in
                             fp32 before the norm, the sum normalised unrounded; 0 when absent */
  float eps;              /* RMSNorm epsilon */
  float inv_cols;         /* unused by the kernels (they divide by cols in fp32, as the program does) */
} ptsim_row_params;

typedef struct ptsim_qkrope_params {
  int64_t tokens, heads, dim;           /* input rows are (token, head) pairs of `dim` values */
  int64_t out_tok_stride, out_head_stride; /* output element offset = t*tok_stride + h*head_stride + d */
  int32_t in_arg, weight_arg, cos_arg, sin_arg, out_arg;
  int32_t no_norm;      /* 1: rotary embedding of the rows as they are (layer_op_rope_*: no RMSNorm, weight_arg unread) */
  float eps, pad1;
} ptsim_qkrope_params;

/* A fused vector program: the M = 1 matmul's vector prologue and output epilogue, a whole-tensor reduction's
 * operand.  Ops as the elementwise program's (PTSIM_OP_*, fp32 registers r0..r7), run for one index i: LOAD dst =
 * widen(argument load[a].arg at load[a].offset + i * load[a].stride) (an element outside the argument
 * records PTSIM_E_OOB and reads 0); the result is the last instruction's register.  An epilogue finds the
 * dot product in r7 when it starts.  ncode 0: no program. */
#define PTSIM_VPROG_LOADS 4
#define PTSIM_VPROG_CODE 16
typedef struct ptsim_vload {
  int32_t arg, pad0;
  int64_t offset, stride;
} ptsim_vload;
typedef struct ptsim_vprog {
  int32_t ncode, nload;
  ptsim_vload load[PTSIM_VPROG_LOADS];
  ptsim_insn code[PTSIM_VPROG_CODE];
} ptsim_vprog;

typedef struct ptsim_gemm_params {
  int64_t M, N, K;
  int64_t lda, ldb, ldc, ldr;  /* row strides in elements: A [M,K] row-major; B [K,N] or [N,K]; C, R [M,N] */
  int32_t a_arg, b_arg, c_arg, r_arg;  /* r_arg: residual added before the store, -1 when absent */
  int32_t b_kmajor;            /* 0: B is [K,N] with N contiguous (the Inductor mm layout); 1: B is [N,K] */
  int32_t pad0;
  ptsim_vprog pro;             /* M = 1, [K,N] B: the vector is this program over k (a_arg unread) */
  ptsim_vprog epi;             /* M = 1: out[n] = this program over n, the dot product in r7 (r_arg -1) */
} ptsim_gemm_params;

/* ATTN_PREFILL: q, o [batch, hq, seq, dim]; k, v [batch, hkv, seq, dim].
 * ATTN_DECODE (batch 1, one unit per KV head): q, o [hkv, hq / hkv, dim]; k, v [hkv, seq, dim];
 * ref_bq = the program's padded row count GP, ref_bkv = its key block BKV. */
typedef struct ptsim_attn_params {
  int64_t batch, hq, hkv, seq, dim;
  int32_t q_arg, k_arg, v_arg, o_arg;
  int32_t causal, pad0;
  float scale, pad1;
  int64_t ref_bq, ref_bkv;     /* the reference program's query/key block sizes (its m_i/l_i restarts) */
} ptsim_attn_params;

/* TOPK and SORT: `rows` rows of `cols` values (row stride `cols`) in `in_arg`.  TOPK writes k values and
 * their int64 column indices per row (row stride k) to `val_arg` / `idx_arg`, choosing among the program's
 * `cols_padded` candidate columns (columns past `cols` hold the spent value); `descending` = the largest.
 * SORT writes every row sorted (ties in source order) with int64 source indices; `descending` sorts high to
 * low; `float_keys` orders fp32 keys by their bits (NaN after +inf, -0 equal to +0, both canonicalised in
 * the sorted values). */
typedef struct ptsim_select_params {
  int64_t rows, cols, k, cols_padded;
  int32_t in_arg, val_arg, idx_arg, descending;
  int32_t float_keys, pad0;
} ptsim_select_params;

/* One instruction of a gather's int64 index program (registers r0..r31):
 *   LOAD  dst = the row's index element            CONST dst = imm
 *   ADD SUB MUL AND OR XOR SHL SHR(arithmetic) dst = a op b
 *   DIV MOD  dst = a / b, a % b truncated toward zero (0 when b == 0)
 *   INV dst = ~a    LT LE GT GE EQ NE  dst = (a op b) ? 1 : 0    WHERE dst = c ? a : b */
#define PTSIM_I_LOAD 1
#define PTSIM_I_CONST 2
#define PTSIM_I_ADD 3
#define PTSIM_I_SUB 4
#define PTSIM_I_MUL 5
#define PTSIM_I_DIV 6
#define PTSIM_I_MOD 7
#define PTSIM_I_INV 8
#define PTSIM_I_LT 9
#define PTSIM_I_LE 10
#define PTSIM_I_GT 11
#define PTSIM_I_GE 12
#define PTSIM_I_EQ 13
#define PTSIM_I_NE 14
#define PTSIM_I_WHERE 15
#define PTSIM_I_AND 16
#define PTSIM_I_OR 17
#define PTSIM_I_XOR 18
#define PTSIM_I_SHR 19
#define PTSIM_I_SHL 20
#define PTSIM_I_LOADI 21   /* dst = argument c's element at position reg[a] (an index read through an index) */
#define PTSIM_I_LOADM 22   /* INT_TABLE: dst = reg[b] ? argument c at maps[a] applied to f : imm (a masked load) */
#define PTSIM_I_IDX 23     /* INT_TABLE: dst = maps[a] applied to f (an index as a value) */
#define PTSIM_MAX_ICODE 32

typedef struct ptsim_iinsn {
  uint8_t op, dst, a, b, c, pad0, pad1, pad2;
  int64_t imm;
} ptsim_iinsn;

/* GATHER_ROWS: out [rows, cols] row-major; row r copies table row t (the result register of the last
 * instruction) of a [table_rows, cols] table, converting the element type where the two differ; the
 * program's LOAD reads idx_arg at idx_map applied to r.  A t outside [0, table_rows) records PTSIM_E_OOB. */
typedef struct ptsim_gather_params {
  int64_t rows, cols, table_rows;
  int32_t out_arg, table_arg, idx_arg, ncode;
  ptsim_map idx_map;
  ptsim_iinsn code[PTSIM_MAX_ICODE];
} ptsim_gather_params;

/* GROUPED_GEMM: A [M, K], B [groups, K, N] (N contiguous; row stride ldb, group stride ldg = K * ldb), C [M, N];
 * int32 tables: group[programs] (the group each program takes; an index past the last group with rows
 * holds 0 rows), start[groups + 1], rows[groups + 1].  C rows no program covers keep their values. */
typedef struct ptsim_ggemm_params {
  int64_t M, N, K, groups, programs, ldb, ldg;
  int32_t a_arg, b_arg, c_arg, group_arg, start_arg, rows_arg;
} ptsim_ggemm_params;

/* GATHER_SUM: out [rows, cols]; term (r, k < terms) adds w(r, k) * table row t(r, k) (fp32, terms in order; a
 * [table_rows, cols] table), the store cast to out's type.  The program runs per term over f = r * terms + k:
 * LOAD dst = maps[a] applied to f (maps[a].arg names the tensor), LOADI dst = argument c at reg[a]; w is
 * w_map applied to f.  A row or index outside its tensor records PTSIM_E_OOB and the term adds nothing. */
#define PTSIM_GSUM_MAPS 4
typedef struct ptsim_gsum_params {
  int64_t rows, cols, terms, table_rows;
  int32_t out_arg, table_arg, w_arg, ncode;
  ptsim_map w_map;
  ptsim_map maps[PTSIM_GSUM_MAPS];
  ptsim_iinsn code[PTSIM_MAX_ICODE];
  /* The MoE layer's fused combine (layer_layer_*: weights renormalised, the residual stream added):
   * wdiv != 0 divides each weight (fp32) by wdiv_arg[wdiv_offset + r * wdiv_stride] of its output row r;
   * nres (0-2) residual tensors res_arg[] are read at the output's own index and added as
   * (res_arg[0] + res_arg[1]) + sum before the store (res_arg[1] may be the output itself). */
  int32_t wdiv, nres;
  int32_t res_arg[2];
  int32_t wdiv_arg, pad0;
  int64_t wdiv_offset, wdiv_stride;
} ptsim_gsum_params;

/* INT_TABLE: an int64 program run for every element f = x * cols + r of a [rows, cols] space (registers
 * r0..r31).  LOAD dst = argument c at maps[a] applied to f, LOADM the same when reg[b] is non-zero and imm
 * otherwise, IDX dst = maps[a] applied to f, LOADI dst = argument c at reg[a]; a position outside its tensor
 * records PTSIM_E_OOB and reads 0.  Output k stores register out[k].reg to argument out[k].arg, cast to its
 * integer type, at maps[out[k].map] applied to
 *   ELEM: f, for every element;
 *   SUM:  x * cols, the row's total over r;
 *   SCAN: f, the inclusive running total over r up to this element.
 * Integer arithmetic wraps at 64 bits.  Partition units are rows. */
#define PTSIM_ITAB_MAPS 5
/* desc->flags bit: run an INT_TABLE program on the element interpreter even where the library has a direct
 * kernel for it (the one-hot count / running count of the combine's 00 program, the indexed select of its
 * 02 program); the results are the same. */
#define PTSIM_FLAG_INTERPRET 1u
/* desc->flags bit, for tests of the timeout path only: the launch's pipelined kernels (tcgen05 GEMM, its
 * split-K cluster and 2-CTA forms, the grouped GEMM, both attention kernels, decode attention and the
 * bulk-copy GEMV) withhold the copies of one pipeline stage in their first CTA (or cluster) and give every
 * bounded wait a 1 ms limit instead of 2 s.  The waits on that stage give up, PTSIM_E_TIMEOUT is recorded
 * and every CTA unwinds (copies in flight land, issued MMAs drain, TMEM is freed, cluster barriers are
 * all met); ptsim_sync() then reports the status and the device stays usable.  The outputs of such a
 * launch are undefined.  Other kinds ignore the bit.  No reference counterpart: it plays the role of a
 * program that ends in one of Spike's named traps (runtime/spike.py:12,36-41). */
#define PTSIM_FLAG_TEST_STALL 2u
#define PTSIM_ITAB_OUTS 4
#define PTSIM_ITAB_ELEM 0
#define PTSIM_ITAB_SUM 1
#define PTSIM_ITAB_SCAN 2
typedef struct ptsim_itab_out {
  int32_t arg, map, reg, mode;
} ptsim_itab_out;
typedef struct ptsim_itab_params {
  int64_t rows, cols;
  int32_t ncode, nout;
  ptsim_map maps[PTSIM_ITAB_MAPS];
  ptsim_itab_out out[PTSIM_ITAB_OUTS];
  ptsim_iinsn code[PTSIM_MAX_ICODE];
} ptsim_itab_params;

typedef struct ptsim_reduce_params {
  int64_t numel;
  int32_t in_arg, out_arg, op, pad0;
  ptsim_vprog pro;             /* the reduced operand as this program over the element index (in_arg unread) */
} ptsim_reduce_params;

typedef struct ptsim_desc {
  uint32_t magic;        /* PTSIM_DESC_MAGIC */
  uint32_t version;      /* PTSIM_ABI_VERSION */
  uint32_t kind;         /* PTSIM_KIND_* */
  uint32_t flags;        /* PTSIM_FLAG_* */
  int32_t nargs, pad0;
  int32_t arg_dtype[PTSIM_MAX_ARGS];
  int64_t arg_numel[PTSIM_MAX_ARGS];
  int64_t grid[3];       /* the reference launch grid the lowering was made for */
  int64_t units;         /* partition units of a launch: [lo, hi) of ptsim_launch index these */
  int64_t unit_size;     /* elements (ELEMENTWISE), rows (row kinds), M rows (GEMM), (b, h) (attention) per unit */
  int64_t workspace_bytes; /* scratch the lowering knows a launch needs (REDUCE_ALL partials); the library's
                              ptsim_workspace_size() gives the full amount for a device (split-K GEMM) */
  union {
    ptsim_ew_params ew;
    ptsim_row_params row;
    ptsim_qkrope_params qk;
    ptsim_gemm_params gemm;
    ptsim_attn_params attn;
    ptsim_reduce_params red;
    ptsim_select_params sel;
    ptsim_gather_params gat;
    ptsim_ggemm_params ggemm;
    ptsim_gsum_params gsum;
    ptsim_itab_params itab;
  } p;
} ptsim_desc;

/* ABI version the library was built with (PTSIM_ABI_VERSION). */
int ptsim_version(void);

/* sizeof(ptsim_desc) as compiled, so a binding can check its own mirror of the struct. */
size_t ptsim_desc_size(void);

/* Select `device`, create its status word, check it is an sm_100 part and look up the device address of
 * the scratch ptsim_launch_reduce_noalloc uses.  Idempotent per device; call it again after a
 * cudaDeviceReset of the device.
 * Replaces the reference's discovery of Spike/pk/model (toolchain.py:19-75, kernel_object.py:289-320). */
int ptsim_init(int device);

/* Validate a descriptor without running it (magic, version, kind, sizes, map ranges).  Host only. */
int ptsim_check(const void *desc, size_t desc_bytes);

/* Number of partition units of the descriptor's launch (the [lo, hi) range ptsim_launch takes). */
int64_t ptsim_units(const void *desc, size_t desc_bytes);

/* Run units [lo, hi) of the launch `desc` over the tensors `dev_ptrs[0..nptr)` (argument order of
 * kernel.json, contract/kernel_object.py:131-133 argv_order) on `stream` (a cudaStream_t; NULL = legacy
 * default).  `workspace` holds desc->workspace_bytes of device scratch, or is NULL when that is 0.
 * Asynchronous: returns once the kernels are enqueued.  Replaces runtime/spike.py:100-120 (launch) and
 * the ELF's program loop codegen/wrapper.py:254-266. */
int ptsim_launch(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr,
                 int64_t lo, int64_t hi, void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of device scratch a launch of `desc` wants on `device` (-1 on a bad descriptor): the REDUCE_ALL
 * pass-1 partials, the ATTN_DECODE per-chunk softmax states, the INT_TABLE segment totals of a split row
 * scan, the M = 1 GEMM's partial columns, else desc->workspace_bytes.  No reference counterpart (Spike needed no device
 * scratch). */
int64_t ptsim_workspace_size(const void *desc, size_t desc_bytes, int device);

/* Run a whole-tensor reduction (desc->kind == PTSIM_KIND_REDUCE_ALL) like ptsim_launch(desc, ..., 0,
 * units, ...), with its scratch -- one fp32 partial per pass-1 CTA -- taken from a 4 KiB array the
 * library holds on every GPU that loads it: nothing is allocated, by the library or anything it calls.
 * For callers that cannot allocate device memory -- a foreign-language binding that only holds the raw
 * pointers it was handed, a host whose memory pool already owns the GPU's memory, or a caller that may
 * not synchronise the device, as cudaMalloc and cudaFree do.  A launch that needs more scratch than the
 * array holds (desc->workspace_bytes above 4096) returns PTSIM_E_RESOURCE; other kinds return
 * PTSIM_E_UNSUPPORTED.  ptsim_init(device) looks the array's device address up (cudaGetSymbolAddress) and
 * caches it; call ptsim_init first, outside any stream capture (without it the first call on a device does
 * the lookup itself, and must then come before any capture).  The cached address dies with the device's
 * context: after a cudaDeviceReset, call ptsim_init again before the next call.  Every call on a device
 * shares the one array: calls that overlap on the GPU (other streams, other threads) race on it, so
 * order them on one stream.  No counterpart in the reference: Spike ran in host memory and needed no
 * device scratch. */
int ptsim_launch_reduce_noalloc(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr, void *stream);

/* Run the whole launch `desc` over tensors in HOST memory, the way a caller holding .raw data runs it end to
 * end: the arguments in `copy_in_mask` (bit a = argument a) are copied from host_ptrs[a] to dev_ptrs[a], the
 * kernels run, and the arguments in `copy_out_mask` are copied back.  Device buffers are the caller's (the
 * library allocates nothing).  A row launch (softmax, RMSNorm) is cut into `chunks` unit ranges (edges
 * units * k / chunks) so that, over three streams (copies in, kernels, copies out), the copy of one range's
 * input rows overlaps the kernel of the range before and the return of that range's output rows; PCIe then
 * carries both directions at once.  Other kinds copy in, run once and copy out.  Host memory should be pinned
 * (page-locked) for the copies to overlap.  Asynchronous like ptsim_launch: synchronise `stream_out` (and
 * check ptsim_sync on `stream_run`) before reading the outputs.  Replaces the reference's .raw round trip
 * around a Spike run (runtime/spike.py:100-120). */
int ptsim_launch_host(const void *desc, size_t desc_bytes, void *const *host_ptrs, void *const *dev_ptrs, int nptr,
                      uint32_t copy_in_mask, uint32_t copy_out_mask, int chunks, void *workspace,
                      size_t workspace_bytes, void *stream_in, void *stream_run, void *stream_out);

/* Peer-visible buffers for the tensor-parallel all-reduce, set up once per process before the launches that use
 * them (these calls allocate and synchronise; the launches do not).  ptsim_peer_alloc makes a zero-filled device
 * buffer on the current device; ptsim_peer_handle writes its 64-byte CUDA IPC handle, which the other ranks'
 * processes pass to ptsim_peer_open to map it (their pointer to this rank's buffer); ptsim_peer_close unmaps a
 * peer's buffer and ptsim_peer_free releases one's own.  No reference counterpart (the reference runs one
 * device). */
int ptsim_peer_alloc(size_t bytes, void **dev_ptr);
int ptsim_peer_free(void *dev_ptr);
int ptsim_peer_handle(void *dev_ptr, void *handle);
int ptsim_peer_open(const void *handle, void **dev_ptr);
int ptsim_peer_close(void *dev_ptr);

/* All-reduce of the tensor-parallel layer's row-parallel partial sums (bf16 [rows, cols]) over NVLink peer
 * memory, on `stream` of the calling rank.  part[r], out[r] and signal[r] are rank r's partial, output and
 * 256-byte signal block (zero-filled before the first call) as this rank addresses them (its own, or the peer
 * mapping).  Rank q sums rows [q R, (q + 1) R), R = rows / nranks, of every partial in rank order (fp32, one
 * bf16 rounding: the same bits on every run) and stores them into every rank's output; the kernel ends once
 * every rank's rows have landed in this rank's output.  Every rank calls it, in the same order, with the same
 * rows and cols.  Waits are bounded (PTSIM_E_TIMEOUT).  Replaces the NCCL all-reduce the tensor-parallel split
 * adds after o_proj and down (no reference counterpart). */
int ptsim_tp_allreduce(void *const *part, void *const *out, void *const *signal, int nranks, int rank, int64_t rows,
                       int64_t cols, int dtype, void *stream);

/* The same all-reduce with its reduce-scatter fused into the row-parallel GEMM, in two calls on `stream`:
 *
 * ptsim_launch_rows_to_owners: ptsim_launch of a GEMM descriptor (bf16 output, M = nowners * owner_rows, N a
 * multiple of 16) whose output rows [q owner_rows, (q + 1) owner_rows) are stored, as they leave the tensor
 * cores, at owner_ptrs[q] (32-byte aligned: rank q's staging slot for this rank, rank q's staging + this rank *
 * owner_rows * N, as this rank maps it; a peer store over NVLink) instead of into the descriptor's output
 * argument, which is not written.
 *
 * ptsim_tp_reduce_gather: `stage` is this rank's staging (nranks slots of rows / nranks rows, slot r filled by
 * rank r's GEMM); it sums the slots in rank order (fp32, one bf16 rounding: the bits ptsim_tp_allreduce gives)
 * and stores the rows into every rank's output out[r]; signal[] as for ptsim_tp_allreduce (one block per
 * collective: this call and ptsim_tp_allreduce must not share one).  Every rank launches both, in the same
 * order.  Replaces the NCCL all-reduce after o_proj and down of the tensor-parallel split (no reference
 * counterpart). */
int ptsim_launch_rows_to_owners(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr, int64_t lo,
                                int64_t hi, void *workspace, size_t workspace_bytes, void *const *owner_ptrs,
                                int nowners, int64_t owner_rows, void *stream);
int ptsim_tp_reduce_gather(const void *stage, void *const *out, void *const *signal, int nranks, int rank, int64_t rows,
                           int64_t cols, int dtype, void *stream);

/* Synchronise `stream` and return (and clear) the device status word of the current device:
 * *device_status receives PTSIM_OK or PTSIM_E_OOB / PTSIM_E_TIMEOUT as a kernel recorded it.
 * Replaces the exit-code check of runtime/spike.py:23-33 (run_process). */
int ptsim_sync(void *stream, int32_t *device_status);

/* Copy the calling thread's last error message into buf (NUL-terminated, truncated to n). */
int ptsim_last_error(char *buf, int n);

#ifdef __cplusplus
}
#endif

#endif /* PTSIM_B200_H */
