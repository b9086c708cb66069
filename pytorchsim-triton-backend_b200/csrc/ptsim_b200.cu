// The C ABI of libptsim_b200.so (declared in include/ptsim_b200.h): descriptor validation, per-device
// setup, dispatch of a launch's unit range to the kernel of its tile-program class, and the status word.
// Everything is one translation unit so the device status word needs no relocatable device code.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "elementwise.cuh"
#include "rowops.cuh"
#include "gemm.cuh"
#include "attention.cuh"
#include "decode.cuh"
#include "moe.cuh"
#include "itable.cuh"
#include "collective.cuh"

namespace ptsim {



static thread_local char t_err[1024] = {0};

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

struct DeviceInfo {
  bool ready = false;
  int sm_count = 0;
  int major = 0, minor = 0;
};
static std::mutex g_dev_mu;
static DeviceInfo g_dev[64];

static int device_info(int dev, DeviceInfo *out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (dev < 0 || dev >= 64) return fail(PTSIM_E_ARGS, "device %d out of range", dev);
  if (!g_dev[dev].ready) {
    cudaDeviceProp prop;
    PTSIM_CUDA(cudaGetDeviceProperties(&prop, dev));
    g_dev[dev].sm_count = prop.multiProcessorCount;
    g_dev[dev].major = prop.major;
    g_dev[dev].minor = prop.minor;
    g_dev[dev].ready = true;
  }
  *out = g_dev[dev];
  return PTSIM_OK;
}

static bool valid_dtype(int dt) { return dt >= PTSIM_DT_F32 && dt <= PTSIM_DT_F64; }

static int check_arg(const ptsim_desc &d, int a, const char *what) {
  if (a < 0 || a >= d.nargs) return fail(PTSIM_E_DESC, "%s refers to argument %d of %d", what, a, d.nargs);
  return PTSIM_OK;
}

// Largest element offset map m reaches over flat indices [0, numel), for non-negative strides.
static int64_t map_max_index(const ptsim_map &m, int64_t numel) {
  int64_t hi = m.offset;
  for (int d = 0; d < m.ndigit; ++d) {
    int64_t top = (numel - 1) / m.div[d];
    if (top > m.mod[d] - 1) top = m.mod[d] - 1;
    hi += top * m.stride[d];
  }
  return hi;
}

// A fused vector program: opcodes, registers, load slots and their arguments.
static int check_vprog(const ptsim_desc &d, const ptsim_vprog &v, const char *what) {
  if (v.ncode == 0) return PTSIM_OK;
  if (v.ncode < 0 || v.ncode > PTSIM_VPROG_CODE || v.nload < 0 || v.nload > PTSIM_VPROG_LOADS)
    return fail(PTSIM_E_DESC, "%s of %d instructions and %d loads", what, v.ncode, v.nload);
  for (int l = 0; l < v.nload; ++l) {
    int rc = check_arg(d, v.load[l].arg, what);
    if (rc) return rc;
    const int dt = d.arg_dtype[v.load[l].arg];
    if (dt != PTSIM_DT_F32 && dt != PTSIM_DT_BF16 && dt != PTSIM_DT_F16)
      return fail(PTSIM_E_UNSUPPORTED, "%s loads a non-floating argument %d", what, v.load[l].arg);
  }
  for (int i = 0; i < v.ncode; ++i) {
    const ptsim_insn &c = v.code[i];
    if (c.op < PTSIM_OP_LOAD || c.op >= PTSIM_OP_STORE || c.dst >= 8 || c.b >= 8 ||
        (c.op == PTSIM_OP_LOAD ? c.a >= v.nload : c.a >= 8))
      return fail(PTSIM_E_DESC, "%s instruction %d", what, i);
  }
  return PTSIM_OK;
}

static int check_desc(const void *p, size_t bytes) {
  if (p == nullptr || bytes < sizeof(ptsim_desc))
    return fail(PTSIM_E_DESC, "descriptor of %zu bytes; this library reads %zu", bytes, sizeof(ptsim_desc));
  const ptsim_desc &d = *reinterpret_cast<const ptsim_desc *>(p);
  if (d.magic != PTSIM_DESC_MAGIC) return fail(PTSIM_E_DESC, "descriptor magic 0x%08x is not PTSB", d.magic);
  if (d.version != PTSIM_ABI_VERSION)
    return fail(PTSIM_E_DESC, "descriptor ABI version %u, this library runs %d", d.version, PTSIM_ABI_VERSION);
  if (d.nargs < 1 || d.nargs > PTSIM_MAX_ARGS) return fail(PTSIM_E_DESC, "descriptor names %d arguments", d.nargs);
  for (int a = 0; a < d.nargs; ++a) {
    if (!valid_dtype(d.arg_dtype[a])) return fail(PTSIM_E_DESC, "argument %d has dtype code %d", a, d.arg_dtype[a]);
    if (d.arg_numel[a] < 0) return fail(PTSIM_E_DESC, "argument %d has %lld elements", a, (long long)d.arg_numel[a]);
  }
  if (d.units < 0 || d.unit_size < 1) return fail(PTSIM_E_DESC, "descriptor has %lld units of %lld", (long long)d.units, (long long)d.unit_size);
  int rc = PTSIM_OK;
  switch (d.kind) {
    case PTSIM_KIND_ELEMENTWISE: {
      const ptsim_ew_params &e = d.p.ew;
      if (e.nmap < 1 || e.nmap > PTSIM_MAX_MAPS || e.ncode < 1 || e.ncode > PTSIM_MAX_CODE)
        return fail(PTSIM_E_DESC, "elementwise program with %d maps and %d instructions", e.nmap, e.ncode);
      if (e.store_map < 0 || e.store_map >= e.nmap) return fail(PTSIM_E_DESC, "store map %d of %d", e.store_map, e.nmap);
      for (int m = 0; m < e.nmap; ++m) {
        const ptsim_map &mp = e.map[m];
        if ((rc = check_arg(d, mp.arg, "index map"))) return rc;
        if (mp.ndigit < 0 || mp.ndigit > PTSIM_MAX_DIGITS) return fail(PTSIM_E_DESC, "map %d has %d digits", m, mp.ndigit);
        for (int k = 0; k < mp.ndigit; ++k) {
          if (mp.div[k] < 1 || mp.mod[k] < 1) return fail(PTSIM_E_DESC, "map %d digit %d divides by %lld mod %lld", m, k, (long long)mp.div[k], (long long)mp.mod[k]);
          if (mp.stride[k] < 0) return fail(PTSIM_E_UNSUPPORTED, "map %d digit %d has a negative stride", m, k);
        }
        if (mp.offset < 0 || (e.numel > 0 && map_max_index(mp, e.numel) >= d.arg_numel[mp.arg]))
          return fail(PTSIM_E_OOB, "index map %d reaches element %lld of argument %d, which holds %lld", m,
                      (long long)map_max_index(mp, e.numel), mp.arg, (long long)d.arg_numel[mp.arg]);
      }
      for (int i = 0; i < e.ncode; ++i) {
        const ptsim_insn &in = e.code[i];
        if (in.op < PTSIM_OP_LOAD || in.op > PTSIM_OP_STORE) return fail(PTSIM_E_DESC, "instruction %d has opcode %d", i, in.op);
        if (in.dst >= PTSIM_MAX_REGS || in.a >= PTSIM_MAX_REGS || in.b >= PTSIM_MAX_REGS)
          return fail(PTSIM_E_DESC, "instruction %d names a register past %d", i, PTSIM_MAX_REGS);
        if (in.op == PTSIM_OP_LOAD && in.a >= e.nmap) return fail(PTSIM_E_DESC, "instruction %d loads map %d", i, in.a);
      }
      break;
    }
    case PTSIM_KIND_ROW_SOFTMAX:
    case PTSIM_KIND_ROW_DIVSUM:
    case PTSIM_KIND_ROW_SUM:
    case PTSIM_KIND_ROW_RMSNORM: {
      const ptsim_row_params &r = d.p.row;
      if ((rc = check_arg(d, r.in_arg, "row input")) || (rc = check_arg(d, r.out_arg, "row output"))) return rc;
      if (d.kind == PTSIM_KIND_ROW_RMSNORM && r.res_arg_p1 > 0) {
        if ((rc = check_arg(d, r.res_arg_p1 - 1, "RMSNorm residual"))) return rc;
        if (r.rows > 0 && (r.rows - 1) * r.in_row_stride + r.cols > d.arg_numel[r.res_arg_p1 - 1])
          return fail(PTSIM_E_OOB, "RMSNorm residual rows extend past their tensor");
      }
      if (d.kind == PTSIM_KIND_ROW_RMSNORM && (rc = check_arg(d, r.weight_arg, "RMSNorm weight"))) return rc;
      if (r.rows < 0 || r.cols < 1) return fail(PTSIM_E_DESC, "row program over %lld x %lld", (long long)r.rows, (long long)r.cols);
      const int64_t out_row = d.kind == PTSIM_KIND_ROW_SUM ? 1 : r.cols;   // a row sum stores one value per row
      if (r.rows > 0) {
        if ((r.rows - 1) * r.in_row_stride + r.cols > d.arg_numel[r.in_arg] ||
            (r.rows - 1) * r.out_row_stride + out_row > d.arg_numel[r.out_arg])
          return fail(PTSIM_E_OOB, "row program reads or writes past its tensors");
        if (d.kind == PTSIM_KIND_ROW_RMSNORM && r.cols > d.arg_numel[r.weight_arg])
          return fail(PTSIM_E_OOB, "RMSNorm weight holds fewer than %lld values", (long long)r.cols);
      }
      break;
    }
    case PTSIM_KIND_QKNORM_ROPE: {
      const ptsim_qkrope_params &q = d.p.qk;
      if ((rc = check_arg(d, q.in_arg, "qk input")) || (!q.no_norm && (rc = check_arg(d, q.weight_arg, "qk weight"))) ||
          (rc = check_arg(d, q.cos_arg, "cos")) || (rc = check_arg(d, q.sin_arg, "sin")) || (rc = check_arg(d, q.out_arg, "qk output")))
        return rc;
      if (q.tokens * q.heads * q.dim > d.arg_numel[q.in_arg] || q.tokens * q.dim > d.arg_numel[q.cos_arg] ||
          q.tokens * q.dim > d.arg_numel[q.sin_arg] ||
          (q.tokens > 0 && (q.tokens - 1) * q.out_tok_stride + (q.heads - 1) * q.out_head_stride + q.dim > d.arg_numel[q.out_arg]))
        return fail(PTSIM_E_OOB, "QK-norm+RoPE reads or writes past its tensors");
      if (d.arg_dtype[q.cos_arg] != PTSIM_DT_F32 || d.arg_dtype[q.sin_arg] != PTSIM_DT_F32 ||
          d.arg_dtype[q.in_arg] != PTSIM_DT_BF16 || d.arg_dtype[q.out_arg] != PTSIM_DT_BF16 ||
          (!q.no_norm && d.arg_dtype[q.weight_arg] != PTSIM_DT_BF16))
        return fail(PTSIM_E_UNSUPPORTED, "QK-norm+RoPE runs bf16 rows with fp32 cos/sin tables");
      break;
    }
    case PTSIM_KIND_GEMM: {
      const ptsim_gemm_params &g = d.p.gemm;
      if ((rc = check_arg(d, g.a_arg, "A")) || (rc = check_arg(d, g.b_arg, "B")) || (rc = check_arg(d, g.c_arg, "C"))) return rc;
      if (g.r_arg >= 0 && (rc = check_arg(d, g.r_arg, "residual"))) return rc;
      if (g.M < 0 || g.N < 1 || g.K < 1) return fail(PTSIM_E_DESC, "GEMM %lldx%lldx%lld", (long long)g.M, (long long)g.N, (long long)g.K);
      if ((g.pro.ncode != 0 || g.epi.ncode != 0) && g.M != 1)
        return fail(PTSIM_E_DESC, "a fused vector prologue or epilogue on a GEMM of M = %lld", (long long)g.M);
      if ((rc = check_vprog(d, g.pro, "GEMV prologue")) || (rc = check_vprog(d, g.epi, "GEMV epilogue"))) return rc;
      if (g.M > 0) {
        const int64_t b_need = g.b_kmajor ? (g.N - 1) * g.ldb + g.K : (g.K - 1) * g.ldb + g.N;
        const int64_t a_need = g.pro.ncode > 0 ? 0 : (g.M - 1) * g.lda + g.K;
        if (a_need > d.arg_numel[g.a_arg] || b_need > d.arg_numel[g.b_arg] ||
            (g.M - 1) * g.ldc + g.N > d.arg_numel[g.c_arg] || (g.r_arg >= 0 && (g.M - 1) * g.ldr + g.N > d.arg_numel[g.r_arg]))
          return fail(PTSIM_E_OOB, "GEMM operands extend past their tensors");
      }
      break;
    }
    case PTSIM_KIND_ATTN_PREFILL: {
      const ptsim_attn_params &a = d.p.attn;
      if ((rc = check_arg(d, a.q_arg, "q")) || (rc = check_arg(d, a.k_arg, "k")) || (rc = check_arg(d, a.v_arg, "v")) ||
          (rc = check_arg(d, a.o_arg, "o")))
        return rc;
      if (a.hkv < 1 || a.hq % a.hkv != 0) return fail(PTSIM_E_DESC, "attention with %lld query heads over %lld KV heads", (long long)a.hq, (long long)a.hkv);
      if (a.batch * a.hq * a.seq * a.dim > d.arg_numel[a.q_arg] || a.batch * a.hq * a.seq * a.dim > d.arg_numel[a.o_arg] ||
          a.batch * a.hkv * a.seq * a.dim > d.arg_numel[a.k_arg] || a.batch * a.hkv * a.seq * a.dim > d.arg_numel[a.v_arg])
        return fail(PTSIM_E_OOB, "attention tensors are smaller than batch x heads x seq x dim");
      break;
    }
    case PTSIM_KIND_ATTN_DECODE: {
      const ptsim_attn_params &a = d.p.attn;
      if ((rc = check_arg(d, a.q_arg, "q")) || (rc = check_arg(d, a.k_arg, "k")) || (rc = check_arg(d, a.v_arg, "v")) ||
          (rc = check_arg(d, a.o_arg, "o")))
        return rc;
      if (a.hkv < 1 || a.hq < a.hkv || a.hq % a.hkv != 0 || a.seq < 1 || a.dim < 1)
        return fail(PTSIM_E_DESC, "decode attention with %lld query rows over %lld KV heads of %lld keys", (long long)a.hq,
                    (long long)a.hkv, (long long)a.seq);
      if (d.units != a.hkv || d.unit_size != 1) return fail(PTSIM_E_DESC, "decode attention has one unit per KV head");
      if (a.hq * a.dim > d.arg_numel[a.q_arg] || a.hq * a.dim > d.arg_numel[a.o_arg] ||
          a.hkv * a.seq * a.dim > d.arg_numel[a.k_arg] || a.hkv * a.seq * a.dim > d.arg_numel[a.v_arg])
        return fail(PTSIM_E_OOB, "decode attention tensors are smaller than heads x (rows | keys) x dim");
      break;
    }
    case PTSIM_KIND_TOPK:
    case PTSIM_KIND_SORT: {
      const ptsim_select_params &e = d.p.sel;
      if ((rc = check_arg(d, e.in_arg, "keys")) || (rc = check_arg(d, e.val_arg, "values")) ||
          (rc = check_arg(d, e.idx_arg, "indices")))
        return rc;
      const int64_t kept = d.kind == PTSIM_KIND_TOPK ? e.k : e.cols;
      if (e.rows < 0 || e.cols < 0 || kept < 0)
        return fail(PTSIM_E_DESC, "selection over %lld x %lld keeping %lld", (long long)e.rows, (long long)e.cols, (long long)kept);
      if (e.rows * e.cols > d.arg_numel[e.in_arg] || e.rows * kept > d.arg_numel[e.val_arg] ||
          e.rows * kept > d.arg_numel[e.idx_arg])
        return fail(PTSIM_E_OOB, "selection reads or writes past its tensors");
      if (d.units * d.unit_size < e.rows) return fail(PTSIM_E_DESC, "selection units do not cover its rows");
      break;
    }
    case PTSIM_KIND_GATHER_ROWS: {
      const ptsim_gather_params &gp = d.p.gat;
      if ((rc = check_arg(d, gp.out_arg, "gather output")) || (rc = check_arg(d, gp.table_arg, "gather table")) ||
          (rc = check_arg(d, gp.idx_arg, "gather index")))
        return rc;
      if (gp.rows < 0 || gp.cols < 1 || gp.table_rows < 0 || gp.ncode < 1 || gp.ncode > PTSIM_MAX_ICODE)
        return fail(PTSIM_E_DESC, "gather of %lld x %lld with %d instructions", (long long)gp.rows, (long long)gp.cols, gp.ncode);
      if (gp.rows * gp.cols > d.arg_numel[gp.out_arg] || gp.table_rows * gp.cols > d.arg_numel[gp.table_arg])
        return fail(PTSIM_E_OOB, "gather rows extend past their tensors");
      const ptsim_map &m = gp.idx_map;
      if (m.ndigit < 0 || m.ndigit > PTSIM_MAX_DIGITS || m.offset < 0) return fail(PTSIM_E_DESC, "gather index map");
      for (int k = 0; k < m.ndigit; ++k)
        if (m.div[k] < 1 || m.mod[k] < 1 || m.stride[k] < 0) return fail(PTSIM_E_DESC, "gather index map digit %d", k);
      if (gp.rows > 0 && map_max_index(m, gp.rows) >= d.arg_numel[gp.idx_arg])
        return fail(PTSIM_E_OOB, "gather index map reaches past the index tensor");
      for (int i = 0; i < gp.ncode; ++i)
        if (gp.code[i].op < PTSIM_I_LOAD || gp.code[i].op > PTSIM_I_SHL || gp.code[i].dst >= PTSIM_MAX_ICODE ||
            gp.code[i].a >= PTSIM_MAX_ICODE || gp.code[i].b >= PTSIM_MAX_ICODE || gp.code[i].c >= PTSIM_MAX_ICODE)
          return fail(PTSIM_E_DESC, "gather instruction %d", i);
      break;
    }
    case PTSIM_KIND_GROUPED_GEMM: {
      const ptsim_ggemm_params &q = d.p.ggemm;
      if ((rc = check_arg(d, q.a_arg, "A")) || (rc = check_arg(d, q.b_arg, "B")) || (rc = check_arg(d, q.c_arg, "C")) ||
          (rc = check_arg(d, q.group_arg, "group ids")) || (rc = check_arg(d, q.start_arg, "group starts")) ||
          (rc = check_arg(d, q.rows_arg, "group rows")))
        return rc;
      if (q.M < 0 || q.N < 1 || q.K < 1 || q.groups < 1 || q.programs < 0 || q.ldb < q.N || q.ldg < q.K * q.ldb)
        return fail(PTSIM_E_DESC, "grouped GEMM %lld x %lld x %lld over %lld groups", (long long)q.M, (long long)q.N,
                    (long long)q.K, (long long)q.groups);
      if (q.M * q.K > d.arg_numel[q.a_arg] || q.M * q.N > d.arg_numel[q.c_arg] ||
          (q.groups - 1) * q.ldg + (q.K - 1) * q.ldb + q.N > d.arg_numel[q.b_arg] || q.programs > d.arg_numel[q.group_arg] ||
          q.groups + 1 > d.arg_numel[q.start_arg] || q.groups + 1 > d.arg_numel[q.rows_arg])
        return fail(PTSIM_E_OOB, "grouped GEMM operands extend past their tensors");
      break;
    }
    case PTSIM_KIND_GATHER_SUM: {
      const ptsim_gsum_params &q = d.p.gsum;
      if ((rc = check_arg(d, q.out_arg, "gather-sum output")) || (rc = check_arg(d, q.table_arg, "gather-sum table")) ||
          (rc = check_arg(d, q.w_arg, "gather-sum weights")) || (rc = check_arg(d, q.w_map.arg, "gather-sum weight map")))
        return rc;
      if (q.rows < 0 || q.cols < 1 || q.terms < 1 || q.table_rows < 0 || q.ncode < 1 || q.ncode > PTSIM_MAX_ICODE)
        return fail(PTSIM_E_DESC, "gather-sum of %lld x %lld over %lld terms", (long long)q.rows, (long long)q.cols, (long long)q.terms);
      if (q.rows * q.cols > d.arg_numel[q.out_arg] || q.table_rows * q.cols > d.arg_numel[q.table_arg])
        return fail(PTSIM_E_OOB, "gather-sum rows extend past their tensors");
      const ptsim_map *ms[PTSIM_GSUM_MAPS + 1] = {&q.w_map, &q.maps[0], &q.maps[1], &q.maps[2], &q.maps[3]};
      for (const ptsim_map *m : ms) {
        if (m->ndigit < 0 || m->ndigit > PTSIM_MAX_DIGITS || m->offset < 0) return fail(PTSIM_E_DESC, "gather-sum map");
        for (int k = 0; k < m->ndigit; ++k)
          if (m->div[k] < 1 || m->mod[k] < 1 || m->stride[k] < 0) return fail(PTSIM_E_DESC, "gather-sum map digit %d", k);
      }
      if (q.nres < 0 || q.nres > 2) return fail(PTSIM_E_DESC, "gather-sum with %d residuals", q.nres);
      for (int k = 0; k < q.nres; ++k)
        if ((rc = check_arg(d, q.res_arg[k], "gather-sum residual"))) return rc;
      if (q.wdiv && (rc = check_arg(d, q.wdiv_arg, "gather-sum weight divisor"))) return rc;
      for (int i = 0; i < q.ncode; ++i)
        if (q.code[i].op < PTSIM_I_LOAD || q.code[i].op > PTSIM_I_LOADI || q.code[i].dst >= PTSIM_MAX_ICODE ||
            q.code[i].a >= PTSIM_MAX_ICODE || q.code[i].b >= PTSIM_MAX_ICODE || q.code[i].c >= PTSIM_MAX_ICODE)
          return fail(PTSIM_E_DESC, "gather-sum instruction %d", i);
      break;
    }
    case PTSIM_KIND_INT_TABLE: {
      const ptsim_itab_params &q = d.p.itab;
      if (q.rows < 0 || q.cols < 1 || q.ncode < 1 || q.ncode > PTSIM_MAX_ICODE || q.nout < 1 || q.nout > PTSIM_ITAB_OUTS)
        return fail(PTSIM_E_DESC, "integer table of %lld x %lld with %d instructions and %d outputs", (long long)q.rows,
                    (long long)q.cols, q.ncode, q.nout);
      if (q.rows > 0 && q.cols > (int64_t(1) << 62) / q.rows) return fail(PTSIM_E_DESC, "integer table too large");
      for (int m = 0; m < PTSIM_ITAB_MAPS; ++m) {
        const ptsim_map &mp = q.maps[m];
        if (mp.ndigit < 0 || mp.ndigit > PTSIM_MAX_DIGITS) return fail(PTSIM_E_DESC, "integer table map %d", m);
        for (int k = 0; k < mp.ndigit; ++k)
          if (mp.div[k] < 1 || mp.mod[k] < 1) return fail(PTSIM_E_DESC, "integer table map %d digit %d", m, k);
      }
      for (int k = 0; k < q.nout; ++k) {
        const ptsim_itab_out &o = q.out[k];
        if ((rc = check_arg(d, o.arg, "integer table output"))) return rc;
        if (o.map < 0 || o.map >= PTSIM_ITAB_MAPS || o.reg < 0 || o.reg >= PTSIM_MAX_ICODE || o.mode < PTSIM_ITAB_ELEM ||
            o.mode > PTSIM_ITAB_SCAN)
          return fail(PTSIM_E_DESC, "integer table output %d", k);
        const int dt = d.arg_dtype[o.arg];
        if (dt != PTSIM_DT_I64 && dt != PTSIM_DT_I32 && dt != PTSIM_DT_I16 && dt != PTSIM_DT_I8 && dt != PTSIM_DT_U8)
          return fail(PTSIM_E_UNSUPPORTED, "integer table output %d is not an integer tensor", k);
      }
      for (int i = 0; i < q.ncode; ++i) {
        const ptsim_iinsn &in = q.code[i];
        const bool known = (in.op >= PTSIM_I_LOAD && in.op <= PTSIM_I_LOADI) || in.op == PTSIM_I_LOADM || in.op == PTSIM_I_IDX;
        if (!known || in.dst >= PTSIM_MAX_ICODE || in.a >= PTSIM_MAX_ICODE || in.b >= PTSIM_MAX_ICODE || in.c >= PTSIM_MAX_ICODE)
          return fail(PTSIM_E_DESC, "integer table instruction %d", i);
        if ((in.op == PTSIM_I_LOAD || in.op == PTSIM_I_LOADM || in.op == PTSIM_I_IDX) && in.a >= PTSIM_ITAB_MAPS)
          return fail(PTSIM_E_DESC, "integer table instruction %d reads map %d", i, in.a);
        if ((in.op == PTSIM_I_LOAD || in.op == PTSIM_I_LOADM || in.op == PTSIM_I_LOADI) && (rc = check_arg(d, in.c, "integer table load")))
          return rc;
      }
      break;
    }
    case PTSIM_KIND_REDUCE_ALL: {
      const ptsim_reduce_params &r = d.p.red;
      if ((rc = check_arg(d, r.in_arg, "reduce input")) || (rc = check_arg(d, r.out_arg, "reduce output"))) return rc;
      if ((rc = check_vprog(d, r.pro, "reduction operand"))) return rc;
      if ((r.pro.ncode == 0 && r.numel > d.arg_numel[r.in_arg]) || d.arg_numel[r.out_arg] < 1)
        return fail(PTSIM_E_OOB, "reduction past its tensors");
      break;
    }
    default:
      return fail(PTSIM_E_DESC, "descriptor kind %u is not one this library runs", d.kind);
  }
  return PTSIM_OK;
}

}  // namespace ptsim

// ---------------------------------------------------------------------------------------------------
// Whole-tensor reduction with library-owned scratch, for callers that cannot allocate device memory: a
// foreign-language binding (ctypes, cgo, JNI) that only holds the raw pointers it was handed, a host
// whose memory pool already owns the GPU's memory, or a caller that may not synchronise the device, as
// cudaMalloc and cudaFree do.  The two-pass reduction parks one fp32 partial per pass-1 CTA in scratch;
// here that scratch is the file-scope array below, which every GPU that loads this library holds until
// the process exits.
// ---------------------------------------------------------------------------------------------------
namespace ptsim {

// 4 KiB: pass 1 never runs more than 1024 CTAs (4 per SM, capped), one fp32 partial each.
constexpr size_t kStaticScratchBytes = 1024 * sizeof(float);
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

static std::mutex g_static_mu;
static void *g_static_ptr[64];

// Device address of g_static_scratch on `dev` (the current device), looked up once per device and again
// whenever `refresh` is set (ptsim_init does, so a call after a cudaDeviceReset finds the new address).  In
// host code the array's name is only a host-side stand-in, so kernels get this address instead.
static int static_scratch(int dev, void **out, bool refresh = false) {
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (dev < 0 || dev >= 64) return fail(PTSIM_E_ARGS, "device %d out of range", dev);
  if (refresh) g_static_ptr[dev] = nullptr;
  if (g_static_ptr[dev] == nullptr) {
    void *p = nullptr;
    PTSIM_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
    if (p == nullptr) return fail(PTSIM_E_CUDA, "no device address for the static scratch on device %d", dev);
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return PTSIM_OK;
}

// One launch of a checked descriptor over device pointers (ptsim_launch); `own` redirects a GEMM's output
// rows to their owner ranks (ptsim_launch_rows_to_owners), null otherwise.
static int launch_desc(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr, int64_t lo, int64_t hi,
                       void *workspace, size_t workspace_bytes, void *stream, const GemmOwners *own);

}  // namespace ptsim

using namespace ptsim;

extern "C" {

int ptsim_version(void) { return PTSIM_ABI_VERSION; }

size_t ptsim_desc_size(void) { return sizeof(ptsim_desc); }

int ptsim_init(int device) {
  int n = 0;
  PTSIM_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(PTSIM_E_ARGS, "device %d of %d", device, n);
  PTSIM_CUDA(cudaSetDevice(device));
  DeviceInfo info;
  int rc = device_info(device, &info);
  if (rc) return rc;
  if (info.major != 10)
    return fail(PTSIM_E_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, info.major, info.minor);
  int zero = 0;
  PTSIM_CUDA(cudaMemcpyToSymbol(g_status, &zero, sizeof(int)));
  // The no-allocation reduction's scratch address, looked up here (outside any stream capture) and again on
  // every call, so re-initialising a device after a reset refreshes it.
  void *scratch = nullptr;
  return static_scratch(device, &scratch, true);
}

int ptsim_check(const void *desc, size_t desc_bytes) { return check_desc(desc, desc_bytes); }

int64_t ptsim_units(const void *desc, size_t desc_bytes) {
  if (check_desc(desc, desc_bytes)) return -1;
  return reinterpret_cast<const ptsim_desc *>(desc)->units;
}

int ptsim_launch(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr, int64_t lo, int64_t hi,
                 void *workspace, size_t workspace_bytes, void *stream) {
  return launch_desc(desc, desc_bytes, dev_ptrs, nptr, lo, hi, workspace, workspace_bytes, stream, nullptr);
}

int ptsim_launch_rows_to_owners(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr, int64_t lo,
                                int64_t hi, void *workspace, size_t workspace_bytes, void *const *owner_ptrs,
                                int nowners, int64_t owner_rows, void *stream) {
  int rc = check_desc(desc, desc_bytes);
  if (rc) return rc;
  if (reinterpret_cast<const ptsim_desc *>(desc)->kind != PTSIM_KIND_GEMM)
    return fail(PTSIM_E_UNSUPPORTED, "rows to owners: GEMM descriptors only");
  if (owner_ptrs == nullptr) return fail(PTSIM_E_ARGS, "rows to owners: no destination pointers");
  GemmOwners own{nowners, owner_rows, owner_ptrs};
  return launch_desc(desc, desc_bytes, dev_ptrs, nptr, lo, hi, workspace, workspace_bytes, stream, &own);
}

int ptsim_tp_reduce_gather(const void *stage, void *const *out, void *const *signal, int nranks, int rank, int64_t rows,
                           int64_t cols, int dtype, void *stream) {
  if (stage == nullptr || out == nullptr || signal == nullptr) return fail(PTSIM_E_ARGS, "reduce-gather pointers");
  return launch_tp_allreduce(nullptr, stage, out, signal, nranks, rank, rows, cols, dtype,
                             reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace ptsim {
static int launch_desc(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr, int64_t lo, int64_t hi,
                       void *workspace, size_t workspace_bytes, void *stream, const GemmOwners *own) {
  int rc = check_desc(desc, desc_bytes);
  if (rc) return rc;
  const ptsim_desc &d = *reinterpret_cast<const ptsim_desc *>(desc);
  if (nptr != d.nargs) return fail(PTSIM_E_ARGS, "%d pointers for a launch of %d arguments", nptr, d.nargs);
  for (int a = 0; a < nptr; ++a)
    if (dev_ptrs[a] == nullptr && d.arg_numel[a] > 0) return fail(PTSIM_E_ARGS, "argument %d is a null pointer", a);
  if (lo < 0 || hi > d.units || lo > hi)
    return fail(PTSIM_E_ARGS, "unit range [%lld, %lld) outside [0, %lld)", (long long)lo, (long long)hi, (long long)d.units);
  if (lo == hi) return PTSIM_OK;
  LaunchCtx c;
  c.stream = reinterpret_cast<cudaStream_t>(stream);
  PTSIM_CUDA(cudaGetDevice(&c.device));
  DeviceInfo info;
  if ((rc = device_info(c.device, &info))) return rc;
  c.sm_count = info.sm_count;
  switch (d.kind) {
    case PTSIM_KIND_ELEMENTWISE: return launch_elementwise(d, dev_ptrs, lo, hi, c);
    case PTSIM_KIND_ROW_SOFTMAX:
    case PTSIM_KIND_ROW_DIVSUM:
    case PTSIM_KIND_ROW_SUM:
    case PTSIM_KIND_ROW_RMSNORM: return launch_rowops(d, dev_ptrs, lo, hi, c);
    case PTSIM_KIND_TOPK: return launch_topk(d, dev_ptrs, lo, hi, c);
    case PTSIM_KIND_SORT: return launch_sort(d, dev_ptrs, lo, hi, workspace, workspace_bytes, c);
    case PTSIM_KIND_GATHER_ROWS: return launch_gather_rows(d, dev_ptrs, lo, hi, c);
    case PTSIM_KIND_GROUPED_GEMM: return launch_grouped_gemm(d, dev_ptrs, c);
    case PTSIM_KIND_GATHER_SUM: return launch_gather_sum(d, dev_ptrs, lo, hi, c);
    case PTSIM_KIND_INT_TABLE: return launch_itab(d, dev_ptrs, lo, hi, workspace, workspace_bytes, c);
    case PTSIM_KIND_QKNORM_ROPE: return launch_qkrope(d, dev_ptrs, lo, hi, c);
    case PTSIM_KIND_GEMM: return launch_gemm(d, dev_ptrs, lo, hi, workspace, workspace_bytes, c, own);
    case PTSIM_KIND_ATTN_PREFILL: return launch_attention(d, dev_ptrs, lo, hi, c);
    case PTSIM_KIND_REDUCE_ALL: return launch_reduce(d, dev_ptrs, lo, hi, workspace, workspace_bytes, c);
    case PTSIM_KIND_ATTN_DECODE: return launch_decode(d, dev_ptrs, lo, hi, workspace, workspace_bytes, c);
  }
  return fail(PTSIM_E_DESC, "descriptor kind %u", d.kind);
}
}  // namespace ptsim

extern "C" {

int64_t ptsim_workspace_size(const void *desc, size_t desc_bytes, int device) {
  if (check_desc(desc, desc_bytes)) return -1;
  const ptsim_desc &d = *reinterpret_cast<const ptsim_desc *>(desc);
  int sm_count = 148;
  DeviceInfo info;
  if (device >= 0 && device_info(device, &info) == PTSIM_OK) sm_count = info.sm_count;
  int64_t need = d.workspace_bytes;
  if (d.kind == PTSIM_KIND_REDUCE_ALL && need < reduce_workspace(sm_count)) need = reduce_workspace(sm_count);
  if (d.kind == PTSIM_KIND_ATTN_DECODE && need < decode_workspace(d, sm_count)) need = decode_workspace(d, sm_count);
  if (d.kind == PTSIM_KIND_INT_TABLE && need < itab_workspace(d, sm_count)) need = itab_workspace(d, sm_count);
  if (d.kind == PTSIM_KIND_GEMM && need < gemv_workspace(d, sm_count)) need = gemv_workspace(d, sm_count);
  if (d.kind == PTSIM_KIND_SORT && need < sort_workspace(d)) need = sort_workspace(d);
  return need;
}

int ptsim_launch_host(const void *desc, size_t desc_bytes, void *const *host_ptrs, void *const *dev_ptrs, int nptr,
                      uint32_t copy_in_mask, uint32_t copy_out_mask, int chunks, void *workspace,
                      size_t workspace_bytes, void *stream_in, void *stream_run, void *stream_out) {
  int rc = check_desc(desc, desc_bytes);
  if (rc) return rc;
  const ptsim_desc &d = *reinterpret_cast<const ptsim_desc *>(desc);
  if (nptr != d.nargs) return fail(PTSIM_E_ARGS, "%d pointers for a launch of %d arguments", nptr, d.nargs);
  for (int a = 0; a < nptr; ++a)
    if ((host_ptrs[a] == nullptr || dev_ptrs[a] == nullptr) && d.arg_numel[a] > 0)
      return fail(PTSIM_E_ARGS, "argument %d has a null host or device pointer", a);
  cudaStream_t s_in = reinterpret_cast<cudaStream_t>(stream_in), s_run = reinterpret_cast<cudaStream_t>(stream_run),
               s_out = reinterpret_cast<cudaStream_t>(stream_out);
  const bool row = d.kind == PTSIM_KIND_ROW_SOFTMAX || d.kind == PTSIM_KIND_ROW_RMSNORM;
  const ptsim_row_params &rp = d.p.row;
  int64_t n = row ? (chunks < 1 ? 1 : chunks) : 1;
  if (n > d.units) n = d.units < 1 ? 1 : d.units;
  auto bytes_of = [&](int a) { return d.arg_numel[a] * int64_t(dtype_size(d.arg_dtype[a])); };
  // The elements [first, end) of a row argument that units [lo, hi) touch (rows at `stride`).
  auto row_span = [&](int a, int64_t lo, int64_t hi, int64_t stride, int64_t &first, int64_t &end) {
    const int64_t r0 = lo * d.unit_size, r1 = hi * d.unit_size < rp.rows ? hi * d.unit_size : rp.rows;
    first = r0 * stride;
    end = r1 > r0 ? (r1 - 1) * stride + rp.cols : first;
    if (end > d.arg_numel[a]) end = d.arg_numel[a];
  };
  // Arguments copied whole, before the first range (a row launch's row-partitioned input and output go by range).
  for (int a = 0; a < nptr; ++a) {
    if (!(copy_in_mask & (1u << a)) || (row && (a == rp.in_arg || a == rp.out_arg))) continue;
    PTSIM_CUDA(cudaMemcpyAsync(dev_ptrs[a], host_ptrs[a], size_t(bytes_of(a)), cudaMemcpyHostToDevice, s_in));
  }
  for (int64_t k = 0; k < n; ++k) {
    const int64_t lo = d.units * k / n, hi = d.units * (k + 1) / n;   // the reference's split edges
    if (lo == hi) continue;
    if (row && (copy_in_mask & (1u << rp.in_arg))) {
      int64_t f, e;
      row_span(rp.in_arg, lo, hi, rp.in_row_stride, f, e);
      const int64_t es = dtype_size(d.arg_dtype[rp.in_arg]);
      if (e > f)
        PTSIM_CUDA(cudaMemcpyAsync(static_cast<char *>(dev_ptrs[rp.in_arg]) + f * es,
                                   static_cast<const char *>(host_ptrs[rp.in_arg]) + f * es, size_t((e - f) * es),
                                   cudaMemcpyHostToDevice, s_in));
    }
    cudaEvent_t ev_in, ev_run;
    PTSIM_CUDA(cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming));
    PTSIM_CUDA(cudaEventCreateWithFlags(&ev_run, cudaEventDisableTiming));
    PTSIM_CUDA(cudaEventRecord(ev_in, s_in));
    PTSIM_CUDA(cudaStreamWaitEvent(s_run, ev_in, 0));
    rc = ptsim_launch(desc, desc_bytes, dev_ptrs, nptr, lo, hi, workspace, workspace_bytes, stream_run);
    if (rc) {
      cudaEventDestroy(ev_in);
      cudaEventDestroy(ev_run);
      return rc;
    }
    PTSIM_CUDA(cudaEventRecord(ev_run, s_run));
    PTSIM_CUDA(cudaStreamWaitEvent(s_out, ev_run, 0));
    cudaEventDestroy(ev_in);    // released once their work completes
    cudaEventDestroy(ev_run);
    for (int a = 0; a < nptr; ++a) {
      if (!(copy_out_mask & (1u << a))) continue;
      int64_t f = 0, e = d.arg_numel[a];
      if (row && a == rp.out_arg) row_span(a, lo, hi, rp.out_row_stride, f, e);
      else if (k + 1 < n) continue;   // copied whole after the last range
      const int64_t es = dtype_size(d.arg_dtype[a]);
      if (e > f)
        PTSIM_CUDA(cudaMemcpyAsync(static_cast<char *>(host_ptrs[a]) + f * es, static_cast<const char *>(dev_ptrs[a]) + f * es,
                                   size_t((e - f) * es), cudaMemcpyDeviceToHost, s_out));
    }
  }
  return PTSIM_OK;
}

int ptsim_peer_alloc(size_t bytes, void **dev_ptr) {
  if (dev_ptr == nullptr || bytes == 0) return fail(PTSIM_E_ARGS, "peer buffer of %zu bytes", bytes);
  *dev_ptr = nullptr;
  PTSIM_CUDA(cudaMalloc(dev_ptr, bytes));
  PTSIM_CUDA(cudaMemset(*dev_ptr, 0, bytes));
  PTSIM_CUDA(cudaDeviceSynchronize());
  return PTSIM_OK;
}

int ptsim_peer_free(void *dev_ptr) {
  PTSIM_CUDA(cudaFree(dev_ptr));
  return PTSIM_OK;
}

int ptsim_peer_handle(void *dev_ptr, void *handle) {
  if (handle == nullptr) return fail(PTSIM_E_ARGS, "no room for the handle");
  cudaIpcMemHandle_t h;
  PTSIM_CUDA(cudaIpcGetMemHandle(&h, dev_ptr));
  memcpy(handle, &h, sizeof(h));
  return PTSIM_OK;
}

int ptsim_peer_open(const void *handle, void **dev_ptr) {
  if (handle == nullptr || dev_ptr == nullptr) return fail(PTSIM_E_ARGS, "peer open without a handle");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  PTSIM_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return PTSIM_OK;
}

int ptsim_peer_close(void *dev_ptr) {
  PTSIM_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return PTSIM_OK;
}

int ptsim_tp_allreduce(void *const *part, void *const *out, void *const *signal, int nranks, int rank, int64_t rows,
                       int64_t cols, int dtype, void *stream) {
  if (part == nullptr || out == nullptr || signal == nullptr) return fail(PTSIM_E_ARGS, "all-reduce pointer arrays");
  return launch_tp_allreduce(part, nullptr, out, signal, nranks, rank, rows, cols, dtype,
                             reinterpret_cast<cudaStream_t>(stream));
}

int ptsim_sync(void *stream, int32_t *device_status) {
  PTSIM_CUDA(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  int st = 0, zero = 0;
  PTSIM_CUDA(cudaMemcpyFromSymbol(&st, g_status, sizeof(int)));
  if (st != 0) PTSIM_CUDA(cudaMemcpyToSymbol(g_status, &zero, sizeof(int)));
  if (device_status) *device_status = st;
  return PTSIM_OK;
}

int ptsim_last_error(char *buf, int n) {
  if (buf == nullptr || n <= 0) return PTSIM_E_ARGS;
  strncpy(buf, t_err, size_t(n) - 1);
  buf[n - 1] = 0;
  return PTSIM_OK;
}

}  // extern "C"

extern "C" int ptsim_launch_reduce_noalloc(const void *desc, size_t desc_bytes, void *const *dev_ptrs, int nptr,
                                           void *stream) {
  using namespace ptsim;
  int rc = check_desc(desc, desc_bytes);
  if (rc) return rc;
  const ptsim_desc &d = *reinterpret_cast<const ptsim_desc *>(desc);
  if (d.kind != PTSIM_KIND_REDUCE_ALL)
    return fail(PTSIM_E_UNSUPPORTED, "ptsim_launch_reduce_noalloc runs whole-tensor reduction descriptors only");
  if (nptr != d.nargs) return fail(PTSIM_E_ARGS, "%d pointers for a launch of %d arguments", nptr, d.nargs);
  for (int a = 0; a < nptr; ++a)
    if (dev_ptrs[a] == nullptr && d.arg_numel[a] > 0) return fail(PTSIM_E_ARGS, "argument %d is a null pointer", a);
  if (d.units == 0) return PTSIM_OK;
  LaunchCtx c;
  c.stream = reinterpret_cast<cudaStream_t>(stream);
  PTSIM_CUDA(cudaGetDevice(&c.device));
  DeviceInfo info;
  if ((rc = device_info(c.device, &info))) return rc;
  c.sm_count = info.sm_count;
  int64_t need = reduce_workspace(c.sm_count);
  if (d.workspace_bytes > need) need = d.workspace_bytes;
  if (need > int64_t(kStaticScratchBytes))
    return fail(PTSIM_E_RESOURCE, "the reduction needs %lld bytes of scratch; the static scratch holds %zu",
                (long long)need, kStaticScratchBytes);
  void *scratch = nullptr;
  if ((rc = static_scratch(c.device, &scratch))) return rc;
  // Nothing in the scratch has to start at zero: pass 1 writes every partial that pass 2 reads, so the
  // previous call's contents never reach a result.
  return launch_reduce(d, dev_ptrs, 0, d.units, scratch, kStaticScratchBytes, c);
}
