"""DMA-access traces of a launch, written under the runtime directory's dma_access/ as the reference's launch
provides that directory for its executor to fill (runtime/spike.py:108, merged over workers at :337-346).

For every unit range a launch ran, the trace lists its access streams: which argument, read or written, and
the elements touched.  The elements are an index map in the descriptors' own form (the analogue of the
reference's 4-D DMA descriptor, targets/tpu/lower_dma.py:11-35): element(i) = offset + sum over digits of
((i * scale // div) % mod) * stride, for i in [index[0], index[1]).  A dense box is the map whose digits are
its extents and strides.  Where the elements depend on data (a gather's table rows, the grouped GEMM's
rows), the stream is `indirect` and names the arguments the rows are read through; the grouped GEMM's rows
are also resolved from the group tables when the launch's host data is given, as the runtime-attribute
records of the reference carry the data-dependent quantities a timing model needs.

Format (JSON, one file per launch, dma_access/trace.json):
    {"format": FORMAT, "kernel": name, "kind": kind, "ranges": [
        {"device": d, "units": [lo, hi], "streams": [
            {"arg": name, "dir": "read" | "write", "dtype": dtype, "access": ACCESS, "elements": n}, ...]}]}
    ACCESS = {"map": {"offset", "digits": [[div, mod, stride], ...], "index": [i0, i1], "scale"?, "masked"?}}
           | {"indirect": {"through": [names], "rows": n, "row_elems": c, "resolved_rows": [[lo, hi], ...]?}}
`elements` counts the map's index range (an element touched twice counts twice, as a DMA moves it twice).  A
`masked` map is read only where the program's mask holds (an upper bound; no element outside the tensor is
read)."""
import json
import os

from ..codegen import descriptors as D

FORMAT = "ptsim-dma-access/1"
DIR = "dma_access"


def _map(offset, digits, i0, i1, scale=1):
    out = {"offset": int(offset), "digits": [[int(dv), int(md), int(st)] for dv, md, st in digits],
           "index": [int(i0), int(i1)]}
    if scale != 1:
        out["scale"] = int(scale)
    return {"map": out}


def _box(offset, dims):
    """A dense box: `dims` outermost first as (extent, stride) in elements."""
    digits, div = [], 1
    for ext, st in reversed(dims):
        digits.append((div, ext, st))
        div *= ext
    return _map(offset, digits, 0, div)


def _desc_map(m, i0, i1, scale=1):
    return _map(m.offset, [(m.div[k], m.mod[k], m.stride[k]) for k in range(m.ndigit)], i0, i1, scale)


def _count(access):
    if "map" in access:
        i0, i1 = access["map"]["index"]
        return max(0, i1 - i0)
    ind = access["indirect"]
    return ind["rows"] * ind["row_elems"]


def _rows(d, lo, hi, total):
    return lo * d.unit_size, min(hi * d.unit_size, total)


def _ew(d, lo, hi):
    e = d.p.ew
    i0, i1 = _rows(d, lo, hi, e.numel)
    return [(m.arg, "write" if k == e.store_map else "read", _desc_map(m, i0, i1)) for k, m in enumerate(list(e.map)[:e.nmap])]


def _row(d, lo, hi):
    p = d.p.row
    r0, r1 = _rows(d, lo, hi, p.rows)
    n = r1 - r0
    out = [(p.in_arg, "read", _box(r0 * p.in_row_stride, [(n, p.in_row_stride), (p.cols, 1)]))]
    if d.kind == D.ROW_SUM:
        out.append((p.out_arg, "write", _box(r0 * p.out_row_stride, [(n, p.out_row_stride)])))
    else:
        out.append((p.out_arg, "write", _box(r0 * p.out_row_stride, [(n, p.out_row_stride), (p.cols, 1)])))
    if d.kind == D.ROW_RMSNORM and p.weight_arg >= 0:
        out.append((p.weight_arg, "read", _box(0, [(p.cols, 1)])))
    if d.kind == D.ROW_RMSNORM and p.res_arg_p1 > 0:
        out.append((p.res_arg_p1 - 1, "read", _box(r0 * p.in_row_stride, [(n, p.in_row_stride), (p.cols, 1)])))
    return out


def _qk(d, lo, hi):
    q = d.p.qk
    r0, r1 = _rows(d, lo, hi, q.tokens * q.heads)
    if r1 <= r0:
        return []
    t0, t1 = r0 // q.heads, (r1 - 1) // q.heads + 1
    out = [(q.in_arg, "read", _box(r0 * q.dim, [((r1 - r0) * q.dim, 1)])),
           (q.cos_arg, "read", _box(t0 * q.dim, [((t1 - t0) * q.dim, 1)])),
           (q.sin_arg, "read", _box(t0 * q.dim, [((t1 - t0) * q.dim, 1)])),
           (q.out_arg, "write", _map(0, [(1, q.dim, 1), (q.dim, q.heads, q.out_head_stride),
                                         (q.dim * q.heads, q.tokens, q.out_tok_stride)], r0 * q.dim, r1 * q.dim))]
    if not q.no_norm:
        out.append((q.weight_arg, "read", _box(0, [(q.dim, 1)])))
    return out


def _vprog_loads(v, n):
    return [(ld.arg, "read", _box(ld.offset, [(n, ld.stride)])) for ld in list(v.load)[:v.nload]]


def _gemm(d, lo, hi):
    g = d.p.gemm
    m0, m1 = (0, 1) if g.M == 1 else _rows(d, lo, hi, g.M)
    n = m1 - m0
    out = []
    if g.M == 1 and g.pro.ncode:
        out += _vprog_loads(g.pro, g.K)
    else:
        out.append((g.a_arg, "read", _box(m0 * g.lda, [(n, g.lda), (g.K, 1)])))
    out.append((g.b_arg, "read", _box(0, [(g.N, g.ldb), (g.K, 1)] if g.b_kmajor else [(g.K, g.ldb), (g.N, 1)])))
    if g.r_arg >= 0:
        out.append((g.r_arg, "read", _box(m0 * g.ldr, [(n, g.ldr), (g.N, 1)])))
    if g.M == 1 and g.epi.ncode:
        out += _vprog_loads(g.epi, g.N)
    out.append((g.c_arg, "write", _box(m0 * g.ldc, [(n, g.ldc), (g.N, 1)])))
    return out


def _attn(d, lo, hi):
    a = d.p.attn
    S, Dm = a.seq, a.dim
    if d.kind == D.ATTN_DECODE:
        G = a.hq // max(1, a.hkv)
        u0, u1 = _rows(d, lo, hi, a.hkv)
        return [(a.q_arg, "read", _box(u0 * G * Dm, [((u1 - u0) * G * Dm, 1)])),
                (a.k_arg, "read", _box(u0 * S * Dm, [((u1 - u0) * S * Dm, 1)])),
                (a.v_arg, "read", _box(u0 * S * Dm, [((u1 - u0) * S * Dm, 1)])),
                (a.o_arg, "write", _box(u0 * G * Dm, [((u1 - u0) * G * Dm, 1)]))]
    u0, u1 = _rows(d, lo, hi, a.batch * a.hq)
    if u1 <= u0:
        return []
    kvh = lambda u: (u // a.hq) * a.hkv + (u % a.hq) // (a.hq // a.hkv)   # noqa: E731
    k0, k1 = kvh(u0), kvh(u1 - 1) + 1
    return [(a.q_arg, "read", _box(u0 * S * Dm, [((u1 - u0) * S * Dm, 1)])),
            (a.k_arg, "read", _box(k0 * S * Dm, [((k1 - k0) * S * Dm, 1)])),
            (a.v_arg, "read", _box(k0 * S * Dm, [((k1 - k0) * S * Dm, 1)])),
            (a.o_arg, "write", _box(u0 * S * Dm, [((u1 - u0) * S * Dm, 1)]))]


def _reduce(d, lo, hi):
    r = d.p.red
    out = _vprog_loads(r.pro, r.numel) if r.pro.ncode else [(r.in_arg, "read", _box(0, [(r.numel, 1)]))]
    return out + [(r.out_arg, "write", _box(0, [(1, 1)]))]


def _select(d, lo, hi):
    e = d.p.sel
    r0, r1 = _rows(d, lo, hi, e.rows)
    width = e.k if d.kind == D.TOPK else e.cols
    return [(e.in_arg, "read", _box(r0 * e.cols, [((r1 - r0) * e.cols, 1)])),
            (e.val_arg, "write", _box(r0 * width, [((r1 - r0) * width, 1)])),
            (e.idx_arg, "write", _box(r0 * width, [((r1 - r0) * width, 1)]))]


def _gather(d, lo, hi, names):
    gp = d.p.gat
    r0, r1 = _rows(d, lo, hi, gp.rows)
    return [(gp.idx_arg, "read", _desc_map(gp.idx_map, r0, r1)),
            (gp.table_arg, "read", {"indirect": {"through": [names[gp.idx_arg]], "rows": r1 - r0, "row_elems": gp.cols}}),
            (gp.out_arg, "write", _box(r0 * gp.cols, [((r1 - r0) * gp.cols, 1)]))]


def _ggemm(d, lo, hi, host=None, names=None):
    p = d.p.ggemm
    tables = [p.group_arg, p.start_arg, p.rows_arg]
    rows = None
    if host is not None and names is not None:
        import numpy as np
        grp = np.asarray(host[names[p.group_arg]]).reshape(-1)[:p.programs].astype(np.int64)
        start = np.asarray(host[names[p.start_arg]]).reshape(-1).astype(np.int64)
        cnt = np.asarray(host[names[p.rows_arg]]).reshape(-1).astype(np.int64)
        spans = sorted({(int(start[g]), int(start[g] + cnt[g])) for g in grp if 0 <= g < start.size and cnt[g] > 0})
        rows = spans
    listed = sum(hi_ - lo_ for lo_, hi_ in rows) if rows is not None else p.M

    def ind(row_elems):
        x = {"through": [names[t] for t in tables] if names else tables, "rows": int(listed), "row_elems": int(row_elems)}
        if rows is not None:
            x["resolved_rows"] = [[a, b] for a, b in rows]
        return {"indirect": x}
    return [(t, "read", _box(0, [(d.arg_numel[t], 1)])) for t in tables] + [
        (p.a_arg, "read", ind(p.K)),
        (p.b_arg, "read", _box(0, [(p.groups * p.K * p.N, 1)])),
        (p.c_arg, "write", ind(p.N))]


def _gsum(d, lo, hi, names):
    p = d.p.gsum
    r0, r1 = _rows(d, lo, hi, p.rows)
    f0, f1 = r0 * p.terms, r1 * p.terms             # terms f = r * terms + k
    out, through = [], []
    for i in list(p.code)[:p.ncode]:
        if i.op == D.IOP["load"] and i.a < D.GSUM_MAPS:
            m = p.maps[i.a]
            out.append((m.arg, "read", _desc_map(m, f0, f1)))
            through.append(names[m.arg])
        elif i.op == D.IOP["loadi"]:
            out.append((i.c, "read", {"indirect": {"through": sorted(set(through)), "rows": f1 - f0, "row_elems": 1}}))
            through.append(names[i.c])
    out += [(p.w_map.arg, "read", _desc_map(p.w_map, f0, f1)),
            (p.table_arg, "read", {"indirect": {"through": sorted(set(through)), "rows": f1 - f0, "row_elems": p.cols}})]
    if p.wdiv:
        out.append((p.wdiv_arg, "read", _box(p.wdiv_offset + r0 * p.wdiv_stride, [(r1 - r0, p.wdiv_stride)])))
    for k in range(p.nres):
        out.append((p.res_arg[k], "read", _box(r0 * p.cols, [((r1 - r0) * p.cols, 1)])))
    out.append((p.out_arg, "write", _box(r0 * p.cols, [((r1 - r0) * p.cols, 1)])))
    return out


def _itab(d, lo, hi, names):
    q = d.p.itab
    r0, r1 = _rows(d, lo, hi, q.rows)
    out = []
    for i in list(q.code)[:q.ncode]:
        if i.op in (D.IOP["load"], D.IOP["loadm"]):
            acc = _desc_map(q.maps[i.a], r0 * q.cols, r1 * q.cols)
            if i.op == D.IOP["loadm"]:
                acc["map"]["masked"] = True   # read only where the program's mask holds: an upper bound
            out.append((i.c, "read", acc))
        elif i.op == D.IOP["loadi"]:
            out.append((i.c, "read", {"indirect": {"through": [names[x.c] for x in list(q.code)[:q.ncode]
                                                                if x.op in (D.IOP["load"], D.IOP["loadm"])],
                                                    "rows": (r1 - r0) * q.cols, "row_elems": 1}}))
    for o in list(q.out)[:q.nout]:
        m = q.maps[o.map]
        if o.mode == D.ITAB_MODE["sum"]:
            out.append((o.arg, "write", _desc_map(m, r0, r1, scale=q.cols)))
        else:
            out.append((o.arg, "write", _desc_map(m, r0 * q.cols, r1 * q.cols)))
    return out


def streams(desc, lo, hi, names, dtypes=None, host=None):
    """The access streams of units [lo, hi) of `desc`, arguments named by `names` (argument order)."""
    d = desc
    k = d.kind
    if k == D.ELEMENTWISE:
        raw = _ew(d, lo, hi)
    elif k in (D.ROW_SOFTMAX, D.ROW_RMSNORM, D.ROW_DIVSUM, D.ROW_SUM):
        raw = _row(d, lo, hi)
    elif k == D.QKNORM_ROPE:
        raw = _qk(d, lo, hi)
    elif k == D.GEMM:
        raw = _gemm(d, lo, hi)
    elif k in (D.ATTN_PREFILL, D.ATTN_DECODE):
        raw = _attn(d, lo, hi)
    elif k == D.REDUCE_ALL:
        raw = _reduce(d, lo, hi)
    elif k in (D.TOPK, D.SORT):
        raw = _select(d, lo, hi)
    elif k == D.GATHER_ROWS:
        raw = _gather(d, lo, hi, names)
    elif k == D.GROUPED_GEMM:
        raw = _ggemm(d, lo, hi, host, names)
    elif k == D.GATHER_SUM:
        raw = _gsum(d, lo, hi, names)
    elif k == D.INT_TABLE:
        raw = _itab(d, lo, hi, names)
    else:
        raise ValueError(f"no DMA-access plan for descriptor kind {k}")
    return [{"arg": names[a], "dir": direction, "dtype": (dtypes or {}).get(names[a]), "access": acc,
             "elements": _count(acc)} for a, direction, acc in raw]


def elements(access):
    """The element indices of a `map` access (numpy int64, in index order); None for an indirect one."""
    if "map" not in access:
        return None
    import numpy as np
    m = access["map"]
    i = np.arange(m["index"][0], m["index"][1], dtype=np.int64) * m.get("scale", 1)
    e = np.full(i.shape, m["offset"], dtype=np.int64)
    for dv, md, st in m["digits"]:
        e += ((i // dv) % md) * st
    return e


def bounds(access):
    """(lowest, highest) element a `map` access can name, from its digits' ranges over the index range (exact
    for dense boxes, never narrower than the truth); None for an indirect one or an empty range."""
    if "map" not in access:
        return None
    m = access["map"]
    i0, i1 = m["index"]
    if i1 <= i0:
        return None
    sc = m.get("scale", 1)
    lo = hi = m["offset"]
    for dv, md, st in m["digits"]:
        q0, q1 = (i0 * sc) // dv, ((i1 - 1) * sc) // dv
        if q1 - q0 + 1 >= md or q0 % md > q1 % md:
            v0, v1 = 0, md - 1
        else:
            v0, v1 = q0 % md, q1 % md
        a, b = v0 * st, v1 * st
        lo += min(a, b)
        hi += max(a, b)
    return lo, hi


def write(runtime, manifest, desc, ranges, host=None):
    """Write dma_access/trace.json under `runtime` for the unit `ranges` ([(device, lo, hi)]) of a launch."""
    names = [a["name"] for a in manifest["args"]]
    dtypes = {a["name"]: a["dtype"] for a in manifest["args"]}
    out = {"format": FORMAT, "kernel": manifest.get("name"), "kind": D.KIND_NAME.get(desc.kind, desc.kind),
           "ranges": [{"device": dev, "units": [lo, hi], "streams": streams(desc, lo, hi, names, dtypes, host)}
                      for dev, lo, hi in ranges]}
    path = os.path.join(runtime, DIR)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "trace.json"), "w") as fh:
        json.dump(out, fh)
    return out
