"""The CUDA device: the package's launcher for a lowered kernel object, in the place of runtime/spike.py.

Same shape as the reference's spike.launch (pytorchsim_triton_compiler/runtime/spike.py:100-120): the caller
owns the tensors (one .raw file per argument, or tensors in memory), the written arguments are left where
they were, a failure raises `error(message)`, and a grid past kernel.json's grid_bound is refused
(contract/kernel_object.py refuse_grid_past_bound).  Where Spike cut the grid into program ranges over
processes (spike.py:83-98, 253-291), this launcher cuts the descriptor's units into ascending ranges over
GPUs, one host thread per GPU, and merges the written bytes exactly as merge_worker_outputs does
(spike.py:310-334): a nonzero byte was written; two ranges writing one byte differently means the split
cannot give the answer, and the grid reruns on one GPU.  An argument read as well as written keeps the
launch on one GPU (kernel_object.splittable)."""
import concurrent.futures as cf
import os

import numpy as np

from ..codegen import descriptors as D
from ..contract import kernel_object as ko
from . import dma_access, native


class CudaError(RuntimeError):
    """A CUDA launch, or the merge around it, failed."""


class NotSplittable(Exception):
    """Which range ran last would decide the answer, so the split cannot give it."""


def _torch():
    import torch
    return torch


TORCH_DTYPE = {"float32": "float32", "float16": "float16", "bfloat16": "bfloat16", "float64": "float64",
               "int64": "int64", "int32": "int32", "int16": "int16", "int8": "int8", "uint8": "uint8", "bool": "int8",
               "float8_e5m2": "uint8", "float8_e4m3fn": "uint8", "uint16": "int16", "uint32": "int32",
               "uint64": "int64"}


def devices_available():
    torch = _torch()
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def jobs(manifest, total, log, want=None, ndev=None):
    """How many GPUs run the units: 1 when an inout argument lets one program read another's store, else
    `want` (the caller's override), else every visible GPU; never more than `total`."""
    if not ko.splittable(manifest):
        inout = [a["name"] for a in manifest["args"] if a["role"] == "inout"]
        log(f"[cuda] one device: {', '.join(inout)} is read as well as written, so a program may depend on "
            f"another one's store")
        return 1
    if want:
        return max(1, min(int(want), total))
    n = devices_available() if ndev is None else ndev
    return max(1, min(n, total))


def split(total, n):
    """Ascending disjoint unit ranges, the edges spike._split uses (total * w // n)."""
    edges = [(total * w) // n for w in range(n + 1)]
    return [(edges[w], edges[w + 1]) for w in range(n) if edges[w] < edges[w + 1]]


_workspaces = {}


def workspace_for(blob, device):
    """Scratch a launch of `blob` wants on `device` (split-K partials, reduction partials), as a device
    tensor kept per device and grown on demand (or None)."""
    n = native.workspace_size(blob, device.index if device.index is not None else 0)
    if n <= 0:
        return None
    torch = _torch()
    ws = _workspaces.get(device)
    if ws is None or ws.numel() < n:
        ws = _workspaces[device] = torch.empty(int(n), dtype=torch.uint8, device=device)
    return ws


def launch_tensors(blob, tensors, lo=0, hi=None, stream=None, sync=True):
    """Run units [lo, hi) of descriptor `blob` over CUDA tensors (argument order), on `stream` (torch's
    current stream by default).  Tensors are used in place.  With sync=True, waits and checks the device
    status word."""
    torch = _torch()
    desc = D.from_bytes(blob)
    if len(tensors) != desc.nargs:
        raise CudaError(f"{len(tensors)} tensors for a launch of {desc.nargs} arguments")
    dev = None
    for i, t in enumerate(tensors):
        if not t.is_cuda:
            raise CudaError(f"argument {i} is not on a CUDA device; the executor has no CPU path")
        if not t.is_contiguous():
            raise CudaError(f"argument {i} is not contiguous; kernel.json tensors are flat")
        if t.numel() != desc.arg_numel[i]:
            raise CudaError(f"argument {i} holds {t.numel()} elements, the descriptor {desc.arg_numel[i]}")
        dev = t.device if dev is None else dev
        if t.device != dev:
            raise CudaError("every argument of one launch is on one device")
    hi = desc.units if hi is None else hi
    with torch.cuda.device(dev):
        native.init(dev.index)
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        ws = workspace_for(blob, dev)
        native.launch(blob, [t.data_ptr() for t in tensors], lo, hi,
                      ws.data_ptr() if ws is not None else 0, ws.numel() if ws is not None else 0, s.cuda_stream)
        if sync:
            native.sync(s.cuda_stream)
    return tensors


def written_args(desc):
    """Indices of the arguments a launch of `desc` writes (the launch's outputs), for every descriptor
    kind; CudaError for a kind this build does not know."""
    k, p = desc.kind, desc.p
    if k == D.ELEMENTWISE:
        return [p.ew.map[p.ew.store_map].arg]
    if k in (D.ROW_SOFTMAX, D.ROW_RMSNORM, D.ROW_DIVSUM, D.ROW_SUM):
        return [p.row.out_arg]
    if k == D.QKNORM_ROPE:
        return [p.qk.out_arg]
    if k == D.GEMM:
        return [p.gemm.c_arg]
    if k in (D.ATTN_PREFILL, D.ATTN_DECODE):
        return [p.attn.o_arg]
    if k == D.REDUCE_ALL:
        return [p.red.out_arg]
    if k in (D.TOPK, D.SORT):
        return [p.sel.val_arg, p.sel.idx_arg]
    if k == D.GATHER_ROWS:
        return [p.gat.out_arg]
    if k == D.GROUPED_GEMM:
        return [p.ggemm.c_arg]
    if k == D.GATHER_SUM:
        return [p.gsum.out_arg]
    if k == D.INT_TABLE:
        return sorted({o.arg for o in list(p.itab.out)[:p.itab.nout]})
    raise CudaError(f"descriptor kind {k} ({D.KIND_NAME.get(k, 'unknown')}) has no known outputs")


class HostPipeline:
    """Launches over tensors in host memory, the way a caller holding `.raw` data runs the executor end to
    end: each launch's arguments are copied to the GPU, the kernels run, and the written arguments are
    copied back into the host tensors.  Copies run on their own streams (host-to-device, device-to-host)
    beside the compute stream, and a row-wise launch (softmax, RMSNorm) is cut into `chunks` unit ranges
    so the transfer of one range overlaps the kernel of the previous one and the return of the one before
    that; PCIe then carries both directions at once.  The copies, kernels and stream ordering of a launch are
    enqueued by one native call (ptsim_launch_host), so the host cost per range is microseconds.  Host
    tensors should be pinned for the copies to be asynchronous.  Launches submitted to one pipeline run in
    submission order; wait() synchronises and raises ExecutorError if a kernel reported a failure."""

    def __init__(self, device=0, chunks=4):
        torch = _torch()
        self.torch = torch
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.chunks = max(1, int(chunks))
        native.init(self.device.index or 0)
        self.s_in = torch.cuda.Stream(self.device)
        self.s_run = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self._live = []

    def submit(self, blob, host):
        torch = self.torch
        desc = D.from_bytes(blob)
        if len(host) != desc.nargs:
            raise CudaError(f"{len(host)} host tensors for a launch of {desc.nargs} arguments")
        for i, t in enumerate(host):
            if t.is_cuda or not t.is_contiguous() or t.numel() != desc.arg_numel[i]:
                raise CudaError(f"argument {i}: a contiguous host tensor of {desc.arg_numel[i]} elements is required")
        outs = written_args(desc)
        dev = [torch.empty(t.numel(), dtype=t.dtype, device=self.device) for t in host]
        ptrs = [t.data_ptr() for t in dev]
        ws = workspace_for(blob, self.device)
        wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (0, 0)
        self._live.append((dev, ws))
        # One native call enqueues the copies in, the kernels and the copies back (a row launch in pipelined unit
        # ranges): every argument goes in (an output's initial bytes matter for arguments read as well as
        # written), the written ones come back.
        with torch.cuda.device(self.device):
            native.launch_host(blob, [t.data_ptr() for t in host], ptrs, range(desc.nargs), outs, self.chunks, wsp, wsn,
                               self.s_in.cuda_stream, self.s_run.cuda_stream, self.s_out.cuda_stream)
        return host

    def wait(self):
        self.s_out.synchronize()
        self.s_in.synchronize()
        native.sync(self.s_run.cuda_stream)
        self._live.clear()


def read_raw(path, arg):
    want = ko.numel(arg)
    data = np.fromfile(path, dtype=np.dtype(ko.NP_DTYPE[arg["dtype"]]), count=want)
    if data.size != want:
        raise CudaError(f"{path}: {data.size} elements, the manifest says {want} (file truncated?)")
    return data


def _to_device(arr, arg, device):
    torch = _torch()
    t = torch.from_numpy(np.ascontiguousarray(arr))
    want = getattr(torch, TORCH_DTYPE[arg["dtype"]])
    if t.dtype != want:
        t = t.view(want)
    return t.to(device, non_blocking=False)


def _run_range(blob, manifest, host, device, lo, hi):
    """Copy every argument to `device`, run units [lo, hi), return the written arguments' bytes."""
    torch = _torch()
    with torch.cuda.device(device):
        ts = [_to_device(host[a["name"]], a, torch.device("cuda", device)) for a in manifest["args"]]
        launch_tensors(blob, ts, lo, hi)
        out = {}
        for a, t in zip(manifest["args"], ts):
            if a["role"] in ("out", "inout"):
                out[a["name"]] = t.view(torch.uint8).cpu().numpy() if t.element_size() == 1 else \
                    t.cpu().contiguous().view(torch.uint8).numpy()
        return out


def merge(manifest, base, parts):
    """Fold the ranges' copies of each written buffer over `base` (the bytes before the launch): a byte
    that differs from base was written; two ranges writing one byte differently raise NotSplittable."""
    merged = {}
    for a in ko.writable(manifest):
        b = base[a["name"]]
        acc, written = b.copy(), np.zeros(b.size, dtype=bool)
        for p in parts:
            got = p[a["name"]]
            if got.size != b.size:
                raise CudaError(f"a range returned {got.size} bytes for {a['name']}, expected {b.size}")
            changed = got != b
            clash = changed & written & (got != acc)
            if clash.any():
                raise NotSplittable(f"two unit ranges wrote {a['name']} byte {int(np.flatnonzero(clash)[0])} "
                                    f"differently, so which ran last decides the answer")
            acc[changed] = got[changed]
            written |= changed
        merged[a["name"]] = acc
    return merged


def launch(desc_blob, manifest, runtime, raw_paths, options=None, *, log=print, error=CudaError, want_jobs=None,
           scalar_values=None, grid=None, devices=None):
    """Run the whole launch over the .raw files in `raw_paths` (name -> path), leaving each written argument
    in its file.  `desc_blob` is the kernel object's descriptor (kernel_object.read_desc).  `devices` lists
    the GPUs to use (all visible ones by default); `want_jobs` caps how many.  `scalar_values` ({name:
    value}) are the launch's scalar arguments, as spike.launch takes them: the descriptor holds the values
    it was lowered with, so a value that differs is refused (relower the kernel for it) instead of ignored."""
    try:
        ko.refuse_grid_past_bound(manifest, manifest["grid"] if grid is None else grid)
        ko.check_launch_scalars(manifest, scalar_values)
        if grid is not None and tuple(ko.grid3(grid)) != tuple(ko.grid3(manifest["grid"])):
            raise error(f"{manifest.get('name')}: the descriptor was lowered for grid {tuple(ko.grid3(manifest['grid']))}"
                        f"; relower for grid {tuple(ko.grid3(grid))}")
        desc = D.from_bytes(desc_blob)
        host = {a["name"]: read_raw(raw_paths[a["name"]], a) for a in manifest["args"]}
    except (ko.ObjectError, ValueError) as e:
        raise error(str(e)) from None
    devs = list(devices) if devices is not None else list(range(devices_available()))
    if not devs:
        raise error("no CUDA device is visible; the B200 executor has no CPU path")
    total = desc.units
    n = jobs(manifest, total, log, want_jobs, ndev=len(devs))
    ranges = split(total, n)
    log(f"[cuda] {total} units over {len(ranges)} device(s)")
    base = {a["name"]: host[a["name"]].view(np.uint8).copy() for a in ko.writable(manifest)}
    ran = [(devs[w], lo, hi) for w, (lo, hi) in enumerate(ranges)]
    try:
        if len(ranges) == 1:
            parts = [_run_range(desc_blob, manifest, host, devs[0], *ranges[0])]
        else:
            with cf.ThreadPoolExecutor(max_workers=len(ranges)) as pool:
                futs = [pool.submit(_run_range, desc_blob, manifest, host, devs[w], lo, hi)
                        for w, (lo, hi) in enumerate(ranges)]
                parts = [f.result() for f in futs]
        try:
            merged = merge(manifest, base, parts)
        except NotSplittable as why:
            log(f"[cuda] {why} -- running the grid on one device instead")
            merged = merge(manifest, base, [_run_range(desc_blob, manifest, host, devs[0], 0, total)])
            ran = [(devs[0], 0, total)]
    except native.ExecutorError as e:
        raise error(str(e)) from None
    for a in ko.writable(manifest):
        merged[a["name"]].tofile(raw_paths[a["name"]])
    # The DMA-access trace of the ranges that ran (runtime/dma_access/trace.json), from the descriptor's index
    # maps; the grouped GEMM's data-dependent rows resolved from the launch's own tables.
    dma_access.write(runtime, manifest, desc, ran, host)
    return runtime
