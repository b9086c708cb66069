"""A launch graph: the kernel objects of one workload run back to back on one stream over named device
buffers -- what PyTorchSim does when it runs a model's kernels one after another (the bundle's
manifest.json lists a workload's launches in order, e.g. validation/pytorchsim/
qwen3_8b_layer_prefill_2048x2048_bf16/manifest.json).  Buffers are allocated once and stay resident;
a graph can be captured into a CUDA graph so a many-launch workload costs one launch from the host."""
import math

from ..codegen import descriptors as D
from . import native


class Graph:
    def __init__(self, device):
        import torch
        self.torch = torch
        self.device = torch.device(device)
        self.buffers = {}
        self.steps = []          # (name, blob, [buffer names], workspace, units, owners)
        self.cuda_graph = None

    def buffer(self, name, numel, dtype, init=None):
        """A device buffer `name` of `numel` elements (`dtype`: a kernel.json dtype name), optionally
        filled from `init` (a CPU tensor of that many elements)."""
        torch = self.torch
        dt = getattr(torch, dtype)
        if name in self.buffers:
            t = self.buffers[name]
            if t.numel() != numel or t.dtype != dt:
                raise ValueError(f"buffer {name} exists as {t.numel()} x {t.dtype}, asked {numel} x {dt}")
        else:
            t = torch.empty(int(numel), dtype=dt, device=self.device)
            self.buffers[name] = t
        if init is not None:
            t.copy_(init.reshape(-1).to(dt))
        return t

    def add(self, name, blob, bufs, owners=None):
        """Append a launch of descriptor `blob` whose tensor arguments are the buffers `bufs`, in the
        descriptor's argument order; every buffer must exist with the descriptor's element count.  `owners`
        = (device pointers, rows): a GEMM whose output rows go to their owner ranks in blocks of `rows`
        (native.launch_rows_to_owners) instead of into its output buffer."""
        d = D.from_bytes(blob)
        if len(bufs) != d.nargs:
            raise ValueError(f"{name}: {len(bufs)} buffers for {d.nargs} arguments")
        for i, b in enumerate(bufs):
            t = self.buffers[b]
            if t.numel() != d.arg_numel[i]:
                raise ValueError(f"{name}: buffer {b} holds {t.numel()} elements, argument {i} wants {d.arg_numel[i]}")
        native.check(blob)
        ws = None
        n = native.workspace_size(blob, self.device.index or 0)
        if n > 0:
            ws = self.torch.empty(int(n), dtype=self.torch.uint8, device=self.device)
        self.steps.append((name, bytes(blob), list(bufs), ws, d.units, owners))

    def launch_count(self):
        return len(self.steps)

    def run(self, stream=None, sync=False):
        """Enqueue every launch in order on `stream` (torch's current stream by default)."""
        torch = self.torch
        s = stream or torch.cuda.current_stream(self.device)
        if self.cuda_graph is not None and stream is None:
            self.cuda_graph.replay()
        else:
            for step in self.steps:
                self._launch(step, s.cuda_stream)
        if sync:
            native.sync(s.cuda_stream)

    def _launch(self, step, stream):
        name, blob, bufs, ws, units, owners = step
        ptrs = [self.buffers[b].data_ptr() for b in bufs]
        wp, wn = (ws.data_ptr(), ws.numel()) if ws is not None else (0, 0)
        if owners is None:
            native.launch(blob, ptrs, 0, units, wp, wn, stream)
        else:
            native.launch_rows_to_owners(blob, ptrs, 0, units, owners[0], owners[1], wp, wn, stream)

    def capture(self):
        """Capture the launch sequence into a CUDA graph (replayed by run())."""
        torch = self.torch
        native.init(self.device.index or 0)
        self.run(sync=True)   # first use of every kernel outside the capture
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for step in self.steps:
                    self._launch(step, s.cuda_stream)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.cuda_graph = g
        return g


def flops_of(blob):
    """Algorithmic flops of one launch (GEMM 2MNK, causal attention 2*B*HQ*S^2*D), else 0."""
    d = D.from_bytes(blob)
    if d.kind == D.GEMM:
        g = d.p.gemm
        return 2 * g.M * g.N * g.K
    if d.kind == D.ATTN_PREFILL:
        a = d.p.attn
        full = 4 * a.batch * a.hq * a.seq * a.seq * a.dim
        return full // 2 if a.causal else full
    return 0


def numel(shape):
    return math.prod(shape)
