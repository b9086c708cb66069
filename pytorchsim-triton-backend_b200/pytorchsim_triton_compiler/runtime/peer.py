"""Buffers that every rank of a tensor-parallel group has mapped, for the all-reduce over NVLink peer memory
(ptsim_tp_allreduce, csrc/collective.cuh).

Each rank allocates its buffer with the executor (ptsim_peer_alloc: a zero-filled cudaMalloc), the ranks trade
the buffers' CUDA IPC handles through the process group, and every rank maps its peers' buffers
(ptsim_peer_open).  A buffer is then known by one pointer per rank, as this rank addresses it, and locally as a
torch tensor over this rank's own memory.  Plain device memory and peer loads and stores only: nothing is bound
to an NVLink multicast object.  Set-up allocates and synchronises; the launches that use the buffers do not."""
from . import native


class _Mem:
    """A __cuda_array_interface__ view of raw device memory, for torch.as_tensor."""

    def __init__(self, ptr, numel, typestr):
        self.__cuda_array_interface__ = {"shape": (int(numel),), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


_TYPESTR = {"bfloat16": ("<i2", 2), "float32": ("<f4", 4), "int32": ("<i4", 4), "uint8": ("|u1", 1)}


class PeerSet:
    """The peer-mapped buffers of rank `rank` of `world` ranks on `device`; `group` is the torch.distributed
    process group the handles travel through (the default group when None)."""

    def __init__(self, device, world, rank, group=None):
        import torch
        self.torch = torch
        self.device = torch.device(device)
        self.world, self.rank, self.group = world, rank, group
        self.tensors, self.ptrs = {}, {}
        self._own, self._opened = [], []

    def alloc(self, name, numel, dtype="bfloat16"):
        """A buffer of `numel` elements on every rank: this rank's torch tensor over it, and every rank's pointer
        to it (list indexed by rank)."""
        import torch.distributed as dist
        typestr, size = _TYPESTR[dtype]
        with self.torch.cuda.device(self.device):
            ptr = native.peer_alloc(max(16, numel * size))
            self._own.append(ptr)
            handles = [None] * self.world
            dist.all_gather_object(handles, native.peer_handle(ptr), group=self.group)
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(ptr)
                else:
                    p = native.peer_open(h)
                    self._opened.append(p)
                    ptrs.append(p)
            t = self.torch.as_tensor(_Mem(ptr, numel, typestr), device=self.device)
            if dtype == "bfloat16":
                t = t.view(self.torch.bfloat16)
        self.tensors[name], self.ptrs[name] = t, ptrs
        return t, ptrs

    def close(self):
        """Unmap the peers' buffers and free this rank's.  Every rank of the group calls it; a barrier makes
        sure no peer still works on a buffer this rank frees."""
        import torch.distributed as dist
        self.torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with self.torch.cuda.device(self.device):
            for p in self._opened:
                native.peer_close(p)
            for p in self._own:
                native.peer_free(p)
        self._opened, self._own, self.tensors, self.ptrs = [], [], {}, {}
