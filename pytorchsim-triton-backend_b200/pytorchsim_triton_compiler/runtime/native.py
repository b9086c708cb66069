"""ctypes binding of libptsim_b200.so, the sm_100a executor (include/ptsim_b200.h).

There is no CPU path behind this module: when the library is missing or cannot load, every call raises
NativeUnavailable, so a launch fails loudly instead of computing anything elsewhere."""
import ctypes as C
import os
import threading

from ..codegen import descriptors as D

LIB_NAME = "libptsim_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_lib", LIB_NAME)

#: Every symbol include/ptsim_b200.h declares, with its ctypes signature.
SYMBOLS = {
    "ptsim_version": (C.c_int, []),
    "ptsim_desc_size": (C.c_size_t, []),
    "ptsim_init": (C.c_int, [C.c_int]),
    "ptsim_check": (C.c_int, [C.c_void_p, C.c_size_t]),
    "ptsim_units": (C.c_int64, [C.c_void_p, C.c_size_t]),
    "ptsim_launch": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p), C.c_int, C.c_int64, C.c_int64,
                               C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptsim_workspace_size": (C.c_int64, [C.c_void_p, C.c_size_t, C.c_int]),
    "ptsim_launch_reduce_noalloc": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p), C.c_int, C.c_void_p]),
    "ptsim_launch_host": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int,
                                    C.c_uint32, C.c_uint32, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                    C.c_void_p]),
    "ptsim_peer_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p)]),
    "ptsim_peer_free": (C.c_int, [C.c_void_p]),
    "ptsim_peer_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ptsim_peer_open": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "ptsim_peer_close": (C.c_int, [C.c_void_p]),
    "ptsim_tp_allreduce": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int,
                                     C.c_int, C.c_int64, C.c_int64, C.c_int, C.c_void_p]),
    "ptsim_launch_rows_to_owners": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p), C.c_int, C.c_int64,
                                              C.c_int64, C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p), C.c_int,
                                              C.c_int64, C.c_void_p]),
    "ptsim_tp_reduce_gather": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int, C.c_int,
                                         C.c_int64, C.c_int64, C.c_int, C.c_void_p]),
    "ptsim_sync": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "ptsim_last_error": (C.c_int, [C.c_char_p, C.c_int]),
}


class NativeUnavailable(RuntimeError):
    """The executor library is not built or does not load: nothing can run."""


class ExecutorError(RuntimeError):
    """A launch the executor refused or a kernel reported; `code` is the PTSIM_E_* status."""

    def __init__(self, code, message):
        super().__init__(f"{D.STATUS_NAME.get(code, code)} ({code}): {message}")
        self.code = code


_lib = None
_lock = threading.Lock()
_inited = set()


def library_path():
    return os.environ.get("PTSIM_B200_LIB", LIB_PATH)


def load():
    """The loaded library (built on first use when nvcc is present and the .so is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not os.path.exists(path):
            raise NativeUnavailable(f"{path} is not built: run __graft_entry__.build() (nvcc, sm_100a)")
        try:
            lib = C.CDLL(path)
        except OSError as e:
            raise NativeUnavailable(f"{path} does not load: {e}") from None
        for name, (res, argt) in SYMBOLS.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, argt
        if lib.ptsim_version() != D.ABI_VERSION:
            raise NativeUnavailable(f"{path} implements ABI {lib.ptsim_version()}, this package {D.ABI_VERSION}")
        if lib.ptsim_desc_size() != D.SIZE:
            raise NativeUnavailable(f"{path} reads {lib.ptsim_desc_size()}-byte descriptors, the Python mirror "
                                    f"writes {D.SIZE}: rebuild the library")
        _lib = lib
        return lib


def last_error():
    buf = C.create_string_buffer(1024)
    load().ptsim_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def _check(rc):
    if rc != 0:
        raise ExecutorError(rc, last_error())


def init(device):
    """Select `device` for this thread and prepare it (idempotent)."""
    lib = load()
    _check(lib.ptsim_init(int(device)))
    _inited.add(int(device))


def check(blob):
    """Validate a descriptor blob on the host (no GPU needed)."""
    buf = C.create_string_buffer(bytes(blob), len(blob))
    _check(load().ptsim_check(buf, len(blob)))


def units(blob):
    buf = C.create_string_buffer(bytes(blob), len(blob))
    n = load().ptsim_units(buf, len(blob))
    if n < 0:
        raise ExecutorError(D.E_DESC, last_error())
    return n


def workspace_size(blob, device=-1):
    """Device scratch bytes a launch of `blob` wants on `device` (the whole-tensor reduction's partials)."""
    n = load().ptsim_workspace_size(_desc_buffer(blob), len(blob), int(device))
    if n < 0:
        raise ExecutorError(D.E_DESC, last_error())
    return n


_desc_buffers = {}


def _desc_buffer(blob):
    """The ctypes copy of a descriptor, made once per distinct descriptor (launch overhead)."""
    blob = bytes(blob)
    buf = _desc_buffers.get(blob)
    if buf is None:
        if len(_desc_buffers) > 4096:
            _desc_buffers.clear()
        buf = _desc_buffers[blob] = C.create_string_buffer(blob, len(blob))
    return buf


def launch(blob, ptrs, lo, hi, workspace=0, workspace_bytes=0, stream=0):
    """Enqueue units [lo, hi) of descriptor `blob` over device pointers `ptrs` on `stream` (a raw
    cudaStream_t as int).  Asynchronous; sync() reports device-side failures."""
    lib = load()
    buf = _desc_buffer(blob)
    arr = (C.c_void_p * max(1, len(ptrs)))(*[C.c_void_p(int(p)) for p in ptrs])
    _check(lib.ptsim_launch(buf, len(blob), arr, len(ptrs), int(lo), int(hi), C.c_void_p(int(workspace) or None),
                            int(workspace_bytes), C.c_void_p(int(stream) or None)))


def launch_reduce_noalloc(blob, ptrs, stream=0):
    """Enqueue a whole-tensor reduction of `blob` with the library's own 4 KiB static scratch: for callers
    that cannot allocate device memory.  Calls that overlap on the GPU share that scratch and race."""
    lib = load()
    buf = _desc_buffer(blob)
    arr = (C.c_void_p * max(1, len(ptrs)))(*[C.c_void_p(int(p)) for p in ptrs])
    _check(lib.ptsim_launch_reduce_noalloc(buf, len(blob), arr, len(ptrs), C.c_void_p(int(stream) or None)))


def launch_host(blob, host_ptrs, dev_ptrs, copy_in, copy_out, chunks, workspace=0, workspace_bytes=0,
                stream_in=0, stream_run=0, stream_out=0):
    """Enqueue the whole launch of `blob` over host tensors (ptsim_launch_host): the arguments whose indices are in
    `copy_in` copied to their device buffers, the kernels run (a row launch in `chunks` pipelined unit ranges),
    the arguments in `copy_out` copied back.  Asynchronous."""
    lib = load()
    buf = _desc_buffer(blob)
    n = max(1, len(host_ptrs))
    hp = (C.c_void_p * n)(*[C.c_void_p(int(p)) for p in host_ptrs])
    dp = (C.c_void_p * n)(*[C.c_void_p(int(p)) for p in dev_ptrs])
    cin = sum(1 << int(i) for i in copy_in)
    cout = sum(1 << int(i) for i in copy_out)
    _check(lib.ptsim_launch_host(buf, len(blob), hp, dp, len(host_ptrs), cin, cout, int(chunks),
                                 C.c_void_p(int(workspace) or None), int(workspace_bytes), C.c_void_p(int(stream_in) or None),
                                 C.c_void_p(int(stream_run) or None), C.c_void_p(int(stream_out) or None)))


def peer_alloc(nbytes):
    """A zero-filled device buffer on the current device that other processes may map; its pointer."""
    p = C.c_void_p()
    _check(load().ptsim_peer_alloc(int(nbytes), C.byref(p)))
    return int(p.value)


def peer_free(ptr):
    _check(load().ptsim_peer_free(C.c_void_p(int(ptr))))


def peer_handle(ptr):
    """The 64-byte CUDA IPC handle of a buffer from peer_alloc."""
    buf = C.create_string_buffer(64)
    _check(load().ptsim_peer_handle(C.c_void_p(int(ptr)), buf))
    return bytes(buf.raw)


def peer_open(handle):
    """This process's pointer to another process's buffer, from its handle."""
    buf = C.create_string_buffer(bytes(handle), 64)
    p = C.c_void_p()
    _check(load().ptsim_peer_open(buf, C.byref(p)))
    return int(p.value)


def peer_close(ptr):
    _check(load().ptsim_peer_close(C.c_void_p(int(ptr))))


def tp_allreduce(part, out, signal, rank, rows, cols, stream=0):
    """Enqueue the tensor-parallel all-reduce (ptsim_tp_allreduce) of bf16 [rows, cols] partials; `part`, `out` and
    `signal` list every rank's pointers as this rank addresses them."""
    n = len(part)
    arr = lambda xs: (C.c_void_p * n)(*[C.c_void_p(int(x)) for x in xs])  # noqa: E731
    _check(load().ptsim_tp_allreduce(arr(part), arr(out), arr(signal), n, int(rank), int(rows), int(cols),
                                     D.DTYPE_CODE["bfloat16"], C.c_void_p(int(stream) or None)))


def sync(stream=0):
    """Wait for `stream`; raise ExecutorError when a kernel recorded a device-side failure."""
    st = C.c_int32(0)
    _check(load().ptsim_sync(C.c_void_p(int(stream) or None), C.byref(st)))
    if st.value:
        raise ExecutorError(st.value, "reported by a kernel on the device (status word)")


def launch_rows_to_owners(blob, ptrs, lo, hi, owners, owner_rows, workspace=0, workspace_bytes=0, stream=0):
    """ptsim_launch of GEMM descriptor `blob` with its output rows pushed to their owner ranks
    (ptsim_launch_rows_to_owners): rows [q owner_rows, (q + 1) owner_rows) go to device pointer owners[q]."""
    lib = load()
    buf = _desc_buffer(blob)
    arr = (C.c_void_p * max(1, len(ptrs)))(*[C.c_void_p(int(p)) for p in ptrs])
    own = (C.c_void_p * max(1, len(owners)))(*[C.c_void_p(int(p)) for p in owners])
    _check(lib.ptsim_launch_rows_to_owners(buf, len(blob), arr, len(ptrs), int(lo), int(hi),
                                           C.c_void_p(int(workspace) or None), int(workspace_bytes), own, len(owners),
                                           int(owner_rows), C.c_void_p(int(stream) or None)))


def tp_reduce_gather(stage, out, signal, rank, rows, cols, stream=0):
    """Enqueue the second half of the fused all-reduce (ptsim_tp_reduce_gather): this rank's staging `stage` (a
    device pointer) summed slot by slot into every rank's `out` (pointers as this rank addresses them)."""
    n = len(out)
    arr = lambda xs: (C.c_void_p * n)(*[C.c_void_p(int(x)) for x in xs])  # noqa: E731
    _check(load().ptsim_tp_reduce_gather(C.c_void_p(int(stage)), arr(out), arr(signal), n, int(rank), int(rows),
                                         int(cols), D.DTYPE_CODE["bfloat16"], C.c_void_p(int(stream) or None)))
