"""The Qwen3-8B-shaped prefill layer end to end on the B200: the 14 launches of the
bundle's workload wired over resident buffers (runtime/qwen3.py), against the oracle's restatement of the
same launches.  The composite is compared by relative L2 error (< 1e-2): each launch is checked
element-wise in test_gpu_objects.py; here the wiring, the buffer reuse and the CUDA-graph replay are
checked.  T = 2048 runs the reference's own lowered kernel objects; T = 256 runs descriptors built for the
shape.  Tensor parallel over 2 GPUs (NCCL all-reduce) runs when the box has two."""
import os

import pytest
import torch

from oracle import programs as O
from pytorchsim_triton_compiler.contract import kernel_object as ko
from pytorchsim_triton_compiler.runtime import qwen3 as Q

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def reference_objects(T):
    tag = f"qwen3_t{T}"
    objdir = os.path.join(HERE, "golden", "objects")
    out = {}
    for name in sorted(os.listdir(objdir)):
        if name.startswith(tag + "_"):
            out[name.split("_")[2]] = ko.read_desc(os.path.join(objdir, name))
    return out


def run_layer(T, objects=None, graph=False):
    p = Q.random_params(0)
    x = torch.randn(T * Q.HIDDEN, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    cos, sin = O.rope_tables(T)
    g, _ = Q.build_layer("cuda:0", T, p, cos, sin, x, objects=objects)
    if graph:
        g.capture()
        g.buffers["y"].zero_()
    g.run(sync=True)
    want = O.decoder_layer(x, p, T, cos=cos, sin=sin).float()
    got = g.buffers["y"].float().cpu()
    return float((got - want).norm() / want.norm())


def test_layer_t256_built_descriptors():
    assert run_layer(256) < 1e-2


def test_layer_t2048_reference_objects_cuda_graph():
    objs = reference_objects(2048)
    assert sorted(objs) == ["00", "01", "02", "03", "04", "05", "06", "07", "08", "09", "10", "11"]
    assert run_layer(2048, objs, graph=True) < 1e-2


def _tp_rank(rank, world, port, q, T, chunks=0):
    import datetime
    import sys
    root = os.path.dirname(HERE)
    sys.path[:0] = [os.path.join(root, "pytorchsim-triton-backend_b200"), root]
    import torch.distributed as dist
    from oracle import programs as O2
    from pytorchsim_triton_compiler.runtime import qwen3 as Q2
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        p = Q2.random_params(0)
        x = torch.randn(T * Q2.HIDDEN, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
        cos, sin = O2.rope_tables(T)
        if chunks:
            layer = Q2.TpLayer(f"cuda:{rank}", T, Q2.shard(p, rank, world), cos, sin, x, world, rank, chunks=chunks)
            layer.capture()
            layer.run(dist.all_reduce)
            buffers = layer.buffers
        else:
            g1, g2 = Q2.build_layer(f"cuda:{rank}", T, Q2.shard(p, rank, world), cos, sin, x, tp=world, rank=rank)
            g1.run()
            dist.all_reduce(g1.buffers["x1"])
            g2.run()
            dist.all_reduce(g1.buffers["y"])
            buffers = g1.buffers
        torch.cuda.synchronize()
        if rank == 0:
            want = O2.decoder_layer(x, p, T, cos=cos, sin=sin).float()
            got = buffers["y"].float().cpu()
            q.put((rank, float((got - want).norm() / want.norm())))
        else:
            q.put((rank, None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="tensor parallel needs two GPUs")
@pytest.mark.parametrize("chunks", [0, 2, 4])
def test_layer_tp2_nccl(chunks):
    """The layer over two GPUs: serial all-reduces (chunks 0), or the o projection and the MLP in row blocks
    whose all-reduces overlap the next block's compute (runtime/qwen3.py TpLayer)."""
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_tp_rank, args=(r, 2, port, q, 256, chunks)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    assert isinstance(got[0], float) and got[0] < 1e-2, got
