"""The tensor-parallel all-reduce over NVLink peer memory (ptsim_tp_allreduce, csrc/collective.cuh), on 2, 4 and 8
GPUs, one process each (each size skipped with fewer GPUs):

  - the kernel alone: every rank's output equals bf16 of the fp32 sum of all ranks' bf16 partials in rank order,
    bit for bit, on four calls in a row of different shapes with new partials each time (the generation counter
    runs on, the done count starts from zero each call);
  - the Qwen3-shaped layer split over the GPUs with both all-reduces done by the executor's kernels
    (runtime/qwen3.py TpLayerPeer, replayed from CUDA graphs), in both forms -- one all-reduce kernel over the
    partials, and the GEMM pushing its rows to their owners (ptsim_launch_rows_to_owners) followed by
    ptsim_tp_reduce_gather -- gives the same bits either way and matches the whole layer within the bf16 bar."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port):
    import sys
    root = os.path.dirname(HERE)
    sys.path[:0] = [os.path.join(root, "pytorchsim-triton-backend_b200"), root]
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


# Calls in a row on one signal block, with shapes whose grids differ (over two ranks: 64, 2, 64 and 1 CTAs).
SHAPES = [(512, 4096), (64, 1024), (512, 4096), (8, 24)]


def _allreduce_rank(rank, world, port, q):
    dist = _setup(rank, world, port)
    try:
        from pytorchsim_triton_compiler.runtime import native
        from pytorchsim_triton_compiler.runtime.peer import PeerSet
        native.init(rank)
        peers = PeerSet(f"cuda:{rank}", world, rank)
        part_all, pp = peers.alloc("part", 512 * 4096)
        out_all, po = peers.alloc("out", 512 * 4096)
        _, ps = peers.alloc("sig", 64, "int32")
        bad = []
        for call, (rows, cols) in enumerate(SHAPES):
            part, out = part_all[:rows * cols], out_all[:rows * cols]
            mine = [torch.randn(rows * cols, generator=torch.Generator().manual_seed(100 * call + r)).to(torch.bfloat16)
                    for r in range(world)]
            part.copy_(mine[rank])
            torch.cuda.synchronize()
            dist.barrier()
            native.tp_allreduce(pp, po, ps, rank, rows, cols, torch.cuda.current_stream().cuda_stream)
            native.sync(torch.cuda.current_stream().cuda_stream)
            acc = torch.zeros(rows * cols)
            for r in range(world):
                acc = acc + mine[r].float()
            want = acc.to(torch.bfloat16)
            if not torch.equal(out.cpu().view(torch.int16), want.view(torch.int16)):
                bad.append(call)
            dist.barrier()
        peers.close()
        q.put((rank, bad))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def _layer_rank(rank, world, port, q, T):
    dist = _setup(rank, world, port)
    try:
        from oracle import programs as O
        from pytorchsim_triton_compiler.runtime import native
        from pytorchsim_triton_compiler.runtime import qwen3 as Q
        native.init(rank)
        p = Q.random_params(0)
        x = torch.randn(T * Q.HIDDEN, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
        cos, sin = O.rope_tables(T)
        got = {}
        for fused in (False, True):
            layer = Q.TpLayerPeer(f"cuda:{rank}", T, Q.shard(p, rank, world), cos, sin, x, world, rank, fused=fused)
            layer.capture()
            for _ in range(2):                  # twice: the second replays the graphs on the advanced generation
                layer.run()
            native.sync(torch.cuda.current_stream().cuda_stream)   # raises on a device-side timeout
            got[fused] = layer.buffers["y"].cpu()
            layer.close()
        same = torch.equal(got[False].view(torch.int16), got[True].view(torch.int16))
        if rank == 0:
            want = O.decoder_layer(x, p, T, cos=cos, sin=sin).float()
            q.put((rank, (float((got[True].float() - want).norm() / want.norm()), same)))
        else:
            q.put((rank, (None, same)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def _spawn(world, target, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    return got


WORLDS = [pytest.param(w, marks=pytest.mark.skipif(torch.cuda.device_count() < w, reason=f"needs {w} GPUs"))
          for w in (2, 4, 8)]


@pytest.mark.parametrize("world", WORLDS)
def test_peer_allreduce_bit_exact(world):
    got = _spawn(world, _allreduce_rank)
    assert all(got[r] == [] for r in range(world)), got


@pytest.mark.parametrize("world", WORLDS)
def test_layer_tp_peer_allreduce(world):
    """Both forms (pull, and the GEMM pushing its rows to their owners) give the same bits on every rank, and the
    layer matches the one-GPU oracle within the bf16 bar."""
    got = _spawn(world, _layer_rank, 256)
    assert all(isinstance(v, tuple) for v in got.values()), got
    assert all(got[r][1] for r in range(world)), got
    assert got[0][0] < 1e-2, got
