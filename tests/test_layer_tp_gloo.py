"""Tensor-parallel split of the Qwen3-8B-shaped layer, host logic on CPU ranks (gloo, world size 2): each
rank runs its shard (runtime/qwen3.py shard: column-split q/k/v/gate_up, row-split o/down) through the
oracle's restatement of the layer's launches, partial o/down outputs are all-reduced (rank 0 alone adds the
residual), and the result matches the whole layer within the bf16 tolerance, measured as relative L2
error (each partial is rounded to bf16 before the sum, as the GPU path's NCCL all-reduce of bf16 does)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

T = 16


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "pytorchsim-triton-backend_b200"), root]
    from oracle import programs as O
    from pytorchsim_triton_compiler.runtime import qwen3 as Q
    torch.set_num_threads(2)
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        p = Q.random_params(0)
        x = torch.randn(T * Q.HIDDEN, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
        cos, sin = O.rope_tables(T)
        ps = Q.shard(p, rank, world)
        x1 = O.layer_attention_half(x, ps, T, Q.HQ // world, Q.HKV // world, rank == 0, cos=cos, sin=sin)
        x1f = x1.float()
        dist.all_reduce(x1f)
        x1 = x1f.to(torch.bfloat16)
        y = O.layer_mlp_half(x1, ps, T, Q.INTER // world, rank == 0).float()
        dist.all_reduce(y)
        if rank == 0:
            want = O.decoder_layer(x, p, T, cos=cos, sin=sin).float()
            rel = float((y - want).norm() / want.norm())
            q.put((rank, rel))
        else:
            q.put((rank, None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_tp2_layer_matches_the_whole_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    assert isinstance(got[0], float), got
    assert got[0] < 1e-2, got
