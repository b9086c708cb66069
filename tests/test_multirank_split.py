"""The multi-GPU partition on CPU ranks (gloo, world size 2): each rank takes its unit range (runtime/cuda.py
split, the edges of the reference's spike._split, runtime/spike.py:253-258), computes only those units with a
stand-in executor, and the ranks' written bytes -- gathered -- merge (runtime/cuda.py merge, the reference's
merge_worker_outputs, spike.py:310-334) into exactly what one rank computing every unit writes.  A rank that
raises makes the launch fail on every rank (a short process-group timeout, no hang)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROWS, COLS = 64, 256


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _units_softmax(x, lo, hi, out):
    """Stand-in executor: units are rows; the oracle's softmax for rows [lo, hi) only."""
    from oracle import programs as O
    if hi > lo:
        out[lo * COLS:hi * COLS] = O.softmax_rows(x[lo * COLS:hi * COLS], hi - lo, COLS)


def _worker(rank, world, port, fail_rank, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "pytorchsim-triton-backend_b200"), root]
    from pytorchsim_triton_compiler.runtime import cuda as RC
    import datetime
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(ROWS * COLS, generator=g).to(torch.bfloat16)
        mine = torch.zeros_like(x)
        lo, hi = RC.split(ROWS, world)[rank]
        if rank == fail_rank:
            raise RuntimeError("planted failure on this rank")
        _units_softmax(x, lo, hi, mine)
        parts = [torch.zeros(ROWS * COLS * 2, dtype=torch.uint8) for _ in range(world)]
        dist.all_gather(parts, mine.view(torch.uint8))
        manifest = {"args": [{"name": "o", "role": "out", "dtype": "bfloat16", "shape": [ROWS * COLS]}]}
        base = {"o": np.zeros(ROWS * COLS * 2, dtype=np.uint8)}
        merged = RC.merge(manifest, base, [{"o": p.numpy()} for p in parts])["o"]
        whole = torch.zeros_like(x)
        _units_softmax(x, 0, ROWS, whole)
        q.put((rank, bool(np.array_equal(merged, whole.view(torch.uint8).numpy())), None))
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        q.put((rank, False, f"{type(e).__name__}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out)


def test_two_ranks_merge_to_the_whole():
    got = _run(2)
    assert [ok for _, ok, _ in got] == [True, True], got


def test_a_failing_rank_fails_the_launch_everywhere():
    got = _run(2, fail_rank=1)
    assert not any(ok for _, ok, _ in got), got
    assert any("planted failure" in (err or "") for _, _, err in got)
