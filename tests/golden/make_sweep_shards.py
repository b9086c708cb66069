"""Generate tests/golden/sweep_shards.json: how the reference spreads a sweep's shapes over a pool of n parts
(validation/gemm/simulate_shapes.py `shard`, by longest processing time), for n = 1..8, on three shape lists: the
GEMM M sweep at N = K = 4096, a list with equal costs (the tie-breaking), and 24 mixed GEMM shapes.  The reference
is imported from the checkout PTSIM_REFERENCE names; runtime/sweep.py restates `shard`, and
tests/test_sweep.py checks the restatement against this file.

    PTSIM_REFERENCE=<reference checkout> python tests/golden/make_sweep_shards.py"""
import json
import os
import sys

REF = os.environ.get("PTSIM_REFERENCE", "")
if not REF or not os.path.isdir(REF):
    raise SystemExit("set PTSIM_REFERENCE to the reference checkout (the PyTorchSim-Triton-Backend source tree)")
sys.path.insert(0, os.path.join(REF, "validation", "gemm"))
import simulate_shapes as S  # noqa: E402

LISTS = {
    "gemm_m_sweep": [(m, 4096, 4096) for m in (128, 512, 2048, 4096, 8192)],
    "ties": [(4096, 4096, 2048), (2048, 4096, 4096), (4096, 2048, 4096), (1024, 1024, 1024), (512, 2048, 1024),
             (1024, 512, 2048), (2048, 1024, 512), (256, 256, 256)],
    "mixed": [(m, k, n) for m in (128, 1024, 4096) for k in (768, 4096) for n in (768, 2048, 4096, 12288)],
}


def main():
    out = {"source": "validation/gemm/simulate_shapes.py shard (KEYS M, K, N; cost M * K * N)", "lists": {}}
    for name, shapes in LISTS.items():
        rows = [{"M": m, "K": k, "N": n} for m, k, n in shapes]
        out["lists"][name] = {
            "shapes": [list(s) for s in shapes],
            "shards": {str(n): [[[r["M"], r["K"], r["N"]] for r in S.shard(rows, p, n, S.KEYS)] for p in range(n)]
                       for n in range(1, 9)},
        }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sweep_shards.json")
    with open(path, "w") as fh:
        json.dump(out, fh, separators=(",", ":"))
    print(path)


if __name__ == "__main__":
    main()
