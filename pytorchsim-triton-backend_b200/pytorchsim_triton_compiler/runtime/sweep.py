"""A sweep's independent points (kernel objects of one sweep, e.g. the GEMM M sweep at N = K = 4096) spread over
the ranks of a job, one GPU each, with no collective: the way the reference spreads a sweep's shapes over its pool
(validation/gemm/simulate_shapes.py:171-193, `cost` / `longest_first` / `shard`).

A point's cost is what it is ranked by: for a GEMM the product M * N * K (the reference's product of a shape's
numbers), for attention its flops, for any other program the bytes of its arguments.  Points go costliest first,
ties broken by the point's key (a GEMM's (M, K, N), the reference's key order; else its name); each goes to the
rank whose points cost least so far, ties to the lower rank (longest processing time).  Every rank computes the
same assignment from the same list, so the shards are disjoint, cover the sweep and need no exchange."""
import math

from ..codegen import descriptors as D

# Bytes per element of each descriptor dtype code (PTSIM_DT_*).
_ITEMSIZE = {0: 4, 1: 2, 2: 2, 3: 4, 4: 8, 5: 2, 6: 1, 7: 1, 8: 8}


class Point:
    """One sweep point: a kernel object's name and descriptor blob, with its cost and tie-break key (both derived
    from the descriptor unless given; a point without a blob must give both).  The points of one sweep share a
    cost unit: one kind of program."""

    def __init__(self, name, blob=None, cost=None, key=None):
        self.name, self.blob = name, (bytes(blob) if blob is not None else None)
        if blob is None:
            if cost is None or key is None:
                raise ValueError(f"sweep point {name}: without a descriptor, give its cost and key")
            self.cost, self.key = int(cost), tuple(key)
            return
        d = D.from_bytes(self.blob)
        if d.kind == D.GEMM:
            g = d.p.gemm
            self.cost = g.M * g.N * g.K
            self.key = (g.M, g.K, g.N)
        elif d.kind == D.ATTN_PREFILL:
            a = d.p.attn
            full = 4 * a.batch * a.hq * a.seq * a.seq * a.dim
            self.cost = full // 2 if a.causal else full
            self.key = (name,)
        else:
            self.cost = sum(int(d.arg_numel[i]) * _ITEMSIZE[int(d.arg_dtype[i])] for i in range(d.nargs))
            self.key = (name,)
        if cost is not None:
            self.cost = int(cost)
        if key is not None:
            self.key = tuple(key)

    def __repr__(self):
        return f"Point({self.name}, cost={self.cost})"


def longest_first(points):
    """The points by cost, largest first, ties in key order."""
    return sorted(points, key=lambda p: (-p.cost, p.key))


def assign(points, world):
    """The rank of every point (a list parallel to longest_first(points)) and each rank's total cost."""
    if world < 1:
        raise ValueError(f"a sweep over {world} ranks")
    load, ranks = [0] * world, []
    for p in longest_first(points):
        r = min(range(world), key=lambda j: (load[j], j))
        load[r] += p.cost
        ranks.append(r)
    return ranks, load


def shard(points, rank, world):
    """Rank `rank`'s points of `world`, costliest first."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    ranks, _ = assign(points, world)
    return [p for p, r in zip(longest_first(points), ranks) if r == rank]


def balance(points, world):
    """The largest rank's cost over the mean: 1.0 is a perfect split (a single point costlier than the mean
    bounds it from below)."""
    _, load = assign(points, world)
    mean = sum(load) / world
    return max(load) / mean if mean > 0 else 1.0


def lower_bound(points, world):
    """No split can finish before its costliest point or before the mean load: the larger of the two."""
    if not points:
        return 0
    return max(max(p.cost for p in points), math.ceil(sum(p.cost for p in points) / world))
