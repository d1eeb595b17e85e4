"""Layer-interval partitioning of a decoder into contiguous pipeline stages.

* ``equal_ranges`` - layer counts differ by at most one;
* ``balanced_ranges`` - minimise the largest per-stage cost (layer cost may
  differ, e.g. dense first layers of DeepSeek-V3) subject to a per-stage
  memory cap, by dynamic programming over prefix sums (exact minimax);
* ``ranges_for_capacities`` - heterogeneous stages: binary search on the
  bottleneck time with each stage's own throughput and memory capacity.

Every layer is assigned exactly once, in order (checked by property tests).

Reference: si/model/partition.py:274-356 and the exact-stage-count search of
si/model/shard_builder.py:306-406.
"""
from __future__ import annotations

from typing import Sequence


class PartitionError(ValueError):
    pass


def equal_ranges(num_layers: int, stages: int) -> list[tuple[int, int]]:
    if stages <= 0 or num_layers < stages:
        raise PartitionError(f"cannot split {num_layers} layers into {stages} stages")
    base, rem = divmod(num_layers, stages)
    out, s = [], 0
    for i in range(stages):
        n = base + (1 if i < rem else 0)
        out.append((s, s + n))
        s += n
    return out


def balanced_ranges(costs: Sequence[float], stages: int, *, mem: Sequence[float] | None = None,
                    mem_cap: float | None = None) -> list[tuple[int, int]]:
    """Contiguous split of ``costs`` into ``stages`` non-empty parts minimising the max part
    cost; parts whose memory exceeds ``mem_cap`` are forbidden."""
    n = len(costs)
    if stages <= 0 or n < stages:
        raise PartitionError(f"cannot split {n} layers into {stages} stages")
    pc = [0.0]
    for c in costs:
        pc.append(pc[-1] + float(c))
    pm = [0.0]
    for m in (mem if mem is not None else [0.0] * n):
        pm.append(pm[-1] + float(m))
    INF = float("inf")

    def ok(i, j):
        return mem_cap is None or pm[j] - pm[i] <= mem_cap + 1e-9

    # best[k][j]: minimal max-cost splitting the first j layers into k stages
    best = [[INF] * (n + 1) for _ in range(stages + 1)]
    arg = [[-1] * (n + 1) for _ in range(stages + 1)]
    best[0][0] = 0.0
    for k in range(1, stages + 1):
        for j in range(k, n - (stages - k) + 1):
            for i in range(k - 1, j):
                if best[k - 1][i] == INF or not ok(i, j):
                    continue
                v = max(best[k - 1][i], pc[j] - pc[i])
                if v < best[k][j] - 1e-12:
                    best[k][j] = v
                    arg[k][j] = i
    if best[stages][n] == INF:
        raise PartitionError("no split satisfies the per-stage memory cap")
    out = []
    j = n
    for k in range(stages, 0, -1):
        i = arg[k][j]
        out.append((i, j))
        j = i
    return out[::-1]


def ranges_for_capacities(costs: Sequence[float], throughput: Sequence[float],
                          memory: Sequence[float], layer_mem: Sequence[float]) -> list[tuple[int, int]]:
    """Heterogeneous stages (in ring order): stage s runs at ``throughput[s]`` cost units/s
    and holds ``memory[s]`` bytes.  Minimises the bottleneck stage time."""
    n, S = len(costs), len(throughput)
    if n < S:
        raise PartitionError("fewer layers than stages")

    def feasible(t):
        out, i = [], 0
        for s in range(S):
            j, c, m = i, 0.0, 0.0
            left_stages = S - s - 1
            while j < n - left_stages and c + costs[j] <= t * throughput[s] + 1e-12 \
                    and m + layer_mem[j] <= memory[s]:
                c += costs[j]
                m += layer_mem[j]
                j += 1
            if j == i:
                return None
            out.append((i, j))
            i = j
        return out if i == n else None

    lo, hi = 0.0, sum(costs) / min(throughput) + 1.0
    if feasible(hi) is None:
        raise PartitionError("model does not fit the stages' memory")
    for _ in range(60):
        mid = (lo + hi) / 2
        if feasible(mid) is None:
            lo = mid
        else:
            hi = mid
    return feasible(hi)
