"""Data-parallel placement of independent utterances over GPUs.

T3 streams share nothing, so a multi-GPU job is a set of replicas: each rank
(one process per GPU) decodes its own streams and no tensor crosses GPUs.
The only host logic is (1) which streams go to which rank and (2) how the
ranks' device times combine into one job time.

Decode cost per step is dominated, for batched decode, by reading each row's
K/V cache (98 304 B per cached position for T3), so streams are placed by
expected context length, longest first, onto the least-loaded rank
(greedy LPT) rather than by count.
"""


def stream_cost(prompt_len, decode_len, cfg=False):
    """Relative per-utterance cost: sum over its decode steps of the positions
    read, times the rows per stream (2 with CFG)."""
    rows = 2 if cfg else 1
    return rows * (decode_len * prompt_len + decode_len * (decode_len + 1) // 2)


def assign_streams(costs, world):
    """Greedy longest-processing-time placement: returns, for every rank, the
    list of stream indices it owns (each list in ascending order)."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0.0] * world
    owned = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        owned[r].append(i)
        load[r] += costs[i]
    return [sorted(o) for o in owned]


def job_throughput(dist, local_ms, units, world):
    """Whole-job units/s: every rank's device time is max-reduced (the job
    ends when the slowest rank does) and all ranks' units are counted.
    `dist` is torch.distributed (or None for one process); `units` is this
    rank's unit count."""
    import torch
    t = torch.tensor([float(local_ms), float(units)], dtype=torch.float64)
    if dist is not None and world > 1:
        dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
        t = t.to(dev)
        tm = t[:1].clone()
        un = t[1:].clone()
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        dist.all_reduce(un, op=dist.ReduceOp.SUM)
        ms, total = float(tm.item()), float(un.item())
    else:
        ms, total = float(t[0]), float(t[1])
    return total / (ms / 1000.0), ms
