"""Request-level data parallelism across the GPUs of one box.

Requests are independent and every estimator layer is row-local except
attention, which stays inside a document; so requests are partitioned into
per-GPU bins and each rank runs its own packed estimator on a full weight
replica.  No collective runs on the hot path.  A CFG pair (a request's
conditional and unconditional rows) always stays on one rank, because the CFG
combine needs both (``flashinfer_flow.py:66-69``).

Bins are balanced by the estimator's algorithmic cost per request,
``2 * (a*L + b*P(L))`` with ``a`` the per-row FLOPs and ``b*P`` the attention
FLOPs over the visible (query, key) pairs -- longest-processing-time-first
(LPT) greedy assignment.
"""

from __future__ import annotations

from typing import Sequence

from .flops import PAIR_FLOPS, ROW_FLOPS, visible_pairs


def request_cost(L: int, chunk: int | None = None) -> int:
    """Estimator FLOPs of one request's CFG pair (two rows of length L)."""
    return 2 * (L * ROW_FLOPS + 22 * PAIR_FLOPS * visible_pairs([L], chunk))


def lpt_bins(lengths: Sequence[int], n_bins: int, chunk: int | None = None) -> list[list[int]]:
    """Assign request indices to ``n_bins`` bins, most expensive first, each to
    the currently lightest bin (ties: lowest bin index).  Deterministic."""
    if n_bins < 1:
        raise ValueError("n_bins must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-request_cost(int(lengths[i]), chunk), i))
    loads = [0] * n_bins
    bins: list[list[int]] = [[] for _ in range(n_bins)]
    for i in order:
        b = min(range(n_bins), key=lambda k: (loads[k], k))
        bins[b].append(i)
        loads[b] += request_cost(int(lengths[i]), chunk)
    for b in bins:
        b.sort()
    return bins


def bin_loads(lengths: Sequence[int], bins: list[list[int]], chunk: int | None = None) -> list[int]:
    return [sum(request_cost(int(lengths[i]), chunk) for i in b) for b in bins]


class ShardError(RuntimeError):
    """Raised on every rank when the estimator failed on at least one rank."""

    def __init__(self, failures: dict):
        super().__init__("estimator failed on rank(s) " + ", ".join(f"{r}: {m}" for r, m in sorted(failures.items())))
        self.failures = failures


def run_sharded(lengths: Sequence[int], run_local, group=None, chunk: int | None = None):
    """Run requests across the ranks of ``group`` and return every request's
    result, in request order, on every rank.

    ``run_local(indices)`` runs the estimator (or a whole ODE) on this rank for
    the request indices of its LPT bin and returns one result per index.  A
    failure on any rank is reported to all ranks as :class:`ShardError` after
    the exchange (no rank is left waiting), mirroring the reference batcher,
    which fails the whole packed batch and keeps serving
    (``token2wav_batcher.py:163-179``).  Only the host-side result exchange is
    a collective; the estimator itself never communicates.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bins = lpt_bins(lengths, world, chunk)
    mine = bins[rank]
    try:
        res = list(run_local(mine))
        if len(res) != len(mine):
            raise RuntimeError(f"run_local returned {len(res)} results for {len(mine)} requests")
        payload = ("ok", mine, res)
    except Exception as exc:  # reported to every rank below
        payload = ("err", mine, f"{type(exc).__name__}: {exc}")
    gathered = [None] * world
    dist.all_gather_object(gathered, payload, group=group)
    failures = {r: p[2] for r, p in enumerate(gathered) if p[0] != "ok"}
    if failures:
        raise ShardError(failures)
    out = [None] * len(lengths)
    for _, idx, res in gathered:
        for i, r in zip(idx, res):
            out[i] = r
    return out
