"""Algorithmic FLOP model of one estimator call (used for roofline reporting).

Per packed row: 22 blocks x (QKV 6.29 M + out-proj 2.10 M + FF 8.39 M) = 22 * 2^24,
plus input projection 0.66 M, two grouped causal convolutions 8.13 M and
proj_out 0.16 M -> 378,044,416 FLOPs.  Attention: 4 * heads * head_dim = 4096
FLOPs per visible (query, key) pair and block.  Per sequence: the fused AdaLN
projection (1024 -> 22*6144 + 2048) and the time MLP.
"""

from __future__ import annotations

from typing import Sequence

ROW_FLOPS = 22 * 2 ** 24 + 2 * 320 * 1024 + 2 * 2 * 1024 * 31 * 64 + 2 * 1024 * 80
GEMM_ROW_FLOPS = 22 * 2 ** 24
PAIR_FLOPS = 4 * 16 * 64
SEQ_FLOPS = 2 * 1024 * (22 * 6144 + 2048) + 2 * (256 * 1024 + 1024 * 1024)


def visible_pairs(lengths: Sequence[int], chunk: int | None) -> int:
    """Visible (q, k) pairs: sum L^2 (full mask) or, with chunk C,
    sum_q min(L, (q // C + 1) * C)."""
    total = 0
    for L in lengths:
        L = int(L)
        if not chunk:
            total += L * L
        else:
            for q0 in range(0, L, chunk):
                total += min(chunk, L - q0) * min(L, q0 + chunk)
    return total


def estimator_flops(lengths: Sequence[int], chunk: int | None, depth: int = 22) -> int:
    N = sum(int(L) for L in lengths)
    per_row = depth * 2 ** 24 + (ROW_FLOPS - GEMM_ROW_FLOPS)
    seq = 2 * 1024 * (depth * 6144 + 2048) + 2 * (256 * 1024 + 1024 * 1024)
    return N * per_row + depth * PAIR_FLOPS * visible_pairs(lengths, chunk) + len(lengths) * seq
