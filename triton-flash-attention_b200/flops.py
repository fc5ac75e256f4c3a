"""Analytic work model of the attention path.

Restates the reference benchmark's definitions so that throughput figures
use the same convention (benchmarks/benchmark_attention.py:36-71).
"""

from __future__ import annotations


def attention_flops(*, batch: int, query_heads: int, sequence: int, head_dim: int,
                    causal: bool, mode: str) -> int:
    """Algorithmic FLOPs (benchmark_attention.py:36-54).

    Causal attention counts the N(N+1)/2 visible (query, key) pairs, full
    attention N^2; the forward costs 4 * B * Hq * pairs * D (two GEMMs), the
    backward 2.5x the forward and forward+backward 3.5x."""
    pairs = sequence * (sequence + 1) // 2 if causal else sequence * sequence
    forward = 4 * batch * query_heads * pairs * head_dim
    if mode == "forward":
        return forward
    if mode == "backward":
        return int(2.5 * forward)
    if mode == "forward-backward":
        return int(3.5 * forward)
    raise ValueError(f"unknown mode: {mode}")


def memory_model(*, batch: int, query_heads: int, sequence: int, element_size: int = 2) -> dict[str, float]:
    """One materialised score matrix versus the saved LSE vector, in MiB
    (benchmark_attention.py:57-71)."""
    mib = 1024 ** 2
    return {
        "naive_score_mib": batch * query_heads * sequence * sequence * element_size / mib,
        "saved_lse_mib": batch * query_heads * sequence * 4 / mib,
    }


def delta_bytes(*, batch: int, heads: int, sequence: int, head_dim: int) -> int:
    """Bytes the Delta preprocess must move: read O and dO (fp16), write
    Delta (fp32) -- the HBM roofline of that kernel."""
    rows = batch * heads * sequence
    return rows * head_dim * 2 * 2 + rows * 4
