"""The analytic work model restates the reference benchmark's
(tests/test_benchmark_model.py:1-42 of the reference)."""

from triton_flash_attention_b200 import attention_flops, delta_bytes, memory_model


def test_causal_forward_counts_only_visible_pairs():
    assert attention_flops(batch=1, query_heads=1, sequence=4, head_dim=8, causal=True,
                           mode="forward") == 4 * 10 * 8


def test_backward_is_two_and_a_half_forward_passes():
    fwd = attention_flops(batch=2, query_heads=4, sequence=16, head_dim=32, causal=False, mode="forward")
    bwd = attention_flops(batch=2, query_heads=4, sequence=16, head_dim=32, causal=False, mode="backward")
    assert bwd == int(2.5 * fwd)


def test_metric_shape_total():
    """C2: B4 H16 N4096 D64 causal fwd+bwd = 4.8115e11 FLOP."""
    total = attention_flops(batch=4, query_heads=16, sequence=4096, head_dim=64, causal=True,
                            mode="forward-backward")
    assert abs(total - 4.8115e11) / 4.8115e11 < 1e-4


def test_memory_model_is_linear_for_saved_lse():
    small = memory_model(batch=1, query_heads=1, sequence=128)
    large = memory_model(batch=1, query_heads=1, sequence=256)
    assert large["saved_lse_mib"] == 2 * small["saved_lse_mib"]
    assert large["naive_score_mib"] == 4 * small["naive_score_mib"]


def test_delta_bytes():
    assert delta_bytes(batch=4, heads=16, sequence=4096, head_dim=64) == 4 * 16 * 4096 * (64 * 4 + 4)
