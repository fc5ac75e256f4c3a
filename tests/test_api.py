"""API contract of the drop-in surface (CPU; no GPU needed).

Ports the reference's API tests (tests/test_api.py:47-109) to this build's
dispatch rule: the same validation messages, and -- where the reference
falls back to PyTorch SDPA -- a RuntimeError naming the reason, because this
package has no fallback."""

from __future__ import annotations

import pytest
import torch

import triton_flash_attention_b200 as fa
from triton_flash_attention_b200 import DispatchDecision, explain_dispatch, scaled_dot_product_attention


def test_exports_match_reference_names():
    for name in ("DispatchDecision", "TritonAttention", "explain_dispatch", "scaled_dot_product_attention"):
        assert hasattr(fa, name)
    assert fa.TritonAttention is fa.B200Attention


def test_dispatch_explains_ineligible_device():
    tensor = torch.randn(1, 1, 3, 32)
    assert explain_dispatch(tensor, tensor, tensor) == DispatchDecision(
        backend="unsupported", reason="the B200 kernel requires a CUDA tensor")


@pytest.mark.parametrize("backend", ["auto", "triton", "cuda"])
def test_ineligible_device_raises_instead_of_falling_back(backend):
    tensor = torch.randn(1, 1, 3, 32)
    with pytest.raises(RuntimeError, match="requires a CUDA tensor"):
        scaled_dot_product_attention(tensor, tensor, tensor, backend=backend)


def test_torch_backend_is_not_provided():
    tensor = torch.randn(1, 1, 3, 32)
    with pytest.raises(RuntimeError, match="not part of this package"):
        scaled_dot_product_attention(tensor, tensor, tensor, backend="torch")


def test_unknown_backend():
    tensor = torch.randn(1, 1, 3, 32)
    with pytest.raises(ValueError, match="backend must be one of"):
        scaled_dot_product_attention(tensor, tensor, tensor, backend="xla")


@pytest.mark.parametrize(
    ("mutator", "message"),
    [
        (lambda q, k, v: (q.squeeze(0), k, v), "query must have shape"),
        (lambda q, k, v: (q[..., :-1], k, v), "query and key head dimensions"),
        (lambda q, k, v: (q, k[:, :1], v[:, :1]), "pass enable_gqa=True"),
        (lambda q, k, v: (q, k, v[:, :, :-1]), "key and value batch, head, and sequence"),
        (lambda q, k, v: (q, k.double(), v), "same dtype"),
        (lambda q, k, v: (q[:, :, :0], k, v), "greater than zero"),
        (lambda q, k, v: (q, k.expand(2, -1, -1, -1), v.expand(2, -1, -1, -1)), "batch dimensions must match"),
    ],
)
def test_validation_errors(mutator, message):
    """Messages pinned by the reference (tests/test_api.py:61-85)."""
    query = torch.randn(1, 2, 5, 32)
    key = torch.randn_like(query)
    value = torch.randn_like(query)
    query, key, value = mutator(query, key, value)
    with pytest.raises(ValueError, match=message):
        scaled_dot_product_attention(query, key, value)


def test_gqa_divisibility():
    q = torch.randn(1, 3, 5, 32)
    k = torch.randn(1, 2, 5, 32)
    with pytest.raises(ValueError, match="divisible"):
        scaled_dot_product_attention(q, k, k, enable_gqa=True)


def test_type_errors():
    t = torch.randn(1, 1, 3, 32)
    with pytest.raises(TypeError, match="must be a torch.Tensor"):
        explain_dispatch(t.numpy(), t, t)
    with pytest.raises(TypeError, match="is_causal must be a bool"):
        scaled_dot_product_attention(t, t, t, is_causal=1)
    with pytest.raises(TypeError, match="enable_gqa must be a bool"):
        scaled_dot_product_attention(t, t, t, enable_gqa=0)
    with pytest.raises(ValueError, match="scale must be a finite"):
        scaled_dot_product_attention(t, t, t, scale=float("nan"))


def test_value_head_size_reasons(monkeypatch):
    """A value head size different from the query/key one is served (the
    reference sends it to PyTorch, attention.py:639-646) when both are 32, 64
    or 128; other value head sizes get their own reason.  Checked with the
    device test bypassed (no GPU here)."""
    class FakeDevice:
        type = "cuda"

    query = torch.randn(1, 2, 3, 32).half()
    key = torch.randn(1, 2, 5, 32).half()
    fake = FakeDevice()
    monkeypatch.setattr(torch.Tensor, "device", property(lambda self: fake), raising=False)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda device=None: (10, 0))
    decision = explain_dispatch(query, key, torch.randn(1, 2, 5, 16).half())
    assert decision.backend == "unsupported"
    assert "value head_dim must be one of (32, 64, 128)" in decision.reason
    decision = explain_dispatch(query, key, torch.randn(1, 2, 5, 128).half())
    assert decision.backend == "cuda"


def test_dtype_and_head_dim_reasons(monkeypatch):
    """Reasons for fp32 inputs and unsupported head dims, checked with the
    device test bypassed (no GPU here)."""
    class FakeDevice:
        type = "cuda"

    q32 = torch.randn(1, 1, 4, 32)
    q48 = torch.randn(1, 1, 4, 48).half()
    fake = FakeDevice()
    monkeypatch.setattr(torch.Tensor, "device", property(lambda self: fake), raising=False)
    assert "float16" in explain_dispatch(q32, q32, q32).reason
    assert "head_dim must be one of (32, 64, 128)" in explain_dispatch(q48, q48, q48).reason
