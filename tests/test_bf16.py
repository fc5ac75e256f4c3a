"""bf16 inputs on the B200 kernels (GPU only).

The reference's kernel path is fp16 only and sends bf16 inputs to PyTorch's
SDPA (triton_flash_attention/attention.py:653-656); this build runs them on
the same kernels with P and dS rounded to bf16.  bf16 carries 8 mantissa bits
against fp16's 11, so the bar is relative to PyTorch's own bf16 SDPA on the
same inputs: this build's max-abs error against float64 attention may be at
most twice PyTorch's bf16 error plus 2e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import triton_flash_attention_b200 as fa
from oracle import fa2_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(b, hq, hkv, nq, nk, d, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(b, hq, nq, d, generator=g).bfloat16()
    k = torch.randn(b, hkv, nk, d, generator=g).bfloat16()
    v = torch.randn(b, hkv, nk, d, generator=g).bfloat16()
    do = torch.randn(b, hq, nq, d, generator=g).bfloat16()
    return q, k, v, do


def _grads(fn, q, k, v, do, causal, **kw):
    qc, kc, vc = (t.cuda().requires_grad_() for t in (q, k, v))
    o = fn(qc, kc, vc, is_causal=causal, enable_gqa=q.shape[1] != k.shape[1], **kw)
    g = torch.autograd.grad(o, (qc, kc, vc), do.cuda())
    torch.cuda.synchronize()
    return [t.detach().float().cpu().numpy() for t in (o, *g)]


def _maxabs(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [32, 64, 128])
@pytest.mark.parametrize("n", [17, 129, 300])
def test_bf16_against_float64(n, d, causal):
    q, k, v, do = _inputs(1, 2, 2, n, n, d, seed=n * 7 + d)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                             scale=d ** -0.5, do=do.float().numpy())
    ours = _grads(fa.scaled_dot_product_attention, q, k, v, do, causal)
    torch_bf16 = _grads(torch.nn.functional.scaled_dot_product_attention, q, k, v, do, causal)
    for name, a, t in zip(("o", "dq", "dk", "dv"), ours, torch_bf16):
        err, terr = _maxabs(a, ref[name]), _maxabs(t, ref[name])
        assert err <= 2 * terr + 2e-3, (name, err, terr)


@pytest.mark.parametrize("hq,hkv", [(4, 2), (8, 2)])
def test_bf16_gqa_cross(hq, hkv):
    q, k, v, do = _inputs(2, hq, hkv, 200, 333, 64, seed=hq)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True,
                             scale=64 ** -0.5, do=do.float().numpy())
    ours = _grads(fa.scaled_dot_product_attention, q, k, v, do, True)
    torch_bf16 = _grads(torch.nn.functional.scaled_dot_product_attention, q, k, v, do, True)
    for name, a, t in zip(("o", "dq", "dk", "dv"), ours, torch_bf16):
        err, terr = _maxabs(a, ref[name]), _maxabs(t, ref[name])
        assert err <= 2 * terr + 2e-3, (name, err, terr)


def test_bf16_full_size_c2_head():
    """C2 shape (B4 H16 N4096 D64 causal) in bf16; two heads checked against
    PyTorch fp32 math, relative to PyTorch's bf16 SDPA error."""
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v, do = (torch.randn(4, 16, 4096, 64, device="cuda", generator=g).bfloat16() for _ in range(4))
    qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))
    o = fa.scaled_dot_product_attention(qc, kc, vc, is_causal=True)
    gq, gk, gv = torch.autograd.grad(o, (qc, kc, vc), do)
    sl = (slice(0, 1), slice(0, 2))
    q32, k32, v32 = (t[sl].float().requires_grad_() for t in (q, k, v))
    o32 = torch.nn.functional.scaled_dot_product_attention(q32, k32, v32, is_causal=True)
    g32 = torch.autograd.grad(o32, (q32, k32, v32), do[sl].float())
    qb, kb, vb = (t[sl].clone().requires_grad_() for t in (q, k, v))
    ob = torch.nn.functional.scaled_dot_product_attention(qb, kb, vb, is_causal=True)
    gb = torch.autograd.grad(ob, (qb, kb, vb), do[sl])
    for ours, ref, tb in zip((o[sl], gq[sl], gk[sl], gv[sl]), (o32, *g32), (ob, *gb)):
        err = float((ours.detach().float() - ref.detach()).abs().max())
        terr = float((tb.detach().float() - ref.detach()).abs().max())
        assert err <= 2 * terr + 2e-3, (err, terr)


def test_bf16_bitwise_determinism(deterministic):
    q, k, v, do = _inputs(1, 8, 2, 500, 500, 64, seed=3)
    a = _grads(fa.scaled_dot_product_attention, q, k, v, do, True)
    b = _grads(fa.scaled_dot_product_attention, q, k, v, do, True)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_bf16_dispatch_reason():
    q = torch.randn(1, 1, 8, 64, device="cuda").bfloat16()
    decision = fa.explain_dispatch(q, q, q)
    assert decision.backend == "cuda" and "bfloat16" in decision.reason
    q32 = q.float()
    assert "float16 and bfloat16" in fa.explain_dispatch(q32, q32, q32).reason
