"""The fused backward (one pass over the key tiles yields dQ, dK and dV;
D = 32, 64 and, with its own kernel, 128) against the separate dQ and dK/dV
kernels and the float64 oracle (GPU only).

dK and dV follow the dK/dV kernel's MMA accumulation order, but the two
kernels split the exponentials differently between MUFU and the FMA-pipe
polynomial (each kernel uses its own measured-fastest split), so single
elements of P and dS may differ by one ulp of the operand type.  dQ is also
summed over key tiles with fp32 reduce-adds in schedule order.  The bars for
all three gradients: max |a - b| <= 1e-3 + 1e-2 |b| for fp16 and
1e-2 + 5e-2 |b| for bf16 (8 mantissa bits); against float64, the fused dQ's
max-abs error may exceed the dQ kernel's by at most 25% plus 5e-4 (fp16) /
4e-3 (bf16), and stays within the parity suite's 1e-2 for fp16.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import triton_flash_attention_b200 as fa
from oracle import fa2_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-2


def _inputs(b, hq, hkv, nq, nk, d, seed, dtype=torch.float16, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = (torch.randn(b, hq, nq, d, generator=g) * scale).to(dtype).cuda()
    k = (torch.randn(b, hkv, nk, d, generator=g) * scale).to(dtype).cuda()
    v = (torch.randn(b, hkv, nk, d, generator=g) * scale).to(dtype).cuda()
    do = torch.randn(b, hq, nq, d, generator=g).to(dtype).cuda()
    return q, k, v, do


def _close_bound(ref, dtype):
    r = ref.float().abs()
    return (1e-3 + 1e-2 * r) if dtype == torch.float16 else (1e-2 + 5e-2 * r)


def _both(q, k, v, do, causal):
    sc = q.shape[-1] ** -0.5
    o, lse = fa.attention_forward(q, k, v, causal, sc)
    fused = fa.attention_backward_fused(q, k, v, o, do, lse, causal, sc)
    delta = fa.attention_delta(o, do)
    dq = fa.attention_backward_dq(q, k, v, do, lse, delta, causal, sc)
    dk, dv = fa.attention_backward_dkdv(q, k, v, do, lse, delta, causal, sc)
    torch.cuda.synchronize()
    return fused, (dq, dk, dv)


CASES = [
    # b, hq, hkv, nq, nk, d, causal
    (1, 2, 2, 17, 17, 64, True),
    (1, 2, 2, 129, 129, 32, False),
    (2, 4, 2, 300, 300, 64, True),
    (1, 8, 2, 257, 257, 64, False),
    (1, 6, 3, 1000, 1000, 32, True),
    (2, 2, 1, 100, 333, 64, True),
    (1, 2, 2, 333, 100, 64, True),
    (1, 4, 4, 2048, 2048, 64, True),
]
# D = 128 (fa_bwd_fused128.cu: 64-query items, dQ^T = K^T dS^T)
CASES_128 = [
    (1, 2, 2, 65, 65, 128, True),
    (2, 4, 2, 300, 300, 128, True),
    (1, 4, 4, 257, 257, 128, False),
    (2, 2, 1, 100, 333, 128, True),
    (1, 2, 2, 333, 100, 128, False),
    (1, 8, 2, 1000, 1000, 128, True),
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", CASES + CASES_128)
def test_fused_matches_separate_kernels(case, dtype):
    b, hq, hkv, nq, nk, d, causal = case
    q, k, v, do = _inputs(b, hq, hkv, nq, nk, d, seed=nq + 3 * nk + d, dtype=dtype)
    (fdq, fdk, fdv), (dq, dk, dv) = _both(q, k, v, do, causal)
    for name, a, ref_t in (("dq", fdq, dq), ("dk", fdk, dk), ("dv", fdv, dv)):
        diff = (a.float() - ref_t.float()).abs()
        assert bool((diff <= _close_bound(ref_t, dtype)).all()), (name, float(diff.max()))
    if nq * hq <= 4096:
        ref = orc.sdpa_reference(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                 causal=causal, scale=d ** -0.5, do=do.float().cpu().numpy())["dq"]
        e_fused = float(np.abs(fdq.float().cpu().numpy().astype(np.float64) - ref).max())
        e_sep = float(np.abs(dq.float().cpu().numpy().astype(np.float64) - ref).max())
        assert e_fused <= 1.25 * e_sep + (5e-4 if dtype == torch.float16 else 4e-3), (e_fused, e_sep)


@pytest.mark.parametrize("case", CASES[:6] + CASES_128[:5])
def test_fused_against_float64(case):
    b, hq, hkv, nq, nk, d, causal = case
    q, k, v, do = _inputs(b, hq, hkv, nq, nk, d, seed=7 * nq + nk)
    sc = d ** -0.5
    o, lse = fa.attention_forward(q, k, v, causal, sc)
    dq, dk, dv = fa.attention_backward_fused(q, k, v, o, do, lse, causal, sc)
    ref = orc.sdpa_reference(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), causal=causal, scale=sc,
                             do=do.cpu().numpy())
    for name, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        err = float(np.abs(t.float().cpu().numpy().astype(np.float64) - ref[name]).max())
        assert err <= GRAD_TOL, (name, err)


def test_api_takes_fused_path_unless_deterministic():
    assert fa.fused_backward_enabled(64) and fa.fused_backward_enabled(32) and fa.fused_backward_enabled(128)
    torch.use_deterministic_algorithms(True)
    try:
        assert not fa.fused_backward_enabled(64) and not fa.fused_backward_enabled(128)
    finally:
        torch.use_deterministic_algorithms(False)


def test_fused_dk_dv_reproducible_dq_close():
    q, k, v, do = _inputs(2, 8, 2, 700, 700, 64, seed=9)
    runs = []
    for _ in range(3):
        qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))
        o = fa.scaled_dot_product_attention(qc, kc, vc, is_causal=True, enable_gqa=True)
        runs.append(torch.autograd.grad(o, (qc, kc, vc), do))
    for dq, dk, dv in runs[1:]:
        assert torch.equal(dk, runs[0][1]) and torch.equal(dv, runs[0][2])
        diff = (dq.float() - runs[0][0].float()).abs()
        assert bool((diff <= _close_bound(runs[0][0], torch.float16)).all())


def test_full_size_c2_against_separate_kernels():
    """The benchmark shape (B4 H16 N4096 D64, causal): fused vs separate."""
    q, k, v, do = _inputs(4, 16, 16, 4096, 4096, 64, seed=1)
    (fdq, fdk, fdv), (dq, dk, dv) = _both(q, k, v, do, True)
    for name, a, ref_t in (("dq", fdq, dq), ("dk", fdk, dk), ("dv", fdv, dv)):
        diff = (a.float() - ref_t.float()).abs()
        assert bool((diff <= 5e-3 + 2e-2 * ref_t.float().abs()).all()), (name, float(diff.max()))
        rel = float(torch.linalg.vector_norm(a.float() - ref_t.float()) / torch.linalg.vector_norm(ref_t.float()))
        assert rel <= 2e-3, (name, rel)
    assert fa._abi.device_status() == 0


def test_full_size_c4_against_separate_kernels():
    """The GQA benchmark shape at D = 128 (C4: N 8191, causal; 8 of its 32
    query heads, 2 K/V heads): fused vs separate."""
    q, k, v, do = _inputs(1, 8, 2, 8191, 8191, 128, seed=4)
    (fdq, fdk, fdv), (dq, dk, dv) = _both(q, k, v, do, True)
    for name, a, ref_t in (("dq", fdq, dq), ("dk", fdk, dk), ("dv", fdv, dv)):
        diff = (a.float() - ref_t.float()).abs()
        assert bool((diff <= 5e-3 + 2e-2 * ref_t.float().abs()).all()), (name, float(diff.max()))
        rel = float(torch.linalg.vector_norm(a.float() - ref_t.float()) / torch.linalg.vector_norm(ref_t.float()))
        assert rel <= 2e-3, (name, rel)
    assert fa._abi.device_status() == 0


def test_fused128_dk_dv_equal_separate_kernel():
    """At D = 128 the fused pass builds P and dS exactly as the dK/dV kernel
    does (same exponentials, same 64-query items in the same order), so its
    dK and dV are bitwise the dK/dV kernel's."""
    q, k, v, do = _inputs(2, 4, 2, 500, 500, 128, seed=21)
    (_, fdk, fdv), (_, dk, dv) = _both(q, k, v, do, True)
    assert torch.equal(fdk, dk) and torch.equal(fdv, dv)
