"""Attention dropout (``dropout_p``).

The reference has none (README.md:93); PyTorch's SDPA semantics are the
model (probabilities dropped at rate p, kept ones scaled by 1 / (1 - p)).
The keep pattern is a stateless hash of (seed, batch * Hq + head, query,
key) that the kernels evaluate (include/fa_b200.h); the oracle restates it
(``dropout_keep_reference``).

CPU tests: the oracle's pattern has the keep rate and independence a
Bernoulli pattern has, repeats for a seed and changes with it; the
oracle's dropout attention equals PyTorch float64 autograd of
(softmax(S) Z r) V with the same pattern; argument checks of the Python API
and the ABI.  GPU tests:
* the kernels' patterns equal the oracle's bit for bit: the forward's read
  out of O with uniform scores and V = I (O[q, k] = Z[q, k] r / Nk), the
  dK/dV kernel's out of dV with dO = I, including query and key indices
  past 2^17;
* parity of forward and backward with the float64 oracle on the same
  pattern (D 32/64/128, causal, GQA, cross-attention, Dv != D, p 0.1 and
  0.5, bf16) at the equal-width tolerances scaled by r;
* one seed gives bitwise the same outputs and gradients twice.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import triton_flash_attention_b200 as fa
from triton_flash_attention_b200 import _abi
from oracle import fa2_oracle as orc

O_TOL = 2e-3
GRAD_TOL = 1e-2


def _maxabs(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


@pytest.mark.parametrize("p", [0.1, 0.5, 0.9])
def test_oracle_pattern_statistics(p):
    keep = orc.dropout_keep_reference(1234, 2, 4, 256, 256, p)
    t, r = orc.dropout_threshold(p)
    n = keep.size
    rate = 1 - t / 256
    sigma = (rate * (1 - rate) / n) ** 0.5
    assert abs(keep.mean() - rate) < 5 * sigma
    # neighbours in the same 2 x 2 block and across blocks are independent
    for a, b in ((keep[..., :, 0::2], keep[..., :, 1::2]), (keep[..., 0::2, :], keep[..., 1::2, :]),
                 (keep[..., :, 1:-1:2], keep[..., :, 2::2])):
        both = (a & b).mean()
        assert abs(both - rate * rate) < 6 * (rate * rate * (1 - rate * rate) / a.size) ** 0.5
    assert abs(r - 1 / (1 - t / 256)) < 1e-12
    assert np.array_equal(keep, orc.dropout_keep_reference(1234, 2, 4, 256, 256, p))
    assert (keep != orc.dropout_keep_reference(1235, 2, 4, 256, 256, p)).mean() > 0.1


def test_oracle_dropout_matches_torch_float64():
    g = torch.Generator().manual_seed(8)
    q, k, v, do = (torch.randn(2, 2, 37, 32, generator=g, dtype=torch.float64) for _ in range(4))
    keep = orc.dropout_keep_reference(99, 2, 2, 37, 37, 0.25)
    t, r = orc.dropout_threshold(0.25)
    ref = orc.sdpa_reference(q.numpy(), k.numpy(), v.numpy(), causal=True, do=do.numpy(), dropout_keep=keep,
                             dropout_scale=r)
    qt, kt, vt = (x.clone().requires_grad_() for x in (q, k, v))
    s = qt @ kt.transpose(-1, -2) * 32 ** -0.5
    s = s.masked_fill(~torch.ones(37, 37, dtype=torch.bool).tril(), float("-inf"))
    o = (torch.softmax(s, dim=-1) * torch.from_numpy(keep) * r) @ vt
    grads = torch.autograd.grad(o, (qt, kt, vt), do)
    for name, x in zip(("o", "dq", "dk", "dv"), (o, *grads)):
        assert _maxabs(x.detach().numpy(), ref[name]) <= 1e-10, name


def test_dropout_argument_checks():
    t = torch.zeros(1, 1, 4, 32, dtype=torch.float16)
    for bad in (1.0, -0.1, float("nan"), True):
        with pytest.raises(ValueError, match="dropout_p must be"):
            fa.scaled_dot_product_attention(t, t, t, dropout_p=bad)
    lib = _abi.lib()
    s = (ctypes.c_int64 * 3)(64 * 64, 64 * 64, 64)
    for p in (0.0, 1.0, -0.5):
        rc = lib.fa_fwd_dropout(16, 16, 16, 16, 16, 1, 1, 1, 64, 64, 64, 64, s, s, s, s, p, 7, 0.125, 0, None)
        assert rc == _abi.FA_ERR_BAD_SHAPE, p
        rc = lib.fa_bwd_dropout(16, 16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 1, 1, 64, 64, 64, 64,
                                s, s, s, s, s, s, s, s, p, 7, 0.125, 0, None)
        assert rc == _abi.FA_ERR_BAD_SHAPE, p


def test_dropout_rate_that_rounds_to_nothing_is_refused():
    """Rates are applied as the nearest multiple of 1/256 (at least 1/256):
    a rate below 1/512 would silently run at 1/256 and is refused."""
    t = torch.zeros(1, 1, 4, 32, dtype=torch.float16)
    for bad in (0.001, 1e-6, 0.999):
        with pytest.raises(ValueError, match="steps of 1/256"):
            fa.scaled_dot_product_attention(t, t, t, dropout_p=bad)


def test_dropout_with_mask_is_refused(monkeypatch):
    """attn_mask and dropout_p together raise before any CUDA call (the
    device checks are faked, no GPU here)."""
    class FakeDevice:
        type = "cuda"

    fake = FakeDevice()
    q = torch.zeros(1, 2, 8, 64, dtype=torch.float16)
    mask = torch.ones(8, 8, dtype=torch.bool)
    monkeypatch.setattr(torch.Tensor, "device", property(lambda self: fake), raising=False)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda device=None: (10, 0))
    with pytest.raises(RuntimeError, match="attn_mask and dropout_p together"):
        fa.scaled_dot_product_attention(q, q, q, attn_mask=mask, dropout_p=0.1)


# ---------------------------------------------------------------------------
# GPU


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,nq", [(2, 3, 256), (1, 1, 2 ** 17 + 256)])
def test_forward_pattern_bitwise(b, h, nq):
    """Q = 0 makes every score 0 (P = 1 / Nk); with V = I (Nk = D = 128),
    O[q, k] = Z[q, k] r / Nk, so O > 0 is the kernel's keep pattern."""
    nk = d = 128
    p, seed = 0.3, 2 ** 40 + 17
    q = torch.zeros(b, h, nq, d, device="cuda", dtype=torch.float16)
    k = torch.zeros(b, h, nk, d, device="cuda", dtype=torch.float16)
    v = torch.eye(nk, d, device="cuda", dtype=torch.float16).expand(b, h, nk, d).contiguous()
    o, _ = fa.attention_forward_dropout(q, k, v, False, 1.0, p, seed)
    torch.cuda.synchronize()
    got = (o > 0).cpu().numpy()
    want = orc.dropout_keep_reference(seed, b, h, nq, nk, p)
    assert np.array_equal(got, want)
    t, r = orc.dropout_threshold(p)
    kept = o[o > 0].float()
    assert torch.allclose(kept, torch.full_like(kept, r / nk), rtol=2e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("d", [32, 64, 128])
def test_dkdv_pattern_bitwise(d):
    """Uniform P and dO = I over the Nq = D queries: dV[k, q] = Z[q, k] r / Nk,
    so dV > 0 is the dK/dV kernel's keep pattern (transposed)."""
    b, h, nq, nk = 2, 2, d, 256
    p, seed = 0.4, 321
    q = torch.zeros(b, h, nq, d, device="cuda", dtype=torch.float16)
    k = torch.zeros(b, h, nk, d, device="cuda", dtype=torch.float16)
    v = torch.randn(b, h, nk, d, device="cuda", dtype=torch.float16)
    o, lse = fa.attention_forward_dropout(q, k, v, False, 1.0, p, seed)
    do = torch.eye(nq, d, device="cuda", dtype=torch.float16).expand(b, h, nq, d).contiguous()
    _, _, dv = fa.attention_backward_dropout(q, k, v, o, do, lse, False, 1.0, p, seed)
    torch.cuda.synchronize()
    got = (dv > 0).cpu().numpy()  # (b, h, nk, d = nq)
    want = orc.dropout_keep_reference(seed, b, h, nq, nk, p).swapaxes(2, 3)
    assert np.array_equal(got, want)


@pytest.mark.gpu
def test_key_index_high_bits_pattern():
    """Key indices past 2^17 (the key half of the block word's high bits,
    drop_key2): the forward's pattern read out of O with V one-hot on the keys
    [2^17 + 128, 2^17 + 160) (O[q, j] = Z[q, k0 + j] r / Nk), and the dK/dV
    kernel's out of dV with dO = I over every key."""
    b = h = 1
    nq = d = 32
    nk, k0 = 2 ** 17 + 256, 2 ** 17 + 128
    p, seed = 0.3, 2 ** 33 + 99
    q = torch.zeros(b, h, nq, d, device="cuda", dtype=torch.float16)
    k = torch.zeros(b, h, nk, d, device="cuda", dtype=torch.float16)
    v = torch.zeros(b, h, nk, d, device="cuda", dtype=torch.float16)
    v[0, 0, k0 + torch.arange(d), torch.arange(d)] = 1
    o, lse = fa.attention_forward_dropout(q, k, v, False, 1.0, p, seed)
    want = orc.dropout_keep_reference(seed, b, h, nq, nk, p)  # (b, h, nq, nk)
    torch.cuda.synchronize()
    assert np.array_equal((o > 0).cpu().numpy(), want[..., k0:k0 + d])
    do = torch.eye(nq, d, device="cuda", dtype=torch.float16).expand(b, h, nq, d).contiguous()
    _, _, dv = fa.attention_backward_dropout(q, k, v, o, do, lse, False, 1.0, p, seed)
    torch.cuda.synchronize()
    assert np.array_equal((dv > 0).cpu().numpy(), want.swapaxes(2, 3))


CASES = [
    # b, hq, hkv, nq, nk, d, dv, causal, p
    (2, 4, 2, 300, 300, 64, 64, True, 0.1),
    (2, 4, 4, 257, 257, 32, 32, False, 0.5),
    (1, 4, 2, 200, 333, 128, 128, True, 0.2),
    (1, 2, 2, 129, 517, 64, 128, False, 0.3),
]


def _inputs(b, hq, hkv, nq, nk, d, dv, seed, dtype=torch.float16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(b, hq, nq, d, generator=g).to(dtype)
    k = torch.randn(b, hkv, nk, d, generator=g).to(dtype)
    v = torch.randn(b, hkv, nk, dv, generator=g).to(dtype)
    do = torch.randn(b, hq, nq, dv, generator=g).to(dtype)
    return q, k, v, do


def _run(q, k, v, do, causal, p, seed):
    qc, kc, vc = (t.cuda() for t in (q, k, v))
    scale = q.shape[-1] ** -0.5
    o, lse = fa.attention_forward_dropout(qc, kc, vc, causal, scale, p, seed)
    dq, dk, dv = fa.attention_backward_dropout(qc, kc, vc, o, do.cuda(), lse, causal, scale, p, seed)
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in (o, dq, dk, dv)]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_dropout_against_float64(case):
    b, hq, hkv, nq, nk, d, dv, causal, p = case
    q, k, v, do = _inputs(b, hq, hkv, nq, nk, d, dv, seed=nq + d)
    seed = 1000 + nq
    keep = orc.dropout_keep_reference(seed, b, hq, nq, nk, p)
    _, r = orc.dropout_threshold(p)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                             scale=d ** -0.5, do=do.float().numpy(), dropout_keep=keep, dropout_scale=r)
    ours = _run(q, k, v, do, causal, p, seed)
    errs = {name: _maxabs(a, ref[name]) for name, a in zip(("o", "dq", "dk", "dv"), ours)}
    assert errs["o"] <= O_TOL * r, errs
    assert max(errs["dq"], errs["dk"], errs["dv"]) <= GRAD_TOL * r, errs
    assert _abi.device_status() == 0


@pytest.mark.gpu
def test_dropout_public_api_and_repeatability():
    q, k, v, do = _inputs(2, 4, 2, 300, 300, 64, 64, seed=5)

    def run():
        torch.manual_seed(77)
        qc, kc, vc = (t.cuda().requires_grad_() for t in (q, k, v))
        o = fa.scaled_dot_product_attention(qc, kc, vc, is_causal=True, enable_gqa=True, dropout_p=0.2)
        g = torch.autograd.grad(o, (qc, kc, vc), do.cuda())
        torch.cuda.synchronize()
        return [t.detach().cpu() for t in (o, *g)]

    first, second = run(), run()
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    torch.manual_seed(78)
    qc, kc, vc = (t.cuda() for t in (q, k, v))
    other = fa.scaled_dot_product_attention(qc, kc, vc, is_causal=True, enable_gqa=True, dropout_p=0.2)
    assert not torch.equal(other.cpu(), first[0])


@pytest.mark.gpu
def test_dropout_bf16():
    q, k, v, do = _inputs(1, 4, 2, 200, 333, 64, 64, seed=9, dtype=torch.bfloat16)
    p, seed = 0.25, 4242
    keep = orc.dropout_keep_reference(seed, 1, 4, 200, 333, p)
    _, r = orc.dropout_threshold(p)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=False,
                             scale=64 ** -0.5, do=do.float().numpy(), dropout_keep=keep, dropout_scale=r)
    ours = _run(q, k, v, do, False, p, seed)
    # bf16: 8 mantissa bits against fp16's 11
    for name, a in zip(("o", "dq", "dk", "dv"), ours):
        assert _maxabs(a, ref[name]) <= (O_TOL if name == "o" else GRAD_TOL) * r * 8, name
