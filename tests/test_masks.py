"""Dense boolean attention masks (``attn_mask``).

The reference has none (README.md:93); PyTorch's SDPA semantics are the
model: ``True`` where the key takes part, broadcast to (batch, query heads,
query length, key length), AND-ed with ``is_causal``.  The kernels read the
mask as packed bit rows (fa_mask_pack).

CPU tests pin the oracle's masked attention against PyTorch's float64 SDPA
and its bit layout (``mask_bits_reference``) by a round trip, and check the
Python validation and the ABI's argument checks.  GPU tests:
* the pack kernel's words equal the oracle's bit for bit (contiguous,
  broadcast and transposed masks, ragged lengths; both the 4-byte and the
  byte-wise variant);
* parity with the float64 oracle through the public API, forward and
  backward, at the equal-width tolerances (O 2e-3, gradients 1e-2), for
  random masks of every broadcast form, with and without causal, self- and
  cross-attention, GQA, D 32/64/128, Dv != D, rows that see no key (o = 0,
  zero gradients), the fused and the deterministic backward, bf16 (twice
  PyTorch's bf16 error + 2e-3);
* an all-True mask gives bitwise the unmasked result (forward, and dK/dV of
  the fused backward; all gradients of the deterministic one).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import triton_flash_attention_b200 as fa
from triton_flash_attention_b200 import _abi
from triton_flash_attention_b200.masks import validate_attention_mask
from oracle import fa2_oracle as orc

O_TOL = 2e-3
GRAD_TOL = 1e-2


def _inputs(b, hq, hkv, nq, nk, d, seed, dv=None, dtype=torch.float16):
    dv = dv or d
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(b, hq, nq, d, generator=g).to(dtype)
    k = torch.randn(b, hkv, nk, d, generator=g).to(dtype)
    v = torch.randn(b, hkv, nk, dv, generator=g).to(dtype)
    do = torch.randn(b, hq, nq, dv, generator=g).to(dtype)
    return q, k, v, do


def _random_mask(shape, seed, density=0.7):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.rand(shape, generator=g) < density


def _maxabs(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


def test_oracle_mask_matches_torch_float64():
    q, k, v, do = (t.double() for t in _inputs(2, 4, 2, 37, 53, 32, seed=3))
    mask = _random_mask((2, 1, 37, 53), seed=4)
    mask[..., 0] = True  # every row sees a key (PyTorch's SDPA gives NaN otherwise)
    ref = orc.sdpa_reference(q.numpy(), k.numpy(), v.numpy(), causal=False, do=do.numpy(), mask=mask.numpy())
    qt, kt, vt = (t.clone().requires_grad_() for t in (q, k, v))
    o = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, enable_gqa=True)
    grads = torch.autograd.grad(o, (qt, kt, vt), do)
    for name, t in zip(("o", "dq", "dk", "dv"), (o, *grads)):
        assert _maxabs(t.detach().numpy(), ref[name]) <= 1e-10, name


@pytest.mark.parametrize("nq,nk", [(1, 1), (37, 300), (256, 129)])
def test_oracle_mask_bits_round_trip(nq, nk):
    mask = _random_mask((2, 3, nq, nk), seed=nq + nk).numpy()
    bits, bits_t = orc.mask_bits_reference(mask)
    assert bits.shape == (2, 3, nq, (nk + 127) // 128 * 4)
    assert bits_t.shape == (2, 3, nk, (nq + 127) // 128 * 4)
    k = np.arange(nk)
    back = (bits[..., k >> 5] >> (k & 31).astype(np.uint32)) & 1
    assert np.array_equal(back.astype(bool), mask)
    q = np.arange(nq)
    back_t = (bits_t[..., q >> 5] >> (q & 31).astype(np.uint32)) & 1
    assert np.array_equal(back_t.astype(bool), np.swapaxes(mask, 2, 3))
    # padding bits are zero
    total = np.unpackbits(bits.view(np.uint8)).sum()
    assert total == mask.sum()


def test_mask_validation_messages():
    q = torch.zeros(2, 4, 5, 32, dtype=torch.float16)
    k = torch.zeros(2, 2, 7, 32, dtype=torch.float16)
    validate_attention_mask(torch.ones(5, 7, dtype=torch.bool), q, k)
    validate_attention_mask(torch.ones(2, 1, 1, 7, dtype=torch.bool), q, k)
    validate_attention_mask(torch.ones(2, 4, 5, 7, dtype=torch.bool), q, k)
    with pytest.raises(TypeError, match="attn_mask must be a torch.Tensor"):
        validate_attention_mask(np.ones((5, 7), dtype=bool), q, k)
    with pytest.raises(ValueError, match="bool tensor"):
        validate_attention_mask(torch.zeros(5, 7), q, k)
    with pytest.raises(ValueError, match="does not broadcast"):
        validate_attention_mask(torch.ones(2, 2, 5, 7, dtype=torch.bool), q, k)  # Hkv, not Hq
    with pytest.raises(ValueError, match="does not broadcast"):
        validate_attention_mask(torch.ones(1, 1, 1, 2, 5, 7, dtype=torch.bool), q, k)


def test_masked_abi_rejections():
    """Argument checks before any CUDA call (runs without a GPU)."""
    lib = _abi.lib()
    s = (ctypes.c_int64 * 3)(64 * 64, 64 * 64, 64)
    ms = (ctypes.c_int64 * 3)(0, 0, 4)
    # no mask
    rc = lib.fa_fwd_masked(16, 16, 16, 16, 16, 1, 1, 1, 64, 64, 64, 64, s, s, s, s, None, ms, 0.125, 0, None)
    assert rc == _abi.FA_ERR_BAD_SHAPE
    # misaligned bits, and a row stride below the padded width of 4 words
    rc = lib.fa_fwd_masked(16, 16, 16, 16, 16, 1, 1, 1, 64, 64, 64, 64, s, s, s, s, 20, ms, 0.125, 0, None)
    assert rc == _abi.FA_ERR_MISALIGNED
    short = (ctypes.c_int64 * 3)(0, 0, 2)
    rc = lib.fa_fwd_masked(16, 16, 16, 16, 16, 1, 1, 1, 64, 64, 64, 64, s, s, s, s, 32, short, 0.125, 0, None)
    assert rc == _abi.FA_ERR_MISALIGNED
    # the backward needs both packed matrices
    rc = lib.fa_bwd_masked(16, 16, 16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 1, 1, 64, 64, 64, 64,
                           s, s, s, s, s, s, s, s, 32, ms, None, ms, 0.125, 0, 1, None)
    assert rc == _abi.FA_ERR_BAD_SHAPE
    # pack: negative stride, misaligned output
    st4 = (ctypes.c_int64 * 4)(0, 0, 64, -1)
    assert lib.fa_mask_pack(16, 1, 1, 64, 64, st4, 32, 32, None) == _abi.FA_ERR_BAD_SHAPE
    st4 = (ctypes.c_int64 * 4)(0, 0, 64, 1)
    assert lib.fa_mask_pack(16, 1, 1, 64, 64, st4, 36, 32, None) == _abi.FA_ERR_MISALIGNED


# ---------------------------------------------------------------------------
# GPU


def _as_u32(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,nq,nk,form", [
    ((2, 3, 200, 300), 200, 300, "plain"),
    ((2, 1, 1, 300), 200, 300, "key padding"),
    ((1, 1, 129, 1000), 129, 1000, "plain"),
    ((2, 3, 300, 200), 200, 300, "transposed view"),
    ((1, 1, 1, 1), 1, 1, "plain"),
    ((2, 3, 77, 333), 77, 333, "plain"),  # Nk % 4 != 0: the byte-wise kernel
])
def test_mask_pack_kernel_bitwise(shape, nq, nk, form):
    mask = _random_mask(shape, seed=nq * 7 + nk).cuda()
    if form == "transposed view":
        mask = mask.transpose(2, 3)  # (2, 3, 200, 300), key stride != 1
    packed = fa.pack_attention_mask(mask, 2, 3, nq, nk)
    torch.cuda.synchronize()
    m4 = mask.reshape((1,) * (4 - mask.ndim) + tuple(mask.shape))
    full = m4.expand(m4.shape[0], m4.shape[1], nq, nk).cpu().numpy()
    bits, bits_t = orc.mask_bits_reference(full)
    assert np.array_equal(_as_u32(packed.bits), bits)
    assert np.array_equal(_as_u32(packed.bits_t), bits_t)
    assert _abi.device_status() == 0


def _grads(q, k, v, do, causal, mask, fn=None):
    fn = fn or fa.scaled_dot_product_attention
    qc, kc, vc = (t.cuda().requires_grad_() for t in (q, k, v))
    o = fn(qc, kc, vc, is_causal=causal, enable_gqa=q.shape[1] != k.shape[1], attn_mask=mask.cuda())
    g = torch.autograd.grad(o, (qc, kc, vc), do.cuda())
    torch.cuda.synchronize()
    return [t.detach().float().cpu().numpy() for t in (o, *g)]


CASES = [
    # b, hq, hkv, nq, nk, d, dv, mask shape (None: full), causal
    (2, 4, 2, 300, 300, 64, 64, None, False),
    (2, 4, 2, 300, 300, 64, 64, None, True),
    (2, 4, 4, 129, 517, 32, 32, "key padding", False),
    (1, 4, 2, 517, 129, 128, 128, None, False),
    (1, 4, 2, 300, 300, 128, 128, "shared", True),
    (2, 2, 2, 200, 333, 64, 128, None, False),
    (1, 8, 2, 64, 64, 32, 32, "per head", True),
]


def _mask_for(kind, b, hq, nq, nk, seed):
    if kind is None:
        return _random_mask((b, hq, nq, nk), seed)
    if kind == "key padding":  # (B, 1, 1, Nk): a batch's trailing keys hidden
        m = torch.ones(b, 1, 1, nk, dtype=torch.bool)
        for i in range(b):
            m[i, ..., nk - 37 * (i + 1):] = False
        return m
    if kind == "shared":  # (Nq, Nk), one mask for every batch and head
        return _random_mask((nq, nk), seed)
    if kind == "per head":  # (1, Hq, Nq, Nk)
        return _random_mask((1, hq, nq, nk), seed, density=0.3)
    raise ValueError(kind)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_masked_against_float64(case):
    b, hq, hkv, nq, nk, d, dv, kind, causal = case
    q, k, v, do = _inputs(b, hq, hkv, nq, nk, d, seed=nq + nk + d, dv=dv)
    mask = _mask_for(kind, b, hq, nq, nk, seed=nq * 3 + d)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                             scale=d ** -0.5, do=do.float().numpy(), mask=mask.numpy())
    ours = _grads(q, k, v, do, causal, mask)
    errs = {name: _maxabs(a, ref[name]) for name, a in zip(("o", "dq", "dk", "dv"), ours)}
    assert errs["o"] <= O_TOL, errs
    assert max(errs["dq"], errs["dk"], errs["dv"]) <= GRAD_TOL, errs
    assert _abi.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("d", [32, 64, 128])
def test_masked_rows_without_keys(d):
    """Rows whose keys are all hidden: o = 0, lse = -inf, zero dQ, and no
    contribution to dK / dV."""
    q, k, v, do = _inputs(1, 2, 2, 200, 200, d, seed=d)
    mask = _random_mask((1, 2, 200, 200), seed=d + 1)
    mask[0, 0, 10:50] = False
    mask[0, 1, 150:] = False
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True,
                             scale=d ** -0.5, do=do.float().numpy(), mask=mask.numpy())
    ours = _grads(q, k, v, do, True, mask)
    assert np.all(ours[0][0, 0, 10:50] == 0) and np.all(ours[0][0, 1, 150:] == 0)
    assert np.all(ours[1][0, 0, 10:50] == 0) and np.all(ours[1][0, 1, 150:] == 0)
    for name, a in zip(("o", "dq", "dk", "dv"), ours):
        assert np.isfinite(a).all(), name
        assert _maxabs(a, ref[name]) <= (O_TOL if name == "o" else GRAD_TOL), name
    packed = fa.pack_attention_mask(mask.cuda(), 1, 2, 200, 200)
    _, lse = fa.attention_forward_masked(q.cuda(), k.cuda(), v.cuda(), packed, True, d ** -0.5)
    lse = lse.cpu()
    assert torch.isneginf(lse[0, 0, 10:50]).all() and torch.isneginf(lse[0, 1, 150:]).all()


@pytest.mark.gpu
@pytest.mark.parametrize("d", [32, 64])
def test_masked_deterministic_backward(d):
    q, k, v, do = _inputs(2, 4, 2, 257, 257, d, seed=d + 5)
    mask = _random_mask((2, 1, 257, 257), seed=d + 6)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=False,
                             scale=d ** -0.5, do=do.float().numpy(), mask=mask.numpy())
    torch.use_deterministic_algorithms(True)
    try:
        first = _grads(q, k, v, do, False, mask)
        second = _grads(q, k, v, do, False, mask)
    finally:
        torch.use_deterministic_algorithms(False)
    for a, b in zip(first, second):
        assert np.array_equal(a, b)
    for name, a in zip(("o", "dq", "dk", "dv"), first):
        assert _maxabs(a, ref[name]) <= (O_TOL if name == "o" else GRAD_TOL), name


@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128])
def test_masked_bf16(d):
    q, k, v, do = _inputs(1, 4, 2, 200, 333, d, seed=d + 9, dtype=torch.bfloat16)
    mask = _random_mask((1, 4, 200, 333), seed=d + 10)
    mask[..., 0] = True  # PyTorch's SDPA gives NaN for rows without keys
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=False,
                             scale=d ** -0.5, do=do.float().numpy(), mask=mask.numpy())
    ours = _grads(q, k, v, do, False, mask)
    theirs = _grads(q, k, v, do, False, mask, fn=torch.nn.functional.scaled_dot_product_attention)
    for name, a, t in zip(("o", "dq", "dk", "dv"), ours, theirs):
        err, terr = _maxabs(a, ref[name]), _maxabs(t, ref[name])
        assert err <= 2 * terr + 2e-3, (name, err, terr)


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [32, 64, 128])
def test_all_true_mask_equals_unmasked(d, causal):
    """The masked instantiations only add the bit test: with every bit set
    they give the unmasked results bitwise (forward; dK/dV of the fused
    backward, whose dQ sums in schedule order; every gradient of the
    deterministic backward)."""
    q, k, v, do = (t.cuda() for t in _inputs(2, 4, 2, 300, 300, d, seed=d + int(causal)))
    scale = d ** -0.5
    packed = fa.pack_attention_mask(torch.ones(300, 300, dtype=torch.bool, device="cuda"), 2, 4, 300, 300)
    o_m, lse_m = fa.attention_forward_masked(q, k, v, packed, causal, scale)
    o, lse = fa.attention_forward(q, k, v, causal, scale)
    torch.cuda.synchronize()
    assert torch.equal(o_m, o) and torch.equal(lse_m, lse)
    if d <= 64:
        dq_m, dk_m, dv_m = fa.attention_backward_masked(q, k, v, o, do, lse, packed, causal, scale)
        dq, dk, dv = fa.attention_backward_fused(q, k, v, o, do, lse, causal, scale)
        torch.cuda.synchronize()
        assert torch.equal(dk_m, dk) and torch.equal(dv_m, dv)
        assert _maxabs(dq_m.float().cpu(), dq.float().cpu()) <= 1e-3 + 1e-2 * float(dq.float().abs().max())
    torch.use_deterministic_algorithms(True)
    try:
        dq_m, dk_m, dv_m = fa.attention_backward_masked(q, k, v, o, do, lse, packed, causal, scale)
    finally:
        torch.use_deterministic_algorithms(False)
    delta = fa.attention_delta(o, do)
    dq = fa.attention_backward_dq(q, k, v, do, lse, delta, causal, scale)
    dk, dv = fa.attention_backward_dkdv(q, k, v, do, lse, delta, causal, scale)
    torch.cuda.synchronize()
    assert torch.equal(dq_m, dq) and torch.equal(dk_m, dk) and torch.equal(dv_m, dv)
