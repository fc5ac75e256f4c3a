"""Value head size Dv different from the query/key head size D.

The reference serves these inputs only through PyTorch's SDPA
(triton_flash_attention/attention.py:639-646: its Triton kernel takes one
head size).  Here the kernels run at width W = max(D, Dv), reading the
narrower operands through tensor maps whose extent is their own width (the
TMA fills the missing columns with zeros), and store only the real columns
of O, dQ, dK and dV.

GPU tests:
* parity with the float64 oracle through the public API, forward and
  backward, for every pair of head sizes, causal and not, self- and
  cross-attention, GQA, fp16 and bf16, the fused and the deterministic
  backward -- the tolerances of the equal-width parity tests (O 2e-3,
  lse2 1e-3, gradients 1e-2; bf16 twice PyTorch's bf16 error + 2e-3);
* the narrow call equals the W-wide call on explicitly zero-padded inputs
  bitwise (same kernels, same arithmetic), for O, lse and the split-path
  gradients;
* outputs written into views of wider buffers leave the columns past their
  width untouched (the store masks).
CPU tests pin the oracle for Dv != D against PyTorch's float64 SDPA.
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
LSE_TOL = 1e-3
GRAD_TOL = 1e-2

PAIRS = [(32, 64), (64, 32), (32, 128), (128, 32), (64, 128), (128, 64)]


def _inputs(b, hq, hkv, nq, nk, d, dv, seed, dtype=torch.float16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(b, hq, nq, d, generator=g).to(dtype)
    k = torch.randn(b, hkv, nk, d, generator=g).to(dtype)
    v = torch.randn(b, hkv, nk, dv, generator=g).to(dtype)
    do = torch.randn(b, hq, nq, dv, generator=g).to(dtype)
    return q, k, v, do


def _maxabs(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


def _grads(fn, q, k, v, do, causal, **kw):
    qc, kc, vc = (t.cuda().requires_grad_() for t in (q, k, v))
    o = fn(qc, kc, vc, is_causal=causal, enable_gqa=q.shape[1] != k.shape[1], **kw)
    g = torch.autograd.grad(o, (qc, kc, vc), do.cuda())
    torch.cuda.synchronize()
    return [t.detach().float().cpu().numpy() for t in (o, *g)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d,dv", [(32, 64), (64, 32)])
def test_oracle_vdim_matches_torch_float64(d, dv, causal):
    """The oracle's Dv != D forward and gradients equal PyTorch's float64
    SDPA (its autograd) on the same inputs."""
    q, k, v, do = (t.double() for t in _inputs(1, 2, 2, 19, 23, d, dv, seed=d + dv))
    ref = orc.sdpa_reference(q.numpy(), k.numpy(), v.numpy(), causal=causal, scale=d ** -0.5, do=do.numpy())
    qt, kt, vt = (t.clone().requires_grad_() for t in (q, k, v))
    o = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=causal)
    grads = torch.autograd.grad(o, (qt, kt, vt), do)
    assert ref["o"].shape == (1, 2, 19, dv)
    for name, t in zip(("o", "dq", "dk", "dv"), (o, *grads)):
        assert _maxabs(t.detach().numpy(), ref[name]) <= 1e-10, name


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d,dv", PAIRS)
@pytest.mark.parametrize("nq,nk", [(129, 129), (300, 200)])
def test_vdim_against_float64(d, dv, nq, nk, causal):
    q, k, v, do = _inputs(2, 4, 2, nq, nk, d, dv, seed=d * 3 + dv + nq)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                             scale=d ** -0.5, do=do.float().numpy())
    ours = _grads(fa.scaled_dot_product_attention, q, k, v, do, causal)
    assert ours[0].shape == (2, 4, nq, dv)
    errs = {name: _maxabs(a, ref[name]) for name, a in zip(("o", "dq", "dk", "dv"), ours)}
    assert errs["o"] <= O_TOL, errs
    assert max(errs["dq"], errs["dk"], errs["dv"]) <= GRAD_TOL, errs
    o, lse = fa.attention_forward(q.cuda(), k.cuda(), v.cuda(), causal, d ** -0.5)
    torch.cuda.synchronize()
    assert _maxabs(lse.cpu(), ref["lse2"]) <= LSE_TOL
    assert _abi.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("d,dv", [(32, 64), (64, 32)])
def test_vdim_deterministic_backward(d, dv):
    """max(D, Dv) <= 64 runs the fused backward; with deterministic
    algorithms on, the separate dQ and dK/dV kernels run, and two runs agree
    bitwise."""
    q, k, v, do = _inputs(1, 4, 4, 257, 257, d, dv, seed=d + 2 * dv)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True,
                             scale=d ** -0.5, do=do.float().numpy())
    torch.use_deterministic_algorithms(True)
    try:
        first = _grads(fa.scaled_dot_product_attention, q, k, v, do, True)
        second = _grads(fa.scaled_dot_product_attention, q, k, v, do, True)
    finally:
        torch.use_deterministic_algorithms(False)
    for a, b in zip(first, second):
        assert np.array_equal(a, b)
    for name, a in zip(("o", "dq", "dk", "dv"), first):
        assert _maxabs(a, ref[name]) <= (O_TOL if name == "o" else GRAD_TOL), name


@pytest.mark.gpu
@pytest.mark.parametrize("d,dv", [(64, 128), (128, 32)])
def test_vdim_bf16(d, dv):
    q, k, v, do = _inputs(1, 4, 2, 200, 333, d, dv, seed=d + dv, dtype=torch.bfloat16)
    ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True,
                             scale=d ** -0.5, do=do.float().numpy())
    ours = _grads(fa.scaled_dot_product_attention, q, k, v, do, True)
    theirs = _grads(torch.nn.functional.scaled_dot_product_attention, q, k, v, do, True)
    for name, a, t in zip(("o", "dq", "dk", "dv"), ours, theirs):
        err, terr = _maxabs(a, ref[name]), _maxabs(t, ref[name])
        assert err <= 2 * terr + 2e-3, (name, err, terr)


def _pad(t, width):
    return torch.nn.functional.pad(t, (0, width - t.shape[-1]))


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d,dv", PAIRS)
def test_vdim_equals_padded_equal_width_call(d, dv, causal):
    """The narrow call runs the W-wide kernels with zero-filled columns, so
    it equals the W-wide call on explicitly zero-padded inputs bitwise: O and
    lse of the forward, and the gradients of the deterministic split path."""
    w = max(d, dv)
    q, k, v, do = (t.cuda() for t in _inputs(1, 4, 2, 300, 300, d, dv, seed=w + d))
    qp, kp, vp, dop = (_pad(t, w) for t in (q, k, v, do))
    scale = d ** -0.5
    o, lse = fa.attention_forward_vdim(q, k, v, causal, scale)
    op, lsep = fa.attention_forward(qp, kp, vp, causal, scale)
    torch.cuda.synchronize()
    assert torch.equal(o, op[..., :dv])
    assert torch.equal(lse, lsep)
    torch.use_deterministic_algorithms(True)
    try:
        dq, dk, dv_ = fa.attention_backward_vdim(q, k, v, o, do, lse, causal, scale)
    finally:
        torch.use_deterministic_algorithms(False)
    delta = fa.attention_delta(op, dop)
    dqp = fa.attention_backward_dq(qp, kp, vp, dop, lsep, delta, causal, scale)
    dkp, dvp = fa.attention_backward_dkdv(qp, kp, vp, dop, lsep, delta, causal, scale)
    torch.cuda.synchronize()
    assert torch.equal(dq, dqp[..., :d])
    assert torch.equal(dk, dkp[..., :d])
    assert torch.equal(dv_, dvp[..., :dv])


@pytest.mark.gpu
@pytest.mark.parametrize("d,dv,deterministic", [(32, 64, 0), (64, 32, 0), (128, 32, 1), (32, 128, 1)])
def test_vdim_leaves_columns_past_the_width_alone(d, dv, deterministic):
    """Outputs handed over as views of wider buffers (row stride 256
    elements): the columns past each output's width keep their sentinel."""
    b, h, n = 1, 2, 200
    q, k, v, do = (t.cuda() for t in _inputs(b, h, h, n, n, d, dv, seed=d * dv))
    scale = d ** -0.5
    sentinel = -7.0

    def wide(width):
        buf = torch.full((b, h, n, 256), sentinel, device="cuda", dtype=torch.float16)
        return buf, buf[..., :width]

    o_buf, o = wide(dv)
    lse = torch.empty((b, h, n), device="cuda", dtype=torch.float32)
    lib = _abi.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.fa_fwd_vdim(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                         b, h, h, n, n, d, dv, _abi.strides3(q), _abi.strides3(k), _abi.strides3(v),
                         _abi.strides3(o), scale, 1, stream)
    _abi.check(rc, "fa_fwd_vdim")
    (dq_buf, dq), (dk_buf, dk), (dv_buf, dvv) = wide(d), wide(d), wide(dv)
    delta = torch.empty((b, h, n), device="cuda", dtype=torch.float32)
    acc = torch.empty((b, h, n, max(d, dv)), device="cuda", dtype=torch.float32)
    rc = lib.fa_bwd_vdim(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                         dq.data_ptr(), dk.data_ptr(), dvv.data_ptr(), delta.data_ptr(), acc.data_ptr(),
                         b, h, h, n, n, d, dv, _abi.strides3(q), _abi.strides3(k), _abi.strides3(v),
                         _abi.strides3(o), _abi.strides3(do), _abi.strides3(dq), _abi.strides3(dk),
                         _abi.strides3(dvv), scale, 1, deterministic, stream)
    _abi.check(rc, "fa_bwd_vdim")
    torch.cuda.synchronize()
    assert _abi.device_status() == 0
    for buf, width in ((o_buf, dv), (dq_buf, d), (dk_buf, d), (dv_buf, dv)):
        assert bool((buf[..., width:] == sentinel).all())
        assert not bool((buf[..., :width] == sentinel).any())
    ref = orc.sdpa_reference(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                             causal=True, scale=scale, do=do.float().cpu().numpy())
    assert _maxabs(o.float().cpu(), ref["o"]) <= O_TOL
    for name, t in (("dq", dq), ("dk", dk), ("dv", dvv)):
        assert _maxabs(t.float().cpu(), ref[name]) <= GRAD_TOL, name


def test_vdim_abi_rejections():
    """Argument checks before any CUDA call (runs without a GPU)."""
    lib = _abi.lib()
    s = (ctypes.c_int64 * 3)(64 * 64, 64 * 64, 64)
    for d, dv in ((64, 48), (96, 64), (64, 0)):
        rc = lib.fa_fwd_vdim(16, 16, 16, 16, 16, 1, 1, 1, 64, 64, d, dv, s, s, s, s, 0.125, 1, None)
        assert rc == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM, (d, dv)
    # the fused backward (max(D, Dv) <= 64, not deterministic) needs dq_accum
    rc = lib.fa_bwd_vdim(16, 16, 16, 16, 16, 16, 16, 16, 16, 16, None, 1, 1, 1, 64, 64, 32, 64,
                         s, s, s, s, s, s, s, s, 0.125, 1, 0, None)
    assert rc == _abi.FA_ERR_BAD_SHAPE
    # a misaligned output pointer
    rc = lib.fa_bwd_vdim(16, 16, 16, 16, 16, 16, 18, 16, 16, 16, 16, 1, 1, 1, 64, 64, 32, 64,
                         s, s, s, s, s, s, s, s, 0.125, 1, 0, None)
    assert rc == _abi.FA_ERR_MISALIGNED
