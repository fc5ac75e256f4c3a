"""Packed variable-length batches (``scaled_dot_product_attention_varlen``,
C ABI ``fa_fwd_varlen`` / ``fa_bwd_varlen``).

The reference has no packed layout; the oracle applies its dense math to
each sequence (``oracle.fa2_oracle.sdpa_varlen_reference``).  GPU bars, as
for the dense path: O within 2e-3 and dQ, dK, dV within 1e-2 max-abs of
float64 for fp16, lse2 within 1e-3; bf16 within twice PyTorch's own bf16
SDPA error (per sequence) plus 2e-3.  Ragged cases cover empty sequences,
single rows, lengths across the 128-row tiles, query and key lengths that
differ per sequence, GQA, every head dim, the fused and the deterministic
backward.  Equal-length sequences must match the dense kernels exactly in
the forward.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import triton_flash_attention_b200 as fa
from oracle import fa2_oracle as orc


def _cu(lens):
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def _inputs(lens_q, lens_k, hq, hkv, d, seed, dtype=torch.float16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    tq, tk = int(sum(lens_q)), int(sum(lens_k))
    q = torch.randn(tq, hq, d, generator=g).to(dtype)
    k = torch.randn(tk, hkv, d, generator=g).to(dtype)
    v = torch.randn(tk, hkv, d, generator=g).to(dtype)
    do = torch.randn(tq, hq, d, generator=g).to(dtype)
    return q, k, v, do


def _maxabs(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


# ---------------------------------------------------------------- CPU
def test_oracle_varlen_matches_dense_for_equal_lengths():
    rng = np.random.default_rng(0)
    b, h, n, d = 3, 2, 37, 32
    q, k, v, do = (rng.standard_normal((b, h, n, d)) for _ in range(4))
    dense = orc.sdpa_reference(q, k, v, causal=True, do=do)
    pack = lambda x: x.transpose(0, 2, 1, 3).reshape(b * n, h, d)
    cu = _cu([n] * b)
    var = orc.sdpa_varlen_reference(pack(q), pack(k), pack(v), cu, cu, causal=True, do=pack(do))
    for name in ("o", "dq", "dk", "dv"):
        assert np.allclose(var[name], pack(dense[name]), atol=1e-12), name
    assert np.allclose(var["lse2"], dense["lse2"].transpose(1, 0, 2).reshape(h, b * n), atol=1e-12)


def test_oracle_varlen_empty_sequences():
    rng = np.random.default_rng(1)
    cu_q, cu_k = _cu([3, 0, 2]), _cu([0, 4, 5])
    q = rng.standard_normal((5, 1, 8))
    k = rng.standard_normal((9, 1, 8))
    r = orc.sdpa_varlen_reference(q, k, k, cu_q, cu_k, causal=False, do=q)
    assert np.all(r["o"][:3] == 0) and np.all(np.isneginf(r["lse2"][:, :3]))
    assert np.all(r["dk"][:4] == 0)  # keys of a sequence without queries get no gradient


def test_validation_messages():
    q = torch.zeros(4, 2, 64, dtype=torch.float16)
    cu = torch.tensor([0, 4], dtype=torch.int32)
    with pytest.raises(ValueError, match="total, heads, head_dim"):
        fa.scaled_dot_product_attention_varlen(q[None], q, q, cu, cu, 4, 4)
    with pytest.raises(ValueError, match="int32"):
        fa.scaled_dot_product_attention_varlen(q, q, q, cu.long(), cu, 4, 4)
    with pytest.raises(ValueError, match="max_seqlen_q"):
        fa.scaled_dot_product_attention_varlen(q, q, q, cu, cu, 0, 4)
    with pytest.raises(TypeError, match="is_causal"):
        fa.scaled_dot_product_attention_varlen(q, q, q, cu, cu, 4, 4, is_causal=1)
    with pytest.raises(ValueError, match="enable_gqa"):
        fa.scaled_dot_product_attention_varlen(q, q[:, :1], q[:, :1], cu, cu, 4, 4)
    # no CPU fallback
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        fa.scaled_dot_product_attention_varlen(q, q, q, cu, cu, 4, 4)


# ---------------------------------------------------------------- GPU
def _run(q, k, v, do, cu_q, cu_k, causal, scale=None):
    dev = "cuda"
    qc, kc, vc = (t.to(dev).requires_grad_() for t in (q, k, v))
    cq, ck = torch.from_numpy(cu_q).to(dev), torch.from_numpy(cu_k).to(dev)
    mq = int(np.diff(cu_q).max())
    mk = int(np.diff(cu_k).max())
    o = fa.scaled_dot_product_attention_varlen(qc, kc, vc, cq, ck, max(mq, 1), max(mk, 1), is_causal=causal,
                                               scale=scale, enable_gqa=q.shape[1] != k.shape[1])
    dq, dk, dv = torch.autograd.grad(o, (qc, kc, vc), do.to(dev))
    torch.cuda.synchronize()
    return o.detach(), dq, dk, dv


CASES = [
    # lens_q, lens_k (None: same), hq, hkv, d, causal
    ([1, 17, 128, 129, 300, 0, 64], None, 2, 2, 64, True),
    ([1, 17, 128, 129, 300, 0, 64], None, 2, 2, 64, False),
    ([200, 3, 257], None, 4, 2, 32, True),
    ([130, 64, 255], None, 2, 1, 128, True),
    ([130, 64, 255], None, 2, 2, 128, False),
    ([50, 129, 7], [300, 20, 7], 2, 2, 64, False),
    ([50, 129, 7], [300, 20, 7], 2, 2, 64, True),
    ([513, 1000], None, 8, 2, 64, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_varlen_against_float64(case):
    lens_q, lens_k, hq, hkv, d, causal = case
    lens_k = lens_q if lens_k is None else lens_k
    cu_q, cu_k = _cu(lens_q), _cu(lens_k)
    q, k, v, do = _inputs(lens_q, lens_k, hq, hkv, d, seed=sum(lens_q) + d + hq)
    o, dq, dk, dv = _run(q, k, v, do, cu_q, cu_k, causal)
    ref = orc.sdpa_varlen_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu_q, cu_k,
                                    causal=causal, do=do.float().numpy())
    assert _maxabs(o.float().cpu(), ref["o"]) <= 2e-3
    for name, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        err = _maxabs(t.float().cpu(), ref[name])
        assert err <= 1e-2, (name, err)
    # the saved log-sum-exp, (Hq, total_q), base 2
    cq = torch.from_numpy(cu_q).cuda()
    ck = torch.from_numpy(cu_k).cuda()
    _, lse = fa.varlen_attention_forward(q.cuda(), k.cuda(), v.cuda(), cq, ck, max(max(lens_q), 1),
                                         max(max(lens_k), 1), causal, d ** -0.5)
    lse = lse.cpu().numpy()
    finite = np.isfinite(ref["lse2"])
    assert np.array_equal(np.isfinite(lse), finite)
    assert _maxabs(lse[finite], ref["lse2"][finite]) <= 1e-3
    assert fa._abi.device_status() == 0


@pytest.mark.gpu
def test_varlen_deterministic_backward(deterministic):
    lens = [1, 200, 129, 64]
    cu = _cu(lens)
    q, k, v, do = _inputs(lens, lens, 4, 2, 64, seed=11)
    runs = [_run(q, k, v, do, cu, cu, True) for _ in range(2)]
    for a, b in zip(runs[0], runs[1]):
        assert torch.equal(a, b)
    ref = orc.sdpa_varlen_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu, cu,
                                    causal=True, do=do.float().numpy())
    for name, t in zip(("o", "dq", "dk", "dv"), runs[0]):
        assert _maxabs(t.float().cpu(), ref[name]) <= (2e-3 if name == "o" else 1e-2), name


@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128])
def test_varlen_bf16(d):
    lens = [77, 300, 1]
    cu = _cu(lens)
    q, k, v, do = _inputs(lens, lens, 2, 2, d, seed=d, dtype=torch.bfloat16)
    ours = _run(q, k, v, do, cu, cu, True)
    ref = orc.sdpa_varlen_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu, cu,
                                    causal=True, do=do.float().numpy())
    # PyTorch's bf16 SDPA, sequence by sequence, as the bar
    tq = [torch.zeros_like(t, device="cuda") for t in (q, q, k, v)]
    for i in range(len(lens)):
        s = slice(int(cu[i]), int(cu[i + 1]))
        qs, ks, vs = (t[s].transpose(0, 1)[None].cuda().requires_grad_() for t in (q, k, v))
        os_ = torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=True)
        gs = torch.autograd.grad(os_, (qs, ks, vs), do[s].transpose(0, 1)[None].cuda())
        for acc, val in zip(tq, (os_.detach(), *gs)):
            acc[s] = val[0].transpose(0, 1)
    for name, a, t in zip(("o", "dq", "dk", "dv"), ours, tq):
        err, terr = _maxabs(a.float().cpu(), ref[name]), _maxabs(t.float().cpu(), ref[name])
        assert err <= 2 * terr + 2e-3, (name, err, terr)


@pytest.mark.gpu
def test_varlen_equal_lengths_match_dense_forward():
    b, h, n, d = 3, 4, 300, 64
    g = torch.Generator(device="cpu").manual_seed(5)
    q, k, v = (torch.randn(b, h, n, d, generator=g).half().cuda() for _ in range(3))
    o_dense, lse_dense = fa.attention_forward(q, k, v, True, d ** -0.5)
    pack = lambda x: x.transpose(1, 2).reshape(b * n, h, d).contiguous()
    cu = torch.tensor(_cu([n] * b), device="cuda")
    o_var, lse_var = fa.varlen_attention_forward(pack(q), pack(k), pack(v), cu, cu, n, n, True, d ** -0.5)
    assert torch.equal(o_var, pack(o_dense))
    assert torch.equal(lse_var, lse_dense.transpose(0, 1).reshape(h, b * n))


# ---------------------------------------------------------------- sliding window
def test_oracle_window_mask():
    m = orc.causal_mask(5, 5, window=2)
    assert m.tolist() == [[i - 2 < j <= i for j in range(5)] for i in range(5)]


def test_window_validation():
    q = torch.zeros(4, 2, 64, dtype=torch.float16)
    cu = torch.tensor([0, 4], dtype=torch.int32)
    with pytest.raises(ValueError, match="is_causal"):
        fa.scaled_dot_product_attention_varlen(q, q, q, cu, cu, 4, 4, window_size=2)
    with pytest.raises(ValueError, match="positive int"):
        fa.scaled_dot_product_attention_varlen(q, q, q, cu, cu, 4, 4, is_causal=True, window_size=0)


WINDOW_CASES = [
    # lens, hq, hkv, d, window
    ([1, 17, 300, 129, 600], 2, 2, 64, 100),
    ([1, 17, 300, 129, 600], 2, 2, 64, 128),
    ([257, 1000], 4, 2, 32, 1),
    ([700, 64], 2, 1, 128, 200),
    ([1000, 513], 2, 2, 64, 333),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", WINDOW_CASES)
def test_varlen_sliding_window_against_float64(case):
    """Causal sliding window: forward (O, lse2) and both backward paths
    (fused and the deterministic split) against float64."""
    lens, hq, hkv, d, window = case
    cu = _cu(lens)
    q, k, v, do = _inputs(lens, lens, hq, hkv, d, seed=window + d)
    ref = orc.sdpa_varlen_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu, cu,
                                    causal=True, do=do.float().numpy(), window=window)
    cq = torch.from_numpy(cu).cuda()
    for det in (False, True):
        prev = torch.are_deterministic_algorithms_enabled()
        torch.use_deterministic_algorithms(det)
        try:
            qc, kc, vc = (t.cuda().requires_grad_() for t in (q, k, v))
            o = fa.scaled_dot_product_attention_varlen(qc, kc, vc, cq, cq, max(lens), max(lens), is_causal=True,
                                                       enable_gqa=hq != hkv, window_size=window)
            grads = torch.autograd.grad(o, (qc, kc, vc), do.cuda())
            torch.cuda.synchronize()
        finally:
            torch.use_deterministic_algorithms(prev)
        assert _maxabs(o.detach().float().cpu(), ref["o"]) <= 2e-3
        for name, t in zip(("dq", "dk", "dv"), grads):
            err = _maxabs(t.float().cpu(), ref[name])
            assert err <= 1e-2, (name, det, err)
    _, lse = fa.varlen_attention_forward(q.cuda(), k.cuda(), v.cuda(), cq, cq, max(lens), max(lens), True,
                                         d ** -0.5, window)
    assert _maxabs(lse.cpu().numpy(), ref["lse2"]) <= 1e-3
    assert fa._abi.device_status() == 0
