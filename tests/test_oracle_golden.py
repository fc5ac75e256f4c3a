"""The oracle is pinned to the reference's own outputs (CPU).

``tests/golden/golden.npz`` holds outputs of the reference's Triton kernels
run on CPU by ``tests/golden/make_golden.py`` (Triton interpreter).  The tiled
restatement must reproduce them (forward bit-exact; backward within fp16
accumulation-order noise), and the float64 dense reference must agree with
them within the reference's own fp16 error."""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import fa2_oracle as orc

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
CASES = sorted({k.split("/")[0] for k in GOLDEN.files})


def _get(name):
    meta = GOLDEN[f"{name}/meta"]
    b, hq, hkv, n, d, causal, seed, bm, bn, bma, bmi = (int(x) for x in meta)
    arrays = {k: GOLDEN[f"{name}/{k}"] for k in ("q", "k", "v", "do", "o", "lse2", "delta", "dq", "dk", "dv")}
    return dict(b=b, hq=hq, hkv=hkv, n=n, d=d, causal=bool(causal), bm=bm, bn=bn, bma=bma, bmi=bmi), arrays


def _mx(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


@pytest.mark.parametrize("name", CASES)
def test_tiled_forward_is_bit_exact(name):
    m, g = _get(name)
    o, lse2 = orc.fa2_forward(g["q"], g["k"], g["v"], causal=m["causal"], scale=m["d"] ** -0.5,
                              block_m=m["bm"], block_n=m["bn"])
    assert np.array_equal(o, g["o"])
    assert np.array_equal(lse2, g["lse2"])


@pytest.mark.parametrize("name", CASES)
def test_tiled_backward_matches(name):
    m, g = _get(name)
    dq, dk, dv, delta = orc.fa2_backward(g["q"], g["k"], g["v"], g["o"], g["lse2"], g["do"],
                                         causal=m["causal"], scale=m["d"] ** -0.5,
                                         block_macro=m["bma"], block_micro=m["bmi"])
    assert np.array_equal(delta, g["delta"])
    # fp16 outputs; accumulation order differs from the interpreter's dot,
    # and GQA adds the reference's fp16 atomics rounding: a few ulps
    assert _mx(dq, g["dq"]) <= 1e-4
    assert _mx(dk, g["dk"]) <= 1e-4
    assert _mx(dv, g["dv"]) <= 1e-3


@pytest.mark.parametrize("name", CASES)
def test_dense_reference_agrees(name):
    m, g = _get(name)
    r = orc.sdpa_reference(g["q"], g["k"], g["v"], causal=m["causal"], scale=m["d"] ** -0.5, do=g["do"])
    assert _mx(r["o"], g["o"]) <= 1e-3
    assert _mx(r["lse2"], g["lse2"]) <= 1e-5
    for key in ("dq", "dk", "dv"):
        assert _mx(r[key], g[key]) <= 1e-3


def test_merge_partials_equals_full():
    """Splitting the keys in two blocks and merging by log-sum-exp gives the
    full result (the ring-context-parallel combine)."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 2, 40, 32))
    k = rng.standard_normal((1, 2, 64, 32))
    v = rng.standard_normal((1, 2, 64, 32))
    full = orc.sdpa_reference(q, k, v, causal=True, scale=0.2, q_offset=30)
    a = orc.attention_block(q, k[:, :, :20], v[:, :, :20], causal=True, scale=0.2, q_offset=30, k_offset=0)
    b = orc.attention_block(q, k[:, :, 20:], v[:, :, 20:], causal=True, scale=0.2, q_offset=30, k_offset=20)
    o, lse2 = orc.merge_partials([a[0], b[0]], [a[1], b[1]])
    assert _mx(o, full["o"]) < 1e-12
    assert _mx(lse2, full["lse2"]) < 1e-12


def test_head_fwd_bwd_fp32_port():
    rng = np.random.default_rng(1)
    q, k, v, do = (rng.standard_normal((70, 32)).astype(np.float16) for _ in range(4))
    o, dq, dk, dv = orc.sdpa_head_fwd_bwd_fp32(q, k, v, do, causal=True, scale=0.3)
    r = orc.sdpa_reference(q[None, None], k[None, None], v[None, None], causal=True, scale=0.3,
                           do=do[None, None])
    for a, key in ((o, "o"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        assert _mx(a, r[key][0, 0]) < 1e-4
