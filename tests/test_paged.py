"""Forward over a paged K/V cache (``scaled_dot_product_attention_paged``,
C ABI ``fa_fwd_paged``).

The reference has no cache; the oracle gathers each sequence's pages and
applies the dense float64 math with the KV-cache causal convention
(bottom-right aligned: ``sdpa_reference`` with ``q_offset = nk - nq``).  GPU
bars as for the dense forward: O within 2e-3 max-abs (fp16), lse2 within
1e-3; bf16 within twice PyTorch's bf16 SDPA error plus 2e-3.  Cases cover
page sizes 16 to 256, shuffled page tables, prefill over a longer cached
context, decode (one query per sequence), sequences whose last page is
partly filled, GQA and every head dim.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import triton_flash_attention_b200 as fa
from oracle import fa2_oracle as orc
from triton_flash_attention_b200 import varlen


def _case(lens_q, lens_k, page, hq, hkv, d, seed, dtype=torch.float16):
    rng = np.random.default_rng(seed)
    pages_per = [(n + page - 1) // page for n in lens_k]
    n_pages = sum(pages_per) + 3  # a few pages no sequence uses
    perm = rng.permutation(n_pages)
    width = max(max(pages_per), 1)
    table = np.zeros((len(lens_k), width), dtype=np.int32)  # unused entries: page 0 (never read)
    at = 0
    for b, p in enumerate(pages_per):
        table[b, :p] = perm[at:at + p]
        at += p
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(int(sum(lens_q)), hq, d, generator=g).to(dtype)
    kc = torch.randn(n_pages, page, hkv, d, generator=g).to(dtype)
    vc = torch.randn(n_pages, page, hkv, d, generator=g).to(dtype)
    cu_q = np.concatenate([[0], np.cumsum(lens_q)]).astype(np.int32)
    return q, kc, vc, table, cu_q, np.asarray(lens_k, dtype=np.int32)


def _run(q, kc, vc, table, cu_q, seqlens_k, causal, num_splits=None):
    dev = "cuda"
    with torch.no_grad():
        return fa.paged_attention_forward(
            q.to(dev), kc.to(dev), vc.to(dev), torch.from_numpy(table).to(dev), torch.from_numpy(cu_q).to(dev),
            torch.from_numpy(seqlens_k).to(dev), max(int(np.diff(cu_q).max()), 1), max(int(seqlens_k.max()), 1),
            causal, q.shape[-1] ** -0.5, num_splits=num_splits)


def _maxabs(a, b):
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())


# ---------------------------------------------------------------- CPU
def test_oracle_paged_matches_varlen_for_contiguous_pages():
    rng = np.random.default_rng(3)
    page, hq, d = 16, 2, 32
    lens = [37, 16, 5]
    q = rng.standard_normal((sum(lens), hq, d))
    k = rng.standard_normal((sum(lens), hq, d))
    v = rng.standard_normal((sum(lens), hq, d))
    # lay each sequence's keys into fresh pages, in order
    pages_per = [(n + page - 1) // page for n in lens]
    kc = np.zeros((sum(pages_per), page, hq, d))
    vc = np.zeros_like(kc)
    table = np.zeros((len(lens), max(pages_per)), dtype=np.int32)
    at, row = 0, 0
    for b, n in enumerate(lens):
        for p in range(pages_per[b]):
            m = min(page, n - p * page)
            kc[at, :m] = k[row + p * page: row + p * page + m]
            vc[at, :m] = v[row + p * page: row + p * page + m]
            table[b, p] = at
            at += 1
        row += n
    cu = np.concatenate([[0], np.cumsum(lens)])
    paged = orc.sdpa_paged_reference(q, kc, vc, table, cu, lens, causal=True)
    var = orc.sdpa_varlen_reference(q, k, v, cu, cu, causal=True)  # nq == nk: both alignments agree
    assert np.allclose(paged["o"], var["o"], atol=1e-12)
    assert np.allclose(paged["lse2"], var["lse2"], atol=1e-12)


def test_validation():
    q = torch.zeros(4, 2, 64, dtype=torch.float16)
    kc = torch.zeros(2, 16, 2, 64, dtype=torch.float16)
    cu = torch.tensor([0, 4], dtype=torch.int32)
    bt = torch.zeros(1, 2, dtype=torch.int32)
    sk = torch.tensor([20], dtype=torch.int32)
    with pytest.raises(ValueError, match="page_size"):
        fa.scaled_dot_product_attention_paged(q, kc[:, :12], kc[:, :12], bt, cu, sk, 4, 20)
    with pytest.raises(ValueError, match="block_table"):
        fa.scaled_dot_product_attention_paged(q, kc, kc, bt.long(), cu, sk, 4, 20)
    with pytest.raises(ValueError, match="one row per sequence"):
        fa.scaled_dot_product_attention_paged(q, kc, kc, bt.repeat(2, 1), cu, sk, 4, 20)
    with pytest.raises(RuntimeError, match="forward only"):
        fa.scaled_dot_product_attention_paged(q.requires_grad_(), kc, kc, bt, cu, sk, 4, 20)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        fa.scaled_dot_product_attention_paged(q.detach(), kc, kc, bt, cu, sk, 4, 20)
    for bad in (0, 65, True, 2.0):
        with pytest.raises(ValueError, match="num_splits"):
            fa.scaled_dot_product_attention_paged(q.detach(), kc, kc, bt, cu, sk, 4, 20, num_splits=bad)


def test_kv_splits_choice():
    """The split count minimises ceil(units * s / sms) / s (the persistent
    forward's waves per unit of keys), taking the smallest s within 1 %."""
    for units, tiles, sms in [(32, 64, 148), (16, 64, 148), (70, 64, 148), (60, 8, 148), (64, 4, 148)]:
        s = varlen.kv_splits(units, tiles, sms)
        top = max(1, min(varlen.MAX_KV_SPLITS, tiles // varlen.MIN_TILES_PER_SPLIT))
        assert 1 <= s <= top
        cost = [math.ceil(units * x / sms) / x for x in range(1, top + 1)]
        assert cost[s - 1] <= min(cost) * 1.01
        assert all(c > min(cost) * 1.01 for c in cost[: s - 1])
    assert varlen.kv_splits(16, 64, 148) == 9  # 144 pieces, one wave
    assert varlen.kv_splits(32, 64, 148) == 9  # 288 pieces, two waves
    # units filling more than half the SMs are not split
    assert varlen.kv_splits(75, 64, 148) == 1 and varlen.kv_splits(128, 64, 148) == 1
    assert varlen.kv_splits(32, 3, 148) == 1  # one range per unit keeps at least two key tiles


def test_gqa_pack_rule():
    """The Python side's packing rule equals the C library's: a power-of-two
    group of 2 to 64 heads with max_seqlen_q * group <= 256."""
    assert varlen.gqa_pack(32, 8, 1) == 4
    assert varlen.gqa_pack(32, 8, 64) == 4 and varlen.gqa_pack(32, 8, 65) == 0
    assert varlen.gqa_pack(32, 32, 1) == 0 and varlen.gqa_pack(24, 8, 1) == 0
    assert varlen.gqa_pack(128, 1, 1) == 0 and varlen.gqa_pack(64, 1, 4) == 64


# ---------------------------------------------------------------- GPU
CASES = [
    # lens_q, lens_k, page, hq, hkv, d, causal
    ([300, 37, 1, 128], [300, 1000, 77, 129], 16, 2, 2, 64, True),
    ([300, 37, 1, 128], [300, 1000, 77, 129], 64, 2, 2, 64, False),
    ([1, 1, 1, 1, 1], [5, 130, 257, 1, 64], 128, 4, 1, 128, True),
    ([200, 64], [513, 64], 256, 4, 2, 32, True),
    ([129, 250], [129, 700], 32, 2, 2, 128, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_paged_against_float64(case):
    lens_q, lens_k, page, hq, hkv, d, causal = case
    q, kc, vc, table, cu_q, seqlens_k = _case(lens_q, lens_k, page, hq, hkv, d, seed=sum(lens_k) + page)
    o, lse = _run(q, kc, vc, table, cu_q, seqlens_k, causal)
    torch.cuda.synchronize()
    ref = orc.sdpa_paged_reference(q.float().numpy(), kc.float().numpy(), vc.float().numpy(), table, cu_q,
                                   seqlens_k, causal=causal)
    assert _maxabs(o.float().cpu(), ref["o"]) <= 2e-3
    lse = lse.cpu().numpy()
    finite = np.isfinite(ref["lse2"])
    assert np.array_equal(np.isfinite(lse), finite)
    assert _maxabs(lse[finite], ref["lse2"][finite]) <= 1e-3
    assert fa._abi.device_status() == 0


@pytest.mark.gpu
def test_paged_bf16():
    lens_q, lens_k = [100, 1], [400, 33]
    q, kc, vc, table, cu_q, seqlens_k = _case(lens_q, lens_k, 64, 2, 2, 64, seed=9, dtype=torch.bfloat16)
    o, _ = _run(q, kc, vc, table, cu_q, seqlens_k, True)
    ref = orc.sdpa_paged_reference(q.float().numpy(), kc.float().numpy(), vc.float().numpy(), table, cu_q,
                                   seqlens_k, causal=True)
    # PyTorch's bf16 SDPA on the gathered keys, sequence by sequence, as the bar
    tq = torch.zeros_like(q, device="cuda")
    for b in range(len(lens_q)):
        q0, q1, nk = int(cu_q[b]), int(cu_q[b + 1]), int(seqlens_k[b])
        pages = torch.from_numpy(table[b, : (nk + 63) // 64]).long()
        k = kc[pages].reshape(-1, 2, 64)[:nk]
        v = vc[pages].reshape(-1, 2, 64)[:nk]
        nq = q1 - q0
        mask = torch.arange(nk)[None, :] <= torch.arange(nq)[:, None] + (nk - nq)
        ob = torch.nn.functional.scaled_dot_product_attention(
            q[q0:q1].transpose(0, 1)[None].cuda(), k.transpose(0, 1)[None].cuda(), v.transpose(0, 1)[None].cuda(),
            attn_mask=mask.cuda())
        tq[q0:q1] = ob[0].transpose(0, 1)
    err, terr = _maxabs(o.float().cpu(), ref["o"]), _maxabs(tq.float().cpu(), ref["o"])
    assert err <= 2 * terr + 2e-3, (err, terr)


@pytest.mark.gpu
def test_paged_matches_varlen_when_pages_are_contiguous():
    """Pages laid out in order with nq == nk: the paged forward equals the
    varlen forward bitwise (same tiles, same arithmetic)."""
    page, hq, d = 64, 4, 64
    lens = [300, 128, 1]
    g = torch.Generator(device="cpu").manual_seed(4)
    q, k, v = (torch.randn(sum(lens), hq, d, generator=g).half().cuda() for _ in range(3))
    pages_per = [(n + page - 1) // page for n in lens]
    kc = torch.zeros(sum(pages_per), page, hq, d, dtype=torch.half, device="cuda")
    vc = torch.zeros_like(kc)
    table = torch.zeros(len(lens), max(pages_per), dtype=torch.int32)
    at, row = 0, 0
    for b, n in enumerate(lens):
        for p in range(pages_per[b]):
            m = min(page, n - p * page)
            kc[at, :m] = k[row + p * page: row + p * page + m]
            vc[at, :m] = v[row + p * page: row + p * page + m]
            table[b, p] = at
            at += 1
        row += n
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device="cuda")
    sk = torch.tensor(lens, dtype=torch.int32, device="cuda")
    o_p, lse_p = fa.paged_attention_forward(q, kc, vc, table.cuda(), cu, sk, 300, 300, True, d ** -0.5)
    o_v, lse_v = fa.varlen_attention_forward(q, k, v, cu, cu, 300, 300, True, d ** -0.5)
    assert torch.equal(o_p, o_v)
    assert torch.equal(lse_p, lse_v)


@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv,nq", [(16, 2, 17), (32, 1, 5), (64, 1, 1), (8, 4, 100)])
def test_gqa_packed_forward_dense(hq, hkv, nq):
    """Short query sides with GQA run the packed forward (a query tile holds
    the group's heads); causal with Nq != Nk (top-left, the dense
    convention) and non-causal, against float64."""
    g = torch.Generator(device="cpu").manual_seed(hq + nq)
    d, nk = 64, 700
    q = torch.randn(2, hq, nq, d, generator=g).half()
    k = torch.randn(2, hkv, nk, d, generator=g).half()
    v = torch.randn(2, hkv, nk, d, generator=g).half()
    for causal in (False, True):
        o, lse = fa.attention_forward(q.cuda(), k.cuda(), v.cuda(), causal, d ** -0.5)
        ref = orc.sdpa_reference(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=causal,
                                 scale=d ** -0.5)
        assert _maxabs(o.float().cpu(), ref["o"]) <= 2e-3
        finite = np.isfinite(ref["lse2"])
        lse = lse.cpu().numpy()
        assert np.array_equal(np.isfinite(lse), finite)
        assert _maxabs(lse[finite], ref["lse2"][finite]) <= 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("lens_q,window", [([1, 1, 1], 100), ([200, 37], 64)])
def test_paged_sliding_window(lens_q, window):
    """Sliding window over a paged cache (bottom-right positions): decode and
    a prefill chunk, against float64."""
    lens_k = [1000, 300, 77][: len(lens_q)]
    q, kc, vc, table, cu_q, seqlens_k = _case(lens_q, lens_k, 64, 4, 2, 64, seed=window)
    with torch.no_grad():
        o, lse = fa.paged_attention_forward(
            q.cuda(), kc.cuda(), vc.cuda(), torch.from_numpy(table).cuda(), torch.from_numpy(cu_q).cuda(),
            torch.from_numpy(seqlens_k).cuda(), max(lens_q), max(lens_k), True, 64 ** -0.5, window)
    ref = orc.sdpa_paged_reference(q.float().numpy(), kc.float().numpy(), vc.float().numpy(), table, cu_q,
                                   seqlens_k, causal=True, window=window)
    assert _maxabs(o.float().cpu(), ref["o"]) <= 2e-3
    assert _maxabs(lse.cpu().numpy(), ref["lse2"]) <= 1e-3


# Split-KV (decode): each unit's keys cut into ranges merged by log-sum-exp.
SPLIT_CASES = [
    # lens_q, lens_k, page, hq, hkv, d, causal, splits
    ([1, 1, 1, 1, 1], [4000, 5, 1000, 129, 2300], 64, 32, 8, 128, True, 8),
    ([1, 1, 1], [700, 256, 33], 16, 8, 2, 64, True, 3),
    ([1, 1], [1300, 600], 128, 8, 4, 32, False, 5),
    ([4, 3], [1000, 300], 32, 16, 4, 128, True, 4),  # several queries: the causal limit crosses the ranges
    ([1, 1, 1, 1], [8192, 8192, 1, 4096], 64, 32, 8, 128, True, None),  # automatic count
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", SPLIT_CASES)
def test_paged_split_kv_against_float64(case):
    lens_q, lens_k, page, hq, hkv, d, causal, splits = case
    q, kc, vc, table, cu_q, seqlens_k = _case(lens_q, lens_k, page, hq, hkv, d, seed=sum(lens_k) + 7)
    o, lse = _run(q, kc, vc, table, cu_q, seqlens_k, causal, num_splits=splits)
    o1, lse1 = _run(q, kc, vc, table, cu_q, seqlens_k, causal, num_splits=1)
    torch.cuda.synchronize()
    ref = orc.sdpa_paged_reference(q.float().numpy(), kc.float().numpy(), vc.float().numpy(), table, cu_q,
                                   seqlens_k, causal=causal)
    assert _maxabs(o.float().cpu(), ref["o"]) <= 2e-3
    assert _maxabs(o.float().cpu(), o1.float().cpu()) <= 2e-3
    lse = lse.cpu().numpy()
    finite = np.isfinite(ref["lse2"])
    assert np.array_equal(np.isfinite(lse), finite)
    assert _maxabs(lse[finite], ref["lse2"][finite]) <= 1e-3
    assert _maxabs(lse[finite], lse1.cpu().numpy()[finite]) <= 1e-3
    assert fa._abi.device_status() == 0


@pytest.mark.gpu
def test_paged_split_kv_bf16():
    lens_q, lens_k = [1, 1, 1], [3000, 77, 1500]
    q, kc, vc, table, cu_q, seqlens_k = _case(lens_q, lens_k, 64, 16, 4, 64, seed=5, dtype=torch.bfloat16)
    o, _ = _run(q, kc, vc, table, cu_q, seqlens_k, True, num_splits=6)
    o1, _ = _run(q, kc, vc, table, cu_q, seqlens_k, True, num_splits=1)
    ref = orc.sdpa_paged_reference(q.float().numpy(), kc.float().numpy(), vc.float().numpy(), table, cu_q,
                                   seqlens_k, causal=True)
    err, err1 = _maxabs(o.float().cpu(), ref["o"]), _maxabs(o1.float().cpu(), ref["o"])
    # one more bf16 rounding (the partials) than the unsplit forward
    assert err <= 2 * err1 + 4e-3, (err, err1)
