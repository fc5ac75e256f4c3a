"""CPU oracle for the FlashAttention-2 hot path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this module, and only as
the checker or as the timed CPU baseline.  The product path
(``triton_flash_attention_b200``) never imports it and fails loudly when its
CUDA library is missing.

Two restatements of the reference live here, both in numpy:

* ``sdpa_reference`` -- the dense scaled-dot-product-attention math that the
  reference's CPU path reaches through ``_torch_sdpa``
  (triton_flash_attention/attention.py:774-786, which forwards to
  ``torch.nn.functional.scaled_dot_product_attention``, torch 2.11.0 here;
  the published algorithm is softmax(scale * Q K^T + causal mask) V with its
  analytic gradient).  Computed in float64, it is the tolerance reference.
* ``fa2_forward`` / ``fa2_backward`` -- the reference's tiled FlashAttention-2
  algorithm as its Triton kernels run it: online softmax in the base-2 domain
  (attention.py:54-77), the base-2 log-sum-exp epilogue (attention.py:230),
  the Delta preprocess (attention.py:247-255), and the split dK/dV and dQ
  sweeps with fp16 rounding of P and dS before each product
  (attention.py:281-306, 334-348, 428-573).

Parity is pinned: ``tests/test_oracle_golden.py`` checks both restatements
against golden vectors that ``tests/golden/make_golden.py`` produced by running
the reference's own Triton kernels (interpreter mode, on CPU).
"""

from __future__ import annotations

import math

import numpy as np

LN2 = math.log(2.0)
INV_LN2 = 1.0 / LN2


def _group(hq: int, hkv: int) -> int:
    if hq % hkv != 0:
        raise ValueError("the number of query heads must be divisible by the number of key/value heads")
    return hq // hkv


def _expand_kv(x: np.ndarray, hq: int) -> np.ndarray:
    """Repeat each K/V head for its query group: kv_head = q_head // (Hq/Hkv)
    (attention.py:128-131)."""
    g = _group(hq, x.shape[1])
    return np.repeat(x, g, axis=1)


def _reduce_kv(dx: np.ndarray, hkv: int) -> np.ndarray:
    b, hq, n, d = dx.shape
    g = _group(hq, hkv)
    return dx.reshape(b, hkv, g, n, d).sum(axis=2)


def causal_mask(nq: int, nk: int, q_offset: int = 0, k_offset: int = 0, window: int = 0) -> np.ndarray:
    """True where a key is visible: key position <= query position.

    With zero offsets and nq == nk this is the reference's ``row >= col``
    (attention.py:65, 300, 343), the same as SDPA ``is_causal`` top-left
    alignment.  The offsets give the global positions of a sequence chunk.
    ``window`` > 0 adds a sliding window (no counterpart in the reference):
    only the ``window`` keys ending at the query's position are visible."""
    qi = np.arange(nq)[:, None] + q_offset
    kj = np.arange(nk)[None, :] + k_offset
    m = kj <= qi
    if window > 0:
        m &= kj > qi - window
    return m


def sdpa_reference(q, k, v, *, causal: bool, scale: float | None = None, do=None,
                   q_offset: int = 0, k_offset: int = 0, window: int = 0, mask=None,
                   dropout_keep=None, dropout_scale: float = 1.0):
    """Dense attention in float64 (the math behind attention.py:774-786).

    ``mask`` (optional) is a bool array broadcastable to (B, Hq, Nq, Nk):
    False hides the key, as ``attn_mask`` of PyTorch's SDPA (combined with
    ``causal`` by AND).  ``dropout_keep`` (optional, (B, Hq, Nq, Nk) bool)
    applies attention dropout: O = (P Z r) V with Z the keep pattern and r
    ``dropout_scale``; then dV = (P Z r)^T dO, dS = P (Z r dP - Delta) with
    Delta = rowsum(O dO), and lse is that of the undropped P.

    Returns a dict with ``o``, ``lse`` (natural log), ``lse2`` (base-2 log of
    the row sum of exp2(scale*log2(e)*s), the unit the reference saves,
    attention.py:177,230) and, when ``do`` is given, ``delta``, ``dq``, ``dk``,
    ``dv``.  Rows whose keys are all masked get o = 0 and lse = -inf."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    b, hq, nq, d = q.shape
    hkv = k.shape[1]
    nk = k.shape[2]
    if scale is None:
        scale = d ** -0.5
    ke = _expand_kv(k, hq)
    ve = _expand_kv(v, hq)
    s = np.einsum("bhqd,bhkd->bhqk", q, ke) * scale
    if causal:
        m = causal_mask(nq, nk, q_offset, k_offset, window)
        s = np.where(m[None, None], s, -np.inf)
    if mask is not None:
        s = np.where(np.broadcast_to(np.asarray(mask, dtype=bool), s.shape), s, -np.inf)
    mx = s.max(axis=-1, keepdims=True)
    mx_safe = np.where(np.isfinite(mx), mx, 0.0)
    e = np.exp(s - mx_safe)
    l = e.sum(axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        p = np.where(l > 0, e / np.where(l > 0, l, 1.0), 0.0)
        lse = np.where(l[..., 0] > 0, mx_safe[..., 0] + np.log(np.where(l[..., 0] > 0, l[..., 0], 1.0)), -np.inf)
    zr = 1.0 if dropout_keep is None else np.asarray(dropout_keep, dtype=np.float64) * dropout_scale
    pd = p * zr
    o = np.einsum("bhqk,bhkd->bhqd", pd, ve)
    out = {"o": o, "lse": lse, "lse2": lse * INV_LN2}
    if do is not None:
        do = np.asarray(do, dtype=np.float64)
        delta = (o * do).sum(axis=-1)
        dp = np.einsum("bhqd,bhkd->bhqk", do, ve)
        ds = p * (dp * zr - delta[..., None])
        dq = np.einsum("bhqk,bhkd->bhqd", ds, ke) * scale
        dke = np.einsum("bhqk,bhqd->bhkd", ds, q) * scale
        dve = np.einsum("bhqk,bhqd->bhkd", pd, do)
        out.update(delta=delta, dq=dq, dk=_reduce_kv(dke, hkv), dv=_reduce_kv(dve, hkv))
    return out


def _mix32(x):
    """The "lowbias32" integer hash (C. Wellons, hash-prospector): xorshift
    16, multiply by 0x7feb352d, xorshift 15, multiply by 0x846ca68b,
    xorshift 16, all modulo 2**32."""
    x = np.asarray(x, dtype=np.uint32)
    x = x ^ (x >> np.uint32(16))
    x = x * np.uint32(0x7FEB352D)
    x = x ^ (x >> np.uint32(15))
    x = x * np.uint32(0x846CA68B)
    x = x ^ (x >> np.uint32(16))
    return x


def dropout_threshold(dropout_p: float):
    """(t, r): the library applies p as t / 256, t = round(256 p) (half to
    even, on the float32 value of p) clamped to [1, 255], and scales kept
    values by r = 256 / (256 - t)."""
    t = int(round(float(np.float32(dropout_p)) * 256.0))
    t = min(max(t, 1), 255)
    return t, 256.0 / (256 - t)


def dropout_keep_reference(seed: int, batch: int, heads: int, nq: int, nk: int, dropout_p: float):
    """The library's dropout pattern (fa_fwd_dropout / fa_bwd_dropout): a
    bool (batch, heads, nq, nk) array, True where the probability is kept.
    One 32-bit word per 2 x 2 block of (query, key) positions; the
    position's byte is byte 2 (q & 1) + (k & 1) of it, kept iff byte >= t.
    No counterpart in the reference (it has no dropout, README.md:93)."""
    t, _ = dropout_threshold(dropout_p)
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    lo, hi = np.uint32(seed & 0xFFFFFFFF), np.uint32(seed >> 32)
    bh = np.arange(batch * heads, dtype=np.uint32).reshape(batch, heads)
    key_bh = _mix32(lo ^ _mix32(hi + bh * np.uint32(0x9E3779B9)))
    q = np.arange(nq, dtype=np.uint32)[:, None]
    k = np.arange(nk, dtype=np.uint32)[None, :]
    key2 = _mix32(key_bh[..., None, None] ^ (((q >> np.uint32(17)) << np.uint32(16)) | (k >> np.uint32(17))))
    ctr = (((q >> np.uint32(1)) & np.uint32(0xFFFF)) << np.uint32(16)) | ((k >> np.uint32(1)) & np.uint32(0xFFFF))
    word = _mix32(key2 ^ ctr)
    shift = np.uint32(8) * (np.uint32(2) * (q & np.uint32(1)) + (k & np.uint32(1)))
    byte = (word >> shift) & np.uint32(0xFF)
    return byte >= np.uint32(t)


def mask_bits_reference(mask):
    """The bit rows the library packs a bool mask (Bm, Hm, Nq, Nk) into
    (fa_mask_pack): ``bits`` (Bm, Hm, Nq, Wk) with bit k & 31 of word k >> 5
    of row q set iff mask[..., q, k], and ``bits_t`` (Bm, Hm, Nk, Wq) its
    transpose; Wk = roundup(Nk, 128) / 32, Wq likewise, padding bits zero.
    No counterpart in the reference (it has no masks, README.md:93)."""
    m = np.asarray(mask, dtype=bool)
    bm, hm, nq, nk = m.shape
    weights = np.left_shift(np.uint64(1), np.arange(32, dtype=np.uint64))

    def pack(rows, n_rows, n_cols):
        words = (n_cols + 127) // 128 * 4
        padded = np.zeros((bm, hm, n_rows, words * 32), dtype=np.uint64)
        padded[..., :n_cols] = rows
        return (padded.reshape(bm, hm, n_rows, words, 32) * weights).sum(axis=-1).astype(np.uint32)

    return pack(m, nq, nk), pack(np.swapaxes(m, 2, 3), nk, nq)


def sdpa_varlen_reference(q, k, v, cu_q, cu_k, *, causal: bool, scale: float | None = None, do=None,
                          window: int = 0):
    """Packed variable-length attention in float64: ``q`` (total_q, Hq, D),
    ``k``/``v`` (total_k, Hkv, D), prefix sums ``cu_q``/``cu_k``; each
    sequence is dense attention over its own rows (``sdpa_reference``, causal
    top-left aligned per sequence).  Returns packed ``o``, ``dq``, ``dk``,
    ``dv`` and ``lse2`` laid out (Hq, total_q).  No counterpart in the
    reference, which has no packed layout; this is its dense math applied per
    sequence."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    total_q, hq, d = q.shape
    if scale is None:
        scale = d ** -0.5
    out = {"o": np.zeros_like(q), "lse2": np.full((hq, total_q), -np.inf)}
    if do is not None:
        do = np.asarray(do, dtype=np.float64)
        out.update(dq=np.zeros_like(q), dk=np.zeros_like(k), dv=np.zeros_like(v))
    for b in range(len(cu_q) - 1):
        q0, q1, k0, k1 = int(cu_q[b]), int(cu_q[b + 1]), int(cu_k[b]), int(cu_k[b + 1])
        if q1 == q0 or k1 == k0:
            continue  # no query rows, or no keys: o = 0, lse = -inf, no gradient
        to4 = lambda x: x.transpose(1, 0, 2)[None]  # (n, H, D) -> (1, H, n, D)
        r = sdpa_reference(to4(q[q0:q1]), to4(k[k0:k1]), to4(v[k0:k1]), causal=causal, scale=scale,
                           do=None if do is None else to4(do[q0:q1]), window=window)
        out["o"][q0:q1] = r["o"][0].transpose(1, 0, 2)
        out["lse2"][:, q0:q1] = r["lse2"][0]
        if do is not None:
            out["dq"][q0:q1] = r["dq"][0].transpose(1, 0, 2)
            out["dk"][k0:k1] = r["dk"][0].transpose(1, 0, 2)
            out["dv"][k0:k1] = r["dv"][0].transpose(1, 0, 2)
    return out


def sdpa_paged_reference(q, k_cache, v_cache, block_table, cu_q, seqlens_k, *, causal: bool,
                         scale: float | None = None, window: int = 0):
    """Forward over a paged K/V cache in float64: sequence b's keys are rows
    0..seqlens_k[b]-1 of its pages block_table[b, :] laid end to end; its
    queries are the last nq positions (causal bottom-right aligned:
    sdpa_reference with q_offset = nk - nq).  Returns packed ``o`` and
    ``lse2`` (Hq, total_q).  No counterpart in the reference (no cache)."""
    q = np.asarray(q, dtype=np.float64)
    k_cache = np.asarray(k_cache, dtype=np.float64)
    v_cache = np.asarray(v_cache, dtype=np.float64)
    total_q, hq, d = q.shape
    page = k_cache.shape[1]
    if scale is None:
        scale = d ** -0.5
    out = {"o": np.zeros_like(q), "lse2": np.full((hq, total_q), -np.inf)}
    for b in range(len(cu_q) - 1):
        q0, q1, nk = int(cu_q[b]), int(cu_q[b + 1]), int(seqlens_k[b])
        nq = q1 - q0
        if nq == 0 or nk == 0:
            continue
        pages = np.asarray(block_table[b][: (nk + page - 1) // page])
        k = k_cache[pages].reshape(-1, *k_cache.shape[2:])[:nk]
        v = v_cache[pages].reshape(-1, *v_cache.shape[2:])[:nk]
        to4 = lambda x: x.transpose(1, 0, 2)[None]
        r = sdpa_reference(to4(q[q0:q1]), to4(k), to4(v), causal=causal, scale=scale, q_offset=nk - nq,
                           window=window)
        out["o"][q0:q1] = r["o"][0].transpose(1, 0, 2)
        out["lse2"][:, q0:q1] = r["lse2"][0]
    return out


def _f16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def fa2_forward(q, k, v, *, causal: bool, scale: float, block_m: int = 64, block_n: int = 32):
    """Tiled forward as attention.py:90-234 runs it, in float32 numpy.

    Per query block: m = -inf, l = 1, acc = 0 (attention.py:173-175);
    qk_scale = scale / ln2 (:177); causal runs the off-diagonal stage then the
    masked diagonal stage (:179-211), non-causal one full stage (:212-228).
    Each K/V tile: s = q k^T * qk_scale, masked to -inf (:61-66);
    m' = max(m, rowmax s); p = exp2(s - m'); alpha = exp2(m - m');
    l = l * alpha + rowsum p; acc = acc * alpha + fp16(p) v (:68-74).
    Epilogue: lse2 = m + log2(l), o = fp16(acc / l) (:230-234).
    Returns (o as float16, lse2 as float32)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    b, hq, n, d = q.shape
    g = _group(hq, k.shape[1])
    qk_scale = np.float32(scale * INV_LN2)
    o = np.zeros((b, hq, n, d), np.float16)
    lse2 = np.zeros((b, hq, n), np.float32)
    for bi in range(b):
        for h in range(hq):
            kh, vh = k[bi, h // g], v[bi, h // g]
            for m0 in range(0, n, block_m):
                rows = np.arange(m0, m0 + block_m)
                qt = np.zeros((block_m, d), np.float32)
                valid_rows = rows < n
                qt[valid_rows] = q[bi, h, rows[valid_rows]]
                m_i = np.full(block_m, -np.inf, np.float32)
                l_i = np.ones(block_m, np.float32)
                acc = np.zeros((block_m, d), np.float32)
                if causal:
                    stages = [(0, m0, False), (m0, m0 + block_m, True)]
                else:
                    stages = [(0, n, False)]
                for lo, hi, diag in stages:
                    for n0 in range(lo, hi, block_n):
                        cols = np.arange(n0, n0 + block_n)
                        kt = np.zeros((block_n, d), np.float32)
                        vt = np.zeros((block_n, d), np.float32)
                        vc = cols < n
                        kt[vc] = kh[cols[vc]]
                        vt[vc] = vh[cols[vc]]
                        s = (qt @ kt.T) * qk_scale
                        valid = np.broadcast_to(vc[None, :], s.shape)
                        if diag:
                            valid = valid & (rows[:, None] >= cols[None, :])
                        s = np.where(valid, s, -np.inf).astype(np.float32)
                        m_ij = np.maximum(m_i, s.max(axis=1))
                        p = np.exp2(s - m_ij[:, None]).astype(np.float32)
                        alpha = np.exp2(m_i - m_ij).astype(np.float32)
                        l_i = l_i * alpha + p.sum(axis=1)
                        acc = acc * alpha[:, None] + _f16(p) @ vt
                        m_i = m_ij
                lse_t = m_i + np.log2(l_i)
                out_t = acc / l_i[:, None]
                o[bi, h, rows[valid_rows]] = out_t[valid_rows].astype(np.float16)
                lse2[bi, h, rows[valid_rows]] = lse_t[valid_rows]
    return o, lse2


def fa2_delta(o, do):
    """Delta_i = sum_d O_id * dO_id in float32 (attention.py:247-255)."""
    return (np.asarray(o, np.float32) * np.asarray(do, np.float32)).sum(axis=-1, dtype=np.float32)


def fa2_backward(q, k, v, o, lse2, do, *, causal: bool, scale: float,
                 block_macro: int = 64, block_micro: int = 16):
    """Split backward as attention.py:377-573 runs it, in float32 numpy.

    dK/dV sweep (attention.py:428-505, inner loop :281-306): k_scaled =
    fp16(k * scale / ln2); per query micro tile s^T = k_scaled q^T,
    p^T = exp2(s^T - lse2) masked for invalid queries and, on the diagonal,
    kv > q; dv += fp16(p^T) dO; dp^T = v dO^T; ds^T = p^T (dp^T - Delta) ln2;
    dk += fp16(ds^T) q; finally dk *= scale / ln2 (:499).  The dQ sweep
    (:507-573, inner loop :334-348) is the mirror image with q_scaled.
    GQA sums each query head's dK/dV into its K/V head (the reference does so
    with atomics, :503-505).  Returns (dq, dk, dv) as float16 and Delta."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    do = np.asarray(do, np.float32)
    lse2 = np.asarray(lse2, np.float32)
    b, hq, n, d = q.shape
    hkv = k.shape[1]
    g = _group(hq, hkv)
    c = np.float32(scale * INV_LN2)
    ln2 = np.float32(0.6931471824645996)
    delta = fa2_delta(o, do)
    dq = np.zeros((b, hq, n, d), np.float32)
    dk = np.zeros((b, hkv, n, d), np.float32)
    dv = np.zeros((b, hkv, n, d), np.float32)
    padded = -(-n // block_macro) * block_macro

    def pad_rows(x, start, count):
        idx = np.arange(start, start + count)
        out = np.zeros((count,) + x.shape[1:], np.float32)
        ok = idx < n
        out[ok] = x[idx[ok]]
        return out, idx, ok

    for bi in range(b):
        for h in range(hq):
            kvh = h // g
            qh, doh, lh, dh = q[bi, h], do[bi, h], lse2[bi, h], delta[bi, h]
            kh, vh = k[bi, kvh], v[bi, kvh]
            for s0 in range(0, n, block_macro):
                # dK/dV for kv rows [s0, s0 + block_macro)
                kt, kv_idx, kv_ok = pad_rows(kh, s0, block_macro)
                vt, _, _ = pad_rows(vh, s0, block_macro)
                k_scaled = _f16(kt * c)
                dk_t = np.zeros((block_macro, d), np.float32)
                dv_t = np.zeros((block_macro, d), np.float32)
                if causal:
                    sweeps = [(s0, block_macro // block_micro, True),
                              (s0 + block_macro, (padded - s0 - block_macro) // block_micro, False)]
                else:
                    sweeps = [(0, -(-n // block_micro), False)]
                for q0, steps, diag in sweeps:
                    for st in range(steps):
                        qs = q0 + st * block_micro
                        qt, q_idx, q_ok = pad_rows(qh, qs, block_micro)
                        dot, _, _ = pad_rows(doh, qs, block_micro)
                        lse_t = np.where(q_ok, lh[np.minimum(q_idx, n - 1)], 0.0).astype(np.float32)
                        del_t = np.where(q_ok, dh[np.minimum(q_idx, n - 1)], 0.0).astype(np.float32)
                        s_t = k_scaled @ qt.T
                        p_t = np.exp2(s_t - lse_t[None, :]).astype(np.float32)
                        p_t = np.where(q_ok[None, :], p_t, 0.0)
                        if diag:
                            p_t = np.where(kv_idx[:, None] <= q_idx[None, :], p_t, 0.0)
                        dv_t += _f16(p_t) @ dot
                        dp_t = vt @ dot.T
                        ds_t = p_t * (dp_t - del_t[None, :]) * ln2
                        dk_t += _f16(ds_t) @ qt
                dk_t *= c
                dk[bi, kvh, kv_idx[kv_ok]] += dk_t[kv_ok]
                dv[bi, kvh, kv_idx[kv_ok]] += dv_t[kv_ok]
                # dQ for query rows [s0, s0 + block_macro)
                qt, q_idx, q_ok = pad_rows(qh, s0, block_macro)
                dot, _, _ = pad_rows(doh, s0, block_macro)
                lse_t = np.where(q_ok, lh[np.minimum(q_idx, n - 1)], 0.0).astype(np.float32)
                del_t = np.where(q_ok, dh[np.minimum(q_idx, n - 1)], 0.0).astype(np.float32)
                q_scaled = _f16(qt * c)
                dq_t = np.zeros((block_macro, d), np.float32)
                if causal:
                    sweeps = [(s0, block_macro // block_micro, True), (0, s0 // block_micro, False)]
                else:
                    sweeps = [(0, -(-n // block_micro), False)]
                for k0, steps, diag in sweeps:
                    for st in range(steps):
                        ks = k0 + st * block_micro
                        kt2, k_idx, k_ok = pad_rows(kh, ks, block_micro)
                        vt2, _, _ = pad_rows(vh, ks, block_micro)
                        s = q_scaled @ kt2.T
                        p = np.exp2(s - lse_t[:, None]).astype(np.float32)
                        p = np.where(k_ok[None, :], p, 0.0)
                        if diag:
                            p = np.where(q_idx[:, None] >= k_idx[None, :], p, 0.0)
                        dp = dot @ vt2.T
                        ds = p * (dp - del_t[:, None]) * ln2
                        dq_t += _f16(ds) @ kt2
                dq_t *= c
                dq[bi, h, q_idx[q_ok]] = dq_t[q_ok]
    return dq.astype(np.float16), dk.astype(np.float16), dv.astype(np.float16), delta


def merge_partials(o_parts, lse2_parts):
    """Merge partial attention outputs over disjoint key sets by their base-2
    log-sum-exp: L = log2(sum_i 2^{L_i}), O = sum_i O_i 2^{L_i - L}.

    This is the combine step of ring context parallelism (no counterpart in
    the reference, which runs one GPU); partials whose keys were all masked
    carry L_i = -inf and weigh zero."""
    lse = np.stack([np.asarray(x, np.float64) for x in lse2_parts])
    mx = lse.max(axis=0)
    mx_safe = np.where(np.isfinite(mx), mx, 0.0)
    w = np.exp2(lse - mx_safe[None])
    tot = w.sum(axis=0)
    with np.errstate(divide="ignore"):
        lse_out = np.where(tot > 0, mx_safe + np.log2(np.where(tot > 0, tot, 1.0)), -np.inf)
    o = sum(np.asarray(oi, np.float64) * (wi / np.where(tot > 0, tot, 1.0))[..., None]
            for oi, wi in zip(o_parts, w))
    return o, lse_out


def attention_block(q, k, v, *, causal: bool, scale: float, q_offset: int = 0, k_offset: int = 0):
    """Partial attention of local queries against one key/value block with
    global positions (float64): returns (o, lse2), the unit a ring step
    produces before merging."""
    r = sdpa_reference(q, k, v, causal=causal, scale=scale, q_offset=q_offset, k_offset=k_offset)
    return r["o"], r["lse2"]


def sdpa_head_fwd_bwd_fp32(q, k, v, do, *, causal: bool, scale: float):
    """One (batch, head) of dense attention forward + backward in float32
    with BLAS matmuls: the reference's CPU path (attention.py:774-786 ->
    PyTorch SDPA math) restated for timing the CPU baseline.  Inputs are
    (N, D) arrays; returns (o, dq, dk, dv)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    do = np.asarray(do, np.float32)
    n = q.shape[0]
    s = (q @ k.T) * np.float32(scale)
    if causal:
        s[np.triu_indices(n, 1, k.shape[0])] = -np.inf
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s, out=s)
    p /= p.sum(axis=1, keepdims=True)
    o = p @ v
    dp = do @ v.T
    delta = (o * do).sum(axis=1, keepdims=True)
    ds = p * (dp - delta)
    dq = (ds @ k) * np.float32(scale)
    dk = (ds.T @ q) * np.float32(scale)
    dv = p.T @ do
    return o, dq, dk, dv


def attention_block_grads(q, k, v, do, lse2, delta, *, causal: bool, scale: float,
                          q_offset: int = 0, k_offset: int = 0):
    """Gradient contributions of one key/value block given the GLOBAL
    base-2 LSE and Delta of the queries (float64): P = 2^(scale*log2(e)*s -
    lse2) on the block's visible keys, dS = P (dO V^T - Delta),
    dQ = scale dS K, dK = scale dS^T Q, dV = P^T dO (dK/dV summed over each
    K/V head's query group).  Summing these over all blocks gives the full
    gradient -- the decomposition a ring backward relies on."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    do = np.asarray(do, np.float64)
    lse2 = np.asarray(lse2, np.float64)
    delta = np.asarray(delta, np.float64)
    b, hq, nq, d = q.shape
    hkv, nk = k.shape[1], k.shape[2]
    ke = _expand_kv(k, hq)
    ve = _expand_kv(v, hq)
    s2 = np.einsum("bhqd,bhkd->bhqk", q, ke) * scale * INV_LN2
    with np.errstate(invalid="ignore"):
        p = np.exp2(s2 - np.where(np.isfinite(lse2), lse2, np.inf)[..., None])
    if causal:
        p = np.where(causal_mask(nq, nk, q_offset, k_offset)[None, None], p, 0.0)
    dp = np.einsum("bhqd,bhkd->bhqk", do, ve)
    ds = p * (dp - delta[..., None])
    dq = np.einsum("bhqk,bhkd->bhqd", ds, ke) * scale
    dke = np.einsum("bhqk,bhqd->bhkd", ds, q) * scale
    dve = np.einsum("bhqk,bhqd->bhkd", p, do)
    return dq, _reduce_kv(dke, hkv), _reduce_kv(dve, hkv)
