"""Packed variable-length attention on the B200 kernels.

No counterpart in the reference: its API takes ``(batch, heads, sequence,
head_dim)`` tensors whose sequences all have one length
(triton_flash_attention/attention.py:584-626).  Serving and packed-sequence
training hold a batch of sequences of different lengths back to back
instead: ``query`` is ``(total_q, Hq, D)``, ``key`` / ``value`` are
``(total_k, Hkv, D)``, and int32 prefix sums ``cu_seqlens_q`` /
``cu_seqlens_k`` (length ``B + 1``, starting at 0) say which rows belong to
which sequence.  Each sequence attends only to its own keys; the causal mask
is applied per sequence and top-left aligned (query ``i`` of a sequence sees
its keys ``j <= i``), like the dense call.

The same sm_100a kernels serve both layouts (the C ABI's ``fa_fwd_varlen`` /
``fa_bwd_varlen``); the saved log-sum-exp is ``(Hq, total_q)`` fp32.

``scaled_dot_product_attention_paged`` is the forward over a paged K/V cache
(``fa_fwd_paged``): packed queries as above, keys and values in
``(num_pages, page_size, Hkv, D)`` caches addressed by a block table, with
the KV-cache convention for the causal mask (bottom-right aligned: query
``i`` of ``nq`` sees keys ``j <= i + nk - nq``).
"""

from __future__ import annotations

import math
from numbers import Real

import torch

from . import _abi
from .attention import SUPPORTED_DTYPES, SUPPORTED_HEAD_DIMS, _stream_handle, fused_backward_enabled


def _validate_varlen(query, key, value, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, *,
                     enable_gqa: bool) -> None:
    tensors = {"query": query, "key": key, "value": value}
    for name, tensor in tensors.items():
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if tensor.ndim != 3:
            raise ValueError(f"{name} must have shape (total, heads, head_dim); got {tuple(tensor.shape)}")
        if tensor.shape[0] == 0 or tensor.shape[1] == 0 or tensor.shape[2] == 0:
            raise ValueError(f"{name} dimensions must all be greater than zero")
    for name, cu in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        if not isinstance(cu, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if cu.ndim != 1 or cu.numel() < 2 or cu.dtype != torch.int32:
            raise ValueError(f"{name} must be a 1-D int32 tensor of batch + 1 prefix sums")
        if cu.device != query.device:
            raise ValueError(f"{name} must be on the same device as query")
    if cu_seqlens_q.numel() != cu_seqlens_k.numel():
        raise ValueError("cu_seqlens_q and cu_seqlens_k must describe the same number of sequences")
    for name, m in (("max_seqlen_q", max_seqlen_q), ("max_seqlen_k", max_seqlen_k)):
        if isinstance(m, bool) or not isinstance(m, int) or m <= 0:
            raise ValueError(f"{name} must be a positive int")
    if query.device != key.device or query.device != value.device:
        raise ValueError("query, key, and value must be on the same device")
    if query.dtype != key.dtype or query.dtype != value.dtype:
        raise ValueError("query, key, and value must have the same dtype")
    if key.shape != value.shape:
        raise ValueError("key and value must have the same shape")
    if query.shape[2] != key.shape[2]:
        raise ValueError("query and key head dimensions must match")
    q_heads, kv_heads = query.shape[1], key.shape[1]
    if q_heads != kv_heads and not enable_gqa:
        raise ValueError(
            "query has a different number of heads from key/value; pass "
            "enable_gqa=True to use grouped-query attention")
    if q_heads % kv_heads != 0:
        raise ValueError("the number of query heads must be divisible by the number of key/value heads")
    if query.device.type != "cuda":
        raise RuntimeError("B200 CUDA backend is unavailable: the B200 kernel requires a CUDA tensor")
    if query.dtype not in SUPPORTED_DTYPES:
        raise RuntimeError("B200 CUDA backend is unavailable: the custom mixed-precision path currently "
                           "supports float16 and bfloat16")
    if query.shape[-1] not in SUPPORTED_HEAD_DIMS:
        supported = ", ".join(str(dim) for dim in SUPPORTED_HEAD_DIMS)
        raise RuntimeError(f"B200 CUDA backend is unavailable: head_dim must be one of ({supported}) "
                           "for the B200 path")
    if torch.cuda.get_device_capability(query.device) != (10, 0):
        raise RuntimeError("B200 CUDA backend is unavailable: the kernels are built for sm_100a (B200) GPUs only")


def varlen_attention_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q: int, max_seqlen_k: int,
                             causal: bool, softmax_scale: float, window: int = 0):
    """Forward over packed sequences: returns ``(o, lse2)`` with ``o`` like
    ``q`` and ``lse2`` the ``(Hq, total_q)`` base-2 log-sum-exp per row."""
    total_q, hq, d = q.shape
    total_k, hkv = k.shape[0], k.shape[1]
    batch = cu_seqlens_q.numel() - 1
    o = torch.empty_like(q)
    lse = torch.empty((hq, total_q), device=q.device, dtype=torch.float32)
    rc = _abi.entry("fa_fwd_varlen", q.dtype)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
        cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), batch, hq, hkv, int(max_seqlen_q), int(max_seqlen_k),
        total_q, total_k, d, float(softmax_scale), 1 if causal else 0, int(window), _stream_handle(q.device))
    _abi.check(rc, "fa_fwd_varlen")
    return o, lse


def varlen_attention_backward(q, k, v, o, do, lse, cu_seqlens_q, cu_seqlens_k, max_seqlen_q: int,
                              max_seqlen_k: int, causal: bool, softmax_scale: float, window: int = 0):
    """dQ, dK, dV over packed sequences.  Every head dim runs the fused
    pass (fp32 dQ accumulator in caller scratch) unless
    ``torch.use_deterministic_algorithms(True)`` asks for the separate,
    bitwise-reproducible dQ and dK/dV kernels."""
    total_q, hq, d = q.shape
    total_k, hkv = k.shape[0], k.shape[1]
    batch = cu_seqlens_q.numel() - 1
    fused = fused_backward_enabled(d)
    delta = torch.empty((hq, total_q), device=q.device, dtype=torch.float32)
    acc = torch.empty((hq, total_q, d), device=q.device, dtype=torch.float32) if fused else None
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    rc = _abi.entry("fa_bwd_varlen", q.dtype)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), delta.data_ptr(), acc.data_ptr() if fused else None,
        cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), batch, hq, hkv, int(max_seqlen_q), int(max_seqlen_k),
        total_q, total_k, d, float(softmax_scale), 1 if causal else 0, int(window), 0 if fused else 1,
        _stream_handle(q.device))
    _abi.check(rc, "fa_bwd_varlen")
    return dq, dk, dv


class B200VarlenAttention(torch.autograd.Function):
    """Autograd bridge for packed variable-length attention; saves
    (q, k, v, O, LSE) like the dense Function, plus the sequence offsets."""

    @staticmethod
    def forward(ctx, query, key, value, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal,
                softmax_scale, window=0):
        output, lse = varlen_attention_forward(query, key, value, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                               max_seqlen_k, bool(causal), float(softmax_scale), int(window))
        ctx.save_for_backward(query, key, value, output, lse, cu_seqlens_q, cu_seqlens_k)
        ctx.max_seqlen = (int(max_seqlen_q), int(max_seqlen_k))
        ctx.causal = bool(causal)
        ctx.softmax_scale = float(softmax_scale)
        ctx.window = int(window)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        query, key, value, output, lse, cu_q, cu_k = ctx.saved_tensors
        dq, dk, dv = varlen_attention_backward(query, key, value, output, grad_output.contiguous(), lse, cu_q, cu_k,
                                               *ctx.max_seqlen, ctx.causal, ctx.softmax_scale, ctx.window)
        return dq, dk, dv, None, None, None, None, None, None, None


def _window_arg(window_size, is_causal: bool) -> int:
    if window_size is None:
        return 0
    if isinstance(window_size, bool) or not isinstance(window_size, int) or window_size < 1:
        raise ValueError("window_size must be a positive int or None")
    if not is_causal:
        raise ValueError("window_size (a sliding window) requires is_causal=True")
    return window_size


def scaled_dot_product_attention_varlen(query, key, value, cu_seqlens_q, cu_seqlens_k, max_seqlen_q: int,
                                        max_seqlen_k: int, *, is_causal: bool = False, scale: float | None = None,
                                        enable_gqa: bool = False, window_size: int | None = None) -> torch.Tensor:
    """Attention over a batch of packed sequences of different lengths.

    ``query``: ``(total_q, Hq, D)``; ``key``, ``value``: ``(total_k, Hkv, D)``;
    ``cu_seqlens_q`` / ``cu_seqlens_k``: int32 prefix sums of the sequence
    lengths on the same device (``[0, n_0, n_0 + n_1, ...]``, ending at the
    totals); ``max_seqlen_q`` / ``max_seqlen_k``: at least the longest
    sequence's lengths.  Sequences may be empty.  Returns ``(total_q, Hq, D)``
    and supports autograd.  The default ``scale`` is ``D ** -0.5``.
    ``window_size`` (with ``is_causal``) is a sliding window: each query sees
    only the ``window_size`` keys ending at its own position."""
    if not isinstance(is_causal, bool):
        raise TypeError("is_causal must be a bool")
    if not isinstance(enable_gqa, bool):
        raise TypeError("enable_gqa must be a bool")
    if scale is not None and (not isinstance(scale, Real) or not math.isfinite(float(scale))):
        raise ValueError("scale must be a finite real number or None")
    window = _window_arg(window_size, is_causal)
    _validate_varlen(query, key, value, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                     enable_gqa=enable_gqa)
    softmax_scale = float(scale) if scale is not None else query.shape[-1] ** -0.5
    return B200VarlenAttention.apply(query.contiguous(), key.contiguous(), value.contiguous(),
                                     cu_seqlens_q.contiguous(), cu_seqlens_k.contiguous(), max_seqlen_q,
                                     max_seqlen_k, is_causal, softmax_scale, window)


# Most key-range splits of the paged forward's split-KV form, and the fewest
# 128-key tiles a range keeps.
MAX_KV_SPLITS = 16
MIN_TILES_PER_SPLIT = 2
_sm_count: dict[int, int] = {}


def gqa_pack(hq: int, hkv: int, max_seqlen_q: int) -> int:
    """Query heads the forward packs into one 128-row query tile (0: none),
    as the C library decides: a power-of-two group of 2 to 64 heads whose
    rows fit 256."""
    g = hq // hkv
    if g < 2 or g > 64 or g & (g - 1) or max_seqlen_q * g > 256:
        return 0
    return g


def kv_splits(units: int, key_tiles: int, sms: int) -> int:
    """How many key ranges the paged forward cuts each unit's keys into.

    The persistent forward runs ``units * s`` equal pieces over ``sms`` CTAs,
    so its time goes as ``ceil(units * s / sms) / s`` units' worth of keys.
    This returns the smallest ``s`` within 1 % of the best such time for
    ``s <= MAX_KV_SPLITS`` with at least ``MIN_TILES_PER_SPLIT`` key tiles
    per range.  Each range pays a query load, an output store and a combine
    pass, and a unit's 128-row tiles cost the same whatever the split, so
    splitting is kept for units that leave more than half the SMs idle
    (measured: 128 units on 148 SMs ran 8 % slower in 8 ranges); otherwise 1."""
    if units <= 0 or 2 * units > sms:
        return 1
    top = max(1, min(MAX_KV_SPLITS, key_tiles // MIN_TILES_PER_SPLIT))
    cost = {s: math.ceil(units * s / sms) / s for s in range(1, top + 1)}
    best = min(cost.values())
    return min(s for s, c in cost.items() if c <= best * 1.01)


def _sms(device: torch.device) -> int:
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index not in _sm_count:
        _sm_count[index] = torch.cuda.get_device_properties(index).multi_processor_count
    return _sm_count[index]


def paged_attention_forward(q, k_cache, v_cache, block_table, cu_seqlens_q, seqlens_k, max_seqlen_q: int,
                            max_seqlen_k: int, causal: bool, softmax_scale: float, window: int = 0,
                            num_splits: int | None = None):
    """Forward over a paged K/V cache: returns ``(o, lse2)`` like
    ``varlen_attention_forward``.

    With GQA packing and no window, few (sequence, K/V head) units leave SMs
    idle (decode of a few sequences): the keys of each unit are then cut
    into ``num_splits`` ranges (``kv_splits`` when None), each range's
    partial output goes to scratch, and ``fa_combine_splits`` merges them by
    their log-sum-exps."""
    total_q, hq, d = q.shape
    num_pages, page_size, hkv = k_cache.shape[0], k_cache.shape[1], k_cache.shape[2]
    batch = cu_seqlens_q.numel() - 1
    key_tiles = (int(max_seqlen_k) + 127) // 128
    pack = gqa_pack(hq, hkv, int(max_seqlen_q))
    if num_splits is None:
        n_qblk = -(-int(max_seqlen_q) // (256 // pack)) if pack else 0
        num_splits = kv_splits(batch * hkv * n_qblk, key_tiles, _sms(q.device)) if pack and not window else 1
    o = torch.empty_like(q)
    lse = torch.empty((hq, total_q), device=q.device, dtype=torch.float32)
    stream = _stream_handle(q.device)
    if num_splits > 1:
        o_part = torch.empty((num_splits, total_q, hq, d), device=q.device, dtype=q.dtype)
        lse_part = torch.empty((num_splits, hq, total_q), device=q.device, dtype=torch.float32)
        rc = _abi.entry("fa_fwd_paged_split", q.dtype)(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o_part.data_ptr(), lse_part.data_ptr(),
            cu_seqlens_q.data_ptr(), seqlens_k.data_ptr(), block_table.data_ptr(), batch, hq, hkv,
            int(max_seqlen_q), int(max_seqlen_k), total_q, num_pages, page_size, block_table.shape[1], d,
            float(softmax_scale), 1 if causal else 0, int(num_splits), stream)
        _abi.check(rc, "fa_fwd_paged_split")
        rc = _abi.entry("fa_combine_splits", q.dtype)(o_part.data_ptr(), lse_part.data_ptr(), o.data_ptr(),
                                                      lse.data_ptr(), int(num_splits), total_q, hq, d, stream)
        _abi.check(rc, "fa_combine_splits")
        return o, lse
    rc = _abi.entry("fa_fwd_paged", q.dtype)(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(), lse.data_ptr(),
        cu_seqlens_q.data_ptr(), seqlens_k.data_ptr(), block_table.data_ptr(), batch, hq, hkv,
        int(max_seqlen_q), int(max_seqlen_k), total_q, num_pages, page_size, block_table.shape[1], d,
        float(softmax_scale), 1 if causal else 0, int(window), stream)
    _abi.check(rc, "fa_fwd_paged")
    return o, lse


def scaled_dot_product_attention_paged(query, k_cache, v_cache, block_table, cu_seqlens_q, seqlens_k,
                                       max_seqlen_q: int, max_seqlen_k: int, *, is_causal: bool = False,
                                       scale: float | None = None, enable_gqa: bool = False,
                                       window_size: int | None = None,
                                       num_splits: int | None = None) -> torch.Tensor:
    """Attention of packed queries over a paged K/V cache (forward only).

    ``query``: ``(total_q, Hq, D)`` with ``cu_seqlens_q`` int32 prefix sums;
    ``k_cache``, ``v_cache``: ``(num_pages, page_size, Hkv, D)``, page_size a
    power of two >= 16; ``block_table``: int32 ``(B, max_pages_per_seq)``,
    the pages of each sequence in order; ``seqlens_k``: int32 ``(B,)`` key
    counts.  Cache rows past a sequence's length must be finite (a zeroed
    cache is).  ``is_causal`` aligns the mask bottom-right, so a sequence's
    queries are its last ``nq`` positions (decode: one query sees every
    key).  ``num_splits`` cuts each (sequence, K/V head) unit's keys into
    that many ranges merged by log-sum-exp (split-KV; GQA-packed queries and
    no window); None picks it from the SM count (``kv_splits``), 1 turns it
    off."""
    if not isinstance(is_causal, bool):
        raise TypeError("is_causal must be a bool")
    if not isinstance(enable_gqa, bool):
        raise TypeError("enable_gqa must be a bool")
    if scale is not None and (not isinstance(scale, Real) or not math.isfinite(float(scale))):
        raise ValueError("scale must be a finite real number or None")
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.ndim != 4:
            raise ValueError(f"{name} must have shape (num_pages, page_size, heads, head_dim); got {tuple(t.shape)}")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must have the same shape")
    page_size = k_cache.shape[1]
    if page_size < 16 or page_size & (page_size - 1):
        raise ValueError("page_size must be a power of two of at least 16")
    for name, t, nd in (("block_table", block_table, 2), ("seqlens_k", seqlens_k, 1)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.ndim != nd or t.dtype != torch.int32 or t.device != query.device:
            raise ValueError(f"{name} must be a {nd}-D int32 tensor on the query's device")
    batch = cu_seqlens_q.numel() - 1 if isinstance(cu_seqlens_q, torch.Tensor) else -1
    if block_table.shape[0] != batch or seqlens_k.numel() != batch:
        raise ValueError("block_table and seqlens_k must have one row per sequence of cu_seqlens_q")
    if any(t.requires_grad for t in (query, k_cache, v_cache)) and torch.is_grad_enabled():
        raise RuntimeError("the paged K/V path is forward only; run it under torch.no_grad()")
    if num_splits is not None and (isinstance(num_splits, bool) or not isinstance(num_splits, int) or
                                   not 1 <= num_splits <= 64):
        raise ValueError("num_splits must be an int from 1 to 64 or None")
    # the varlen checks on (query, one page of the cache seen as keys)
    kv_view = k_cache[0]
    window = _window_arg(window_size, is_causal)
    _validate_varlen(query, kv_view, kv_view, cu_seqlens_q, cu_seqlens_q, max_seqlen_q, max_seqlen_k,
                     enable_gqa=enable_gqa)
    softmax_scale = float(scale) if scale is not None else query.shape[-1] ** -0.5
    o, _ = paged_attention_forward(query.contiguous(), k_cache.contiguous(), v_cache.contiguous(),
                                   block_table.contiguous(), cu_seqlens_q.contiguous(), seqlens_k.contiguous(),
                                   max_seqlen_q, max_seqlen_k, is_causal, softmax_scale, window, num_splits)
    return o
