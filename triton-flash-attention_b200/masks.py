"""Dense boolean attention masks on the B200 kernels.

The reference has none (README.md:93: "Dropout and arbitrary attention masks
are not currently implemented"); this module adds PyTorch SDPA's boolean
``attn_mask`` to ``scaled_dot_product_attention``.  ``True`` marks a key
that takes part, as in ``torch.nn.functional.scaled_dot_product_attention``;
the mask broadcasts to (batch, query heads, query length, key length) and
may be combined with ``is_causal`` (a key must pass both).

A mask is packed once per forward by a CUDA kernel (``fa_mask_pack``) into
two bit matrices: rows of query bits for the forward and dQ kernels, and the
transpose for the dK/dV kernels, whose threads own key rows.  A 128-key tile
of a row is one 16-byte load; broadcast batch or head dimensions stay
broadcast (word stride 0).  A query row that sees no key gets o = 0, lse =
-inf and zero gradients, where PyTorch's SDPA returns NaN.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _abi


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@dataclass(frozen=True)
class PackedMask:
    """A mask packed for the kernels: ``bits`` (Bm, Hm, Nq, Wk) and
    ``bits_t`` (Bm, Hm, Nk, Wq) int32 words, with their word strides
    {batch, head, row} (0 where the mask broadcasts)."""

    bits: torch.Tensor
    strides: tuple
    bits_t: torch.Tensor
    t_strides: tuple

    def c_strides(self):
        return (ctypes.c_int64 * 3)(*self.strides)

    def c_t_strides(self):
        return (ctypes.c_int64 * 3)(*self.t_strides)


def validate_attention_mask(attn_mask, query, key) -> None:
    """Type, dtype, device and shape checks of ``attn_mask``."""
    if not isinstance(attn_mask, torch.Tensor):
        raise TypeError("attn_mask must be a torch.Tensor or None")
    if attn_mask.dtype != torch.bool:
        raise ValueError("attn_mask must be a bool tensor (True = the key takes part); "
                         "additive float masks are not supported")
    if attn_mask.device != query.device:
        raise ValueError("attn_mask must be on the same device as query")
    b, hq, nq = query.shape[0], query.shape[1], query.shape[2]
    nk = key.shape[2]
    full = (b, hq, nq, nk)
    if attn_mask.ndim < 1 or attn_mask.ndim > 4 or any(
            m not in (1, f) for m, f in zip(attn_mask.shape[::-1], full[::-1])):
        raise ValueError(
            f"attn_mask of shape {tuple(attn_mask.shape)} does not broadcast to "
            f"(batch, query heads, query length, key length) = {full}")


def pack_attention_mask(attn_mask: torch.Tensor, batch: int, q_heads: int, nq: int, nk: int) -> PackedMask:
    """Pack a bool mask broadcastable to (batch, q_heads, nq, nk) with the
    library's fa_mask_pack kernel.  Batch and head dimensions of size 1 stay
    broadcast; query and key dimensions of size 1 are expanded."""
    m4 = attn_mask.reshape((1,) * (4 - attn_mask.ndim) + tuple(attn_mask.shape))
    bm, hm = m4.shape[0], m4.shape[1]
    m4 = m4.expand(bm, hm, nq, nk)
    wk = (nk + 127) // 128 * 4
    wq = (nq + 127) // 128 * 4
    bits = torch.empty((bm, hm, nq, wk), dtype=torch.int32, device=attn_mask.device)
    bits_t = torch.empty((bm, hm, nk, wq), dtype=torch.int32, device=attn_mask.device)
    rc = _abi.lib().fa_mask_pack(m4.data_ptr(), bm, hm, nq, nk, (ctypes.c_int64 * 4)(*m4.stride()),
                                 bits.data_ptr(), bits_t.data_ptr(), _stream_handle(attn_mask.device))
    _abi.check(rc, "fa_mask_pack")
    strides = (0 if bm == 1 else hm * nq * wk, 0 if hm == 1 else nq * wk, wk)
    t_strides = (0 if bm == 1 else hm * nk * wq, 0 if hm == 1 else nk * wq, wq)
    return PackedMask(bits, strides, bits_t, t_strides)


def attention_forward_masked(q, k, v, mask: PackedMask, causal: bool, softmax_scale: float):
    """Forward under a packed mask: returns (o, lse2) as attention_forward
    does; v may be narrower or wider than q (value head size 32/64/128)."""
    b, hq, nq, d = q.shape
    hkv, nk, dv = k.shape[1], k.shape[2], v.shape[3]
    o = torch.empty((b, hq, nq, dv), device=q.device, dtype=q.dtype)
    lse = torch.empty((b, hq, nq), device=q.device, dtype=torch.float32)
    rc = _abi.entry("fa_fwd_masked", q.dtype)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), b, hq, hkv, nq, nk, d, dv,
        _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o),
        mask.bits.data_ptr(), mask.c_strides(), float(softmax_scale), 1 if causal else 0,
        _stream_handle(q.device))
    _abi.check(rc, "fa_fwd_masked")
    return o, lse


def attention_backward_masked(q, k, v, o, do, lse, mask: PackedMask, causal: bool, softmax_scale: float):
    """dQ, dK, dV under a packed mask: the fused pass when max(D, Dv) <= 64
    and deterministic algorithms are off, else the separate dQ and dK/dV
    kernels (bitwise reproducible)."""
    b, hq, nq, d = q.shape
    hkv, nk, dv_dim = k.shape[1], k.shape[2], v.shape[3]
    width = max(d, dv_dim)
    deterministic = torch.are_deterministic_algorithms_enabled()
    delta = torch.empty((b, hq, nq), device=q.device, dtype=torch.float32)
    acc = None
    if width <= 64 and not deterministic:
        acc = torch.empty((b, hq, nq, width), device=q.device, dtype=torch.float32)
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
    dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
    rc = _abi.entry("fa_bwd_masked", q.dtype)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), delta.data_ptr(), acc.data_ptr() if acc is not None else None,
        b, hq, hkv, nq, nk, d, dv_dim,
        _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o), _abi.strides3(do),
        _abi.strides3(dq), _abi.strides3(dk), _abi.strides3(dv),
        mask.bits.data_ptr(), mask.c_strides(), mask.bits_t.data_ptr(), mask.c_t_strides(),
        float(softmax_scale), 1 if causal else 0, 1 if deterministic else 0, _stream_handle(q.device))
    _abi.check(rc, "fa_bwd_masked")
    return dq, dk, dv


class B200MaskedAttention(torch.autograd.Function):
    """Autograd bridge for masked attention: ``apply(q, k, v, attn_mask,
    causal, softmax_scale)``; the mask is packed once in the forward and the
    packed bits are saved for the backward.  Returns 6 gradients (None for
    the mask, the flag and the scale)."""

    @staticmethod
    def forward(ctx, query, key, value, attn_mask, causal, softmax_scale):
        b, hq, nq, _ = query.shape
        mask = pack_attention_mask(attn_mask, b, hq, nq, key.shape[2])
        output, lse = attention_forward_masked(query, key, value, mask, bool(causal), float(softmax_scale))
        ctx.save_for_backward(query, key, value, output, lse, mask.bits, mask.bits_t)
        ctx.mask_strides = (mask.strides, mask.t_strides)
        ctx.softmax_scale = float(softmax_scale)
        ctx.causal = bool(causal)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        query, key, value, output, lse, bits, bits_t = ctx.saved_tensors
        mask = PackedMask(bits, ctx.mask_strides[0], bits_t, ctx.mask_strides[1])
        dq, dk, dv = attention_backward_masked(query, key, value, output, grad_output.contiguous(), lse, mask,
                                               ctx.causal, ctx.softmax_scale)
        return dq, dk, dv, None, None, None
