"""Attention dropout on the B200 kernels.

The reference has none (README.md:93); PyTorch's SDPA ``dropout_p`` is the
model: the softmax probabilities are dropped at rate p and the kept ones
scaled by 1 / (1 - p), in the forward and consistently in the backward.

The keep pattern is a stateless function of a 64-bit seed and the position
(batch, head, query, key), evaluated inside the kernels (include/fa_b200.h
states it exactly), so nothing of size N^2 is stored: the forward and the
backward of one step regenerate it from the seed the autograd Function
saves.  p is applied in steps of 1/256 (t = round(256 p) of 256 random byte
values are dropped), and the scale is 256 / (256 - t), so the expectation is
exact for the p actually applied.  The seed comes from PyTorch's default
CPU generator, so ``torch.manual_seed`` makes runs repeatable.  The backward
runs the separate dQ and dK/dV kernels (bitwise reproducible).  The seed is
a kernel argument: a CUDA graph captured around a dropout call replays the
pattern it was captured with; call the functions below with a new seed per
step to draw new patterns outside a graph.
"""

from __future__ import annotations

import torch

from . import _abi


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def new_dropout_seed() -> int:
    """A 63-bit seed from PyTorch's default CPU generator."""
    return int(torch.randint(0, 2 ** 63 - 1, (1,), dtype=torch.int64).item())


def attention_forward_dropout(q, k, v, causal: bool, softmax_scale: float, dropout_p: float, seed: int):
    """Forward with dropout: returns (o, lse2); lse2 is that of the undropped
    probabilities.  v may be narrower or wider than q (32/64/128)."""
    b, hq, nq, d = q.shape
    hkv, nk, dv = k.shape[1], k.shape[2], v.shape[3]
    o = torch.empty((b, hq, nq, dv), device=q.device, dtype=q.dtype)
    lse = torch.empty((b, hq, nq), device=q.device, dtype=torch.float32)
    rc = _abi.entry("fa_fwd_dropout", q.dtype)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), b, hq, hkv, nq, nk, d, dv,
        _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o),
        float(dropout_p), int(seed), float(softmax_scale), 1 if causal else 0, _stream_handle(q.device))
    _abi.check(rc, "fa_fwd_dropout")
    return o, lse


def attention_backward_dropout(q, k, v, o, do, lse, causal: bool, softmax_scale: float, dropout_p: float,
                               seed: int):
    """dQ, dK, dV of attention_forward_dropout with the same seed."""
    b, hq, nq, d = q.shape
    hkv, nk, dv_dim = k.shape[1], k.shape[2], v.shape[3]
    delta = torch.empty((b, hq, nq), device=q.device, dtype=torch.float32)
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
    dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
    rc = _abi.entry("fa_bwd_dropout", q.dtype)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), delta.data_ptr(), b, hq, hkv, nq, nk, d, dv_dim,
        _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o), _abi.strides3(do),
        _abi.strides3(dq), _abi.strides3(dk), _abi.strides3(dv),
        float(dropout_p), int(seed), float(softmax_scale), 1 if causal else 0, _stream_handle(q.device))
    _abi.check(rc, "fa_bwd_dropout")
    return dq, dk, dv


class B200DropoutAttention(torch.autograd.Function):
    """Autograd bridge for attention with dropout: ``apply(q, k, v, causal,
    softmax_scale, dropout_p, seed)``; the seed is saved for the backward.
    Returns 7 gradients (None for the flag, scale, rate and seed)."""

    @staticmethod
    def forward(ctx, query, key, value, causal, softmax_scale, dropout_p, seed):
        output, lse = attention_forward_dropout(query, key, value, bool(causal), float(softmax_scale),
                                                float(dropout_p), int(seed))
        ctx.save_for_backward(query, key, value, output, lse)
        ctx.args = (bool(causal), float(softmax_scale), float(dropout_p), int(seed))
        return output

    @staticmethod
    def backward(ctx, grad_output):
        query, key, value, output, lse = ctx.saved_tensors
        causal, scale, p, seed = ctx.args
        dq, dk, dv = attention_backward_dropout(query, key, value, output, grad_output.contiguous(), lse, causal,
                                                scale, p, seed)
        return dq, dk, dv, None, None, None, None
