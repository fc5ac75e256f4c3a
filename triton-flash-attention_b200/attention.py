"""Public attention API, mirroring the reference's surface
(triton_flash_attention/attention.py:576-845) on top of the B200 kernels.

Same names, argument meaning and validation messages as the reference.  The
one deliberate difference is dispatch: the reference falls back to
``torch.nn.functional.scaled_dot_product_attention`` for inputs its kernel
does not serve; this package has a single backend -- the hand-written
sm_100a CUDA kernels -- and raises ``RuntimeError`` for every ineligible
input instead of falling back.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from numbers import Real
from typing import Literal

import torch

from . import _abi

SUPPORTED_HEAD_DIMS = (32, 64, 128)
# float16 is the reference's kernel dtype (attention.py:653-656); bfloat16 is
# served by the same kernels here, where the reference falls back to SDPA.
SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)
Backend = Literal["auto", "triton", "cuda"]
_BACKENDS = ("auto", "triton", "cuda")


@dataclass(frozen=True)
class DispatchDecision:
    """The selected backend and the concrete reason for the decision
    (attention.py:576-581).  ``backend`` is ``"cuda"`` when the B200 kernels
    serve the inputs and ``"unsupported"`` otherwise."""

    backend: Literal["cuda", "unsupported"]
    reason: str


def _validate_inputs(query, key, value, *, enable_gqa: bool) -> None:
    """Shape/device/dtype checks with the reference's messages
    (attention.py:584-626)."""
    tensors = {"query": query, "key": key, "value": value}
    for name, tensor in tensors.items():
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if tensor.ndim != 4:
            raise ValueError(
                f"{name} must have shape (batch, heads, sequence, head_dim); "
                f"got {tuple(tensor.shape)}")
        if any(dimension == 0 for dimension in tensor.shape):
            raise ValueError(f"{name} dimensions must all be greater than zero")
    if query.device != key.device or query.device != value.device:
        raise ValueError("query, key, and value must be on the same device")
    if query.dtype != key.dtype or query.dtype != value.dtype:
        raise ValueError("query, key, and value must have the same dtype")
    if query.shape[0] != key.shape[0] or key.shape[0] != value.shape[0]:
        raise ValueError("query, key, and value batch dimensions must match")
    if key.shape[:3] != value.shape[:3]:
        raise ValueError("key and value batch, head, and sequence dimensions must match")
    if query.shape[3] != key.shape[3]:
        raise ValueError("query and key head dimensions must match")
    q_heads, kv_heads = query.shape[1], key.shape[1]
    if q_heads != kv_heads and not enable_gqa:
        raise ValueError(
            "query has a different number of heads from key/value; pass "
            "enable_gqa=True to use grouped-query attention")
    if q_heads % kv_heads != 0:
        raise ValueError(
            "the number of query heads must be divisible by the number of "
            "key/value heads")


_capability: dict = {}


def _device_capability(device: torch.device) -> tuple[int, int]:
    """(major, minor) compute capability of a CUDA device, queried once per
    device index."""
    index = getattr(device, "index", None)
    if index is None:
        return torch.cuda.get_device_capability(device)
    cap = _capability.get(index)
    if cap is None:
        cap = _capability[index] = torch.cuda.get_device_capability(device)
    return cap


def explain_dispatch(query, key, value, *, enable_gqa: bool = False) -> DispatchDecision:
    """Explain whether the B200 kernels can serve these inputs
    (attention.py:629-670).  Query and key lengths may differ (the causal
    mask is then top-left aligned, as in PyTorch's SDPA), and so may the
    query/key and value head sizes (the reference sends both to PyTorch,
    attention.py:639-646); each head size must be 32, 64 or 128."""
    _validate_inputs(query, key, value, enable_gqa=enable_gqa)
    return _dispatch(query, value)


def _dispatch(query, value) -> DispatchDecision:
    """The dispatch decision for inputs that passed ``_validate_inputs``."""
    if query.device.type != "cuda":
        return DispatchDecision("unsupported", "the B200 kernel requires a CUDA tensor")
    if torch.version.hip is not None:
        return DispatchDecision("unsupported", "this project targets NVIDIA CUDA, not ROCm")
    if query.dtype not in SUPPORTED_DTYPES:
        return DispatchDecision(
            "unsupported", "the custom mixed-precision path currently supports float16 and bfloat16")
    supported = ", ".join(str(dim) for dim in SUPPORTED_HEAD_DIMS)
    if query.shape[-1] not in SUPPORTED_HEAD_DIMS:
        return DispatchDecision(
            "unsupported", f"head_dim must be one of ({supported}) for the B200 path")
    if value.shape[-1] not in SUPPORTED_HEAD_DIMS:
        return DispatchDecision(
            "unsupported", f"the value head_dim must be one of ({supported}) for the B200 path")
    major, minor = _device_capability(query.device)
    if (major, minor) != (10, 0):
        return DispatchDecision(
            "unsupported", "the kernels are built for sm_100a (B200) GPUs only")
    return DispatchDecision(
        "cuda", f"CUDA {str(query.dtype).replace('torch.', '')} attention on sm_100a with a supported head dimension")


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def attention_forward(q, k, v, causal: bool, softmax_scale: float, *, q_offset: int = 0, k_offset: int = 0):
    """Launch the forward kernel: returns (o, lse2) with lse2 the base-2
    log-sum-exp per query row in the scaled domain (attention.py:230)."""
    b, hq, nq, d = q.shape
    hkv, nk = k.shape[1], k.shape[2]
    if v.shape[-1] != d:
        if q_offset or k_offset:
            raise ValueError("position offsets need equal query/key and value head sizes")
        return attention_forward_vdim(q, k, v, causal, softmax_scale)
    o = torch.empty(q.shape, device=q.device, dtype=q.dtype)  # contiguous even for strided q
    lse = torch.empty((b, hq, nq), device=q.device, dtype=torch.float32)
    rc = _abi.entry("fa_fwd", q.dtype)(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                    b, hq, hkv, nq, nk, d,
                    _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o),
                    float(softmax_scale), 1 if causal else 0, int(q_offset), int(k_offset),
                    _stream_handle(q.device))
    _abi.check(rc, "fa_fwd")
    return o, lse


def attention_forward_vdim(q, k, v, causal: bool, softmax_scale: float):
    """Forward with a value head size Dv different from the query/key head
    size D: returns o (B, Hq, Nq, Dv) and lse2 as attention_forward does.
    The kernels run at width max(D, Dv) with the narrower operands' missing
    columns read as zeros."""
    b, hq, nq, d = q.shape
    hkv, nk, dv = k.shape[1], k.shape[2], v.shape[3]
    o = torch.empty((b, hq, nq, dv), device=q.device, dtype=q.dtype)
    lse = torch.empty((b, hq, nq), device=q.device, dtype=torch.float32)
    rc = _abi.entry("fa_fwd_vdim", q.dtype)(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                            b, hq, hkv, nq, nk, d, dv,
                                            _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o),
                                            float(softmax_scale), 1 if causal else 0, _stream_handle(q.device))
    _abi.check(rc, "fa_fwd_vdim")
    return o, lse


def attention_backward_vdim(q, k, v, o, do, lse, causal: bool, softmax_scale: float):
    """dQ, dK (D wide) and dV (Dv wide) for attention_forward_vdim: the fused
    pass when max(D, Dv) <= 64 and deterministic algorithms are off, else the
    separate dQ and dK/dV kernels."""
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
    rc = _abi.entry("fa_bwd_vdim", q.dtype)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), delta.data_ptr(), acc.data_ptr() if acc is not None else None,
        b, hq, hkv, nq, nk, d, dv_dim,
        _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o), _abi.strides3(do),
        _abi.strides3(dq), _abi.strides3(dk), _abi.strides3(dv),
        float(softmax_scale), 1 if causal else 0, 1 if deterministic else 0, _stream_handle(q.device))
    _abi.check(rc, "fa_bwd_vdim")
    return dq, dk, dv


def attention_delta(o, do):
    """Delta = rowsum(O * dO) in fp32 (attention.py:237-255)."""
    b, h, n, d = o.shape
    delta = torch.empty((b, h, n), device=o.device, dtype=torch.float32)
    rc = _abi.entry("fa_bwd_delta", o.dtype)(o.data_ptr(), do.data_ptr(), delta.data_ptr(), b, h, n, d,
                                 _abi.strides3(o), _abi.strides3(do), _stream_handle(o.device))
    _abi.check(rc, "fa_bwd_delta")
    return delta


def attention_backward_dq(q, k, v, do, lse, delta, causal: bool, softmax_scale: float, *,
                          dq=None, q_offset: int = 0, k_offset: int = 0):
    """dQ for one key/value block.  With ``dq`` given as an fp32 tensor the
    result is added into it; otherwise a new fp16 tensor is returned."""
    b, hq, nq, d = q.shape
    hkv, nk = k.shape[1], k.shape[2]
    acc = dq is not None
    if acc:
        if dq.dtype != torch.float32 or dq.shape != q.shape:
            raise ValueError("dq accumulator must be an fp32 tensor shaped like q")
    else:
        dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    rc = _abi.entry("fa_bwd_dq", q.dtype)(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                              lse.data_ptr(), delta.data_ptr(), dq.data_ptr(),
                              b, hq, hkv, nq, nk, d,
                              _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(do),
                              _abi.strides3(dq), float(softmax_scale), 1 if causal else 0,
                              int(q_offset), int(k_offset), 1 if acc else 0, _stream_handle(q.device))
    _abi.check(rc, "fa_bwd_dq")
    return dq


def attention_backward_dkdv(q, k, v, do, lse, delta, causal: bool, softmax_scale: float, *,
                            dk=None, dv=None, q_offset: int = 0, k_offset: int = 0):
    """dK, dV for one key/value block (GQA groups summed in-kernel).  With
    ``dk``/``dv`` given as fp32 tensors the results are added into them."""
    b, hq, nq, d = q.shape
    hkv, nk = k.shape[1], k.shape[2]
    acc = dk is not None or dv is not None
    if acc:
        if dk is None or dv is None:
            raise ValueError("pass both dk and dv accumulators or neither")
        for name, t in (("dk", dk), ("dv", dv)):
            if t.dtype != torch.float32 or t.shape != k.shape:
                raise ValueError(f"{name} accumulator must be an fp32 tensor shaped like k")
    else:
        dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
        dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
    rc = _abi.entry("fa_bwd_dkdv", q.dtype)(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                lse.data_ptr(), delta.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                b, hq, hkv, nq, nk, d,
                                _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(do),
                                _abi.strides3(dk), _abi.strides3(dv), float(softmax_scale),
                                1 if causal else 0, int(q_offset), int(k_offset), 1 if acc else 0,
                                _stream_handle(q.device))
    _abi.check(rc, "fa_bwd_dkdv")
    return dk, dv


FUSED_BWD_HEAD_DIMS = (32, 64, 128)
# dropout rates are applied in steps of 1/256 (include/fa_b200.h, fa_fwd_dropout)
DROPOUT_STEP = 1.0 / 256


def fused_backward_enabled(head_dim: int) -> bool:
    """Whether the backward runs as one fused dK/dV + dQ pass: every head
    dim (32, 64, 128), unless ``torch.use_deterministic_algorithms(True)`` asks for
    bitwise-reproducible gradients (the fused pass sums dQ with fp32
    reduce-adds in schedule order; the separate dQ kernel does not)."""
    return head_dim in FUSED_BWD_HEAD_DIMS and not torch.are_deterministic_algorithms_enabled()


def attention_backward_fused(q, k, v, o, do, lse, causal: bool, softmax_scale: float):
    """dQ, dK, dV in one pass over the (key tile, query tile) pairs: the
    preprocess computes Delta and zeroes an fp32 dQ accumulator, the fused
    kernel adds every dQ partial into it with TMA reduce-adds while it keeps
    dK/dV per key tile in TMEM, and a cast writes dQ in the operand type.
    Replaces the reference's _attn_bwd_preprocess + _attn_bwd launches
    (attention.py:731-783)."""
    b, hq, nq, d = q.shape
    hkv, nk = k.shape[1], k.shape[2]
    stream = _stream_handle(q.device)
    # Delta and the dQ accumulator in one allocation; the accumulator starts
    # 256 bytes aligned
    rows = b * hq * nq
    rows_pad = (rows + 63) // 64 * 64
    scratch = torch.empty(rows_pad + rows * d, device=q.device, dtype=torch.float32)
    delta = scratch[:rows].view(b, hq, nq)
    dq_acc = scratch[rows_pad:].view(b, hq, nq, d)
    rc = _abi.entry("fa_bwd_preprocess", o.dtype)(o.data_ptr(), do.data_ptr(), delta.data_ptr(), dq_acc.data_ptr(),
                                                  b, hq, nq, d, _abi.strides3(o), _abi.strides3(do), stream)
    _abi.check(rc, "fa_bwd_preprocess")
    dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
    dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
    rc = _abi.entry("fa_bwd_fused", q.dtype)(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                             lse.data_ptr(), delta.data_ptr(), dq_acc.data_ptr(),
                                             dk.data_ptr(), dv.data_ptr(), b, hq, hkv, nq, nk, d,
                                             _abi.strides3(q), _abi.strides3(k), _abi.strides3(v),
                                             _abi.strides3(do), _abi.strides3(dk), _abi.strides3(dv),
                                             float(softmax_scale), 1 if causal else 0, 0, 0, 0, stream)
    _abi.check(rc, "fa_bwd_fused")
    dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
    rc = _abi.entry("fa_bwd_dq_convert", q.dtype)(dq_acc.data_ptr(), dq.data_ptr(), b, hq, nq, d,
                                                  _abi.strides3(dq), stream)
    _abi.check(rc, "fa_bwd_dq_convert")
    return dq, dk, dv


class B200Attention(torch.autograd.Function):
    """Autograd bridge for the B200 forward and backward kernels
    (counterpart of ``TritonAttention``, attention.py:673-771).

    ``apply(q, k, v, causal, softmax_scale)`` saves (q, k, v, O, LSE) with one
    fp32 base-2 log-sum-exp per query row and returns 5 gradients."""

    @staticmethod
    def forward(ctx, query, key, value, causal, softmax_scale):
        output, lse = attention_forward(query, key, value, bool(causal), float(softmax_scale))
        ctx.save_for_backward(query, key, value, output, lse)
        ctx.softmax_scale = float(softmax_scale)
        ctx.causal = bool(causal)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        query, key, value, output, lse = ctx.saved_tensors
        grad_output = grad_output.contiguous()
        if value.shape[-1] != query.shape[-1]:
            grad_query, grad_key, grad_value = attention_backward_vdim(
                query, key, value, output, grad_output, lse, ctx.causal, ctx.softmax_scale)
            return grad_query, grad_key, grad_value, None, None
        if fused_backward_enabled(query.shape[-1]):
            grad_query, grad_key, grad_value = attention_backward_fused(
                query, key, value, output, grad_output, lse, ctx.causal, ctx.softmax_scale)
            return grad_query, grad_key, grad_value, None, None
        delta = attention_delta(output, grad_output)
        grad_query = attention_backward_dq(query, key, value, grad_output, lse, delta,
                                           ctx.causal, ctx.softmax_scale)
        grad_key, grad_value = attention_backward_dkdv(query, key, value, grad_output, lse, delta,
                                                       ctx.causal, ctx.softmax_scale)
        return grad_query, grad_key, grad_value, None, None


# The reference's name for the autograd Function (attention.py:673).
TritonAttention = B200Attention


def scaled_dot_product_attention(query, key, value, *, is_causal: bool = False, scale: float | None = None,
                                 enable_gqa: bool = False, backend: Backend = "auto",
                                 attn_mask: torch.Tensor | None = None, dropout_p: float = 0.0) -> torch.Tensor:
    """Scaled dot-product attention on the B200 kernels (attention.py:789-845).

    Forward and backward, causal and bidirectional attention, arbitrary
    positive sequence lengths, GQA.  ``backend`` is kept for drop-in
    compatibility: ``"auto"``, ``"triton"`` (the reference's name for its
    custom kernel) and ``"cuda"`` all select the B200 kernels.  Inputs they
    cannot serve raise ``RuntimeError`` -- there is no PyTorch fallback.

    ``attn_mask`` (an addition; the reference has no masks, README.md:93) is
    a bool tensor broadcastable to (batch, query heads, query length, key
    length), ``True`` where the key takes part, as in PyTorch's SDPA; with
    ``is_causal`` a key must pass both.  A query row that sees no key gets
    zeros (PyTorch returns NaN).

    ``dropout_p`` (an addition; the reference has no dropout) drops the
    softmax probabilities at that rate, as PyTorch's SDPA does, applied as
    the nearest multiple of 1/256 (rates below 1/512, which would round to
    nothing, raise ``ValueError``); the pattern is drawn from a seed taken
    from PyTorch's default generator (``torch.manual_seed`` repeats it).  It
    cannot be combined with ``attn_mask``."""
    if backend == "torch":
        raise RuntimeError(
            "backend='torch' (the PyTorch SDPA fallback) is not part of this package; "
            "call torch.nn.functional.scaled_dot_product_attention directly")
    if backend not in _BACKENDS:
        raise ValueError("backend must be one of: 'auto', 'triton', 'cuda'")
    if not isinstance(is_causal, bool):
        raise TypeError("is_causal must be a bool")
    if not isinstance(enable_gqa, bool):
        raise TypeError("enable_gqa must be a bool")
    if scale is not None and (not isinstance(scale, Real) or not math.isfinite(float(scale))):
        raise ValueError("scale must be a finite real number or None")
    if isinstance(dropout_p, bool) or not isinstance(dropout_p, Real) or not 0.0 <= float(dropout_p) < 1.0:
        raise ValueError("dropout_p must be a real number in [0, 1)")
    if dropout_p > 0.0 and not DROPOUT_STEP / 2 <= float(dropout_p) <= 1.0 - DROPOUT_STEP / 2:
        raise ValueError(
            f"dropout_p is applied in steps of 1/256 (the nearest multiple, from 1/256 to 255/256); "
            f"{float(dropout_p):g} would run at {max(1, min(255, round(256 * float(dropout_p)))) / 256:g}: "
            f"pass 0 or a rate in [1/512, 511/512]")
    _validate_inputs(query, key, value, enable_gqa=enable_gqa)
    decision = _dispatch(query, value)
    if decision.backend != "cuda":
        raise RuntimeError(f"B200 CUDA backend is unavailable: {decision.reason}")
    if attn_mask is not None:
        from .masks import validate_attention_mask
        validate_attention_mask(attn_mask, query, key)
        if dropout_p > 0.0:
            raise RuntimeError("B200 CUDA backend is unavailable: attn_mask and dropout_p together are not supported")
    query_c = query.contiguous()
    key_c = key.contiguous()
    value_c = value.contiguous()
    softmax_scale = float(scale) if scale is not None else query.shape[-1] ** -0.5
    if attn_mask is not None:
        from .masks import B200MaskedAttention
        return B200MaskedAttention.apply(query_c, key_c, value_c, attn_mask, is_causal, softmax_scale)
    if dropout_p > 0.0:
        from .dropout import B200DropoutAttention, new_dropout_seed
        return B200DropoutAttention.apply(query_c, key_c, value_c, is_causal, softmax_scale, float(dropout_p),
                                          new_dropout_seed())
    return B200Attention.apply(query_c, key_c, value_c, is_causal, softmax_scale)
