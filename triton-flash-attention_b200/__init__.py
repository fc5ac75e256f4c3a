"""B200-native (sm_100a) FlashAttention-2 behind the public surface of
AmanPandey28/triton-flash-attention (triton_flash_attention/__init__.py:3-15).

The package directory is ``triton-flash-attention_b200/``; it is imported as
``triton_flash_attention_b200`` (through the loader module of that name at
the repository root, or an install that maps the name to this directory).
"""

from .attention import (
    B200Attention,
    DispatchDecision,
    SUPPORTED_HEAD_DIMS,
    FUSED_BWD_HEAD_DIMS,
    TritonAttention,
    attention_backward_dkdv,
    attention_backward_dq,
    attention_backward_fused,
    attention_backward_vdim,
    attention_delta,
    attention_forward,
    attention_forward_vdim,
    explain_dispatch,
    fused_backward_enabled,
    scaled_dot_product_attention,
)
from .dropout import (
    B200DropoutAttention,
    attention_backward_dropout,
    attention_forward_dropout,
)
from .flops import attention_flops, delta_bytes, memory_model
from .masks import (
    B200MaskedAttention,
    attention_backward_masked,
    attention_forward_masked,
    pack_attention_mask,
)
from .varlen import (
    B200VarlenAttention,
    paged_attention_forward,
    scaled_dot_product_attention_paged,
    scaled_dot_product_attention_varlen,
    varlen_attention_backward,
    varlen_attention_forward,
)

__all__ = [
    "B200Attention",
    "B200DropoutAttention",
    "B200MaskedAttention",
    "B200VarlenAttention",
    "DispatchDecision",
    "SUPPORTED_HEAD_DIMS",
    "FUSED_BWD_HEAD_DIMS",
    "TritonAttention",
    "attention_backward_dkdv",
    "attention_backward_dq",
    "attention_backward_dropout",
    "attention_backward_fused",
    "attention_backward_masked",
    "attention_backward_vdim",
    "attention_delta",
    "attention_flops",
    "attention_forward",
    "attention_forward_dropout",
    "attention_forward_masked",
    "attention_forward_vdim",
    "delta_bytes",
    "explain_dispatch",
    "fused_backward_enabled",
    "memory_model",
    "pack_attention_mask",
    "paged_attention_forward",
    "scaled_dot_product_attention",
    "scaled_dot_product_attention_paged",
    "scaled_dot_product_attention_varlen",
    "varlen_attention_backward",
    "varlen_attention_forward",
]
