"""The C-ABI library loads and exports every symbol include/fa_b200.h
declares; argument validation answers without touching a GPU (CPU)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from triton_flash_attention_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "fa_b200.h")).read()
    return re.findall(r"FA_API\s+(?:const\s+)?\w+\**\s+\**(fa_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = _declared()
    core = {"fa_fwd", "fa_bwd_delta", "fa_bwd_dq", "fa_bwd_dkdv", "fa_merge_partial"}
    assert core | {n + "_bf16" for n in core} | {"fa_device_status", "fa_status_string", "fa_version"} <= set(names)


def test_library_exports_every_declared_symbol():
    lib = _abi.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) == set(_abi.SIGNATURES)


def test_version_and_status_strings():
    lib = _abi.lib()
    assert lib.fa_version() >= 100
    assert "head_dim" in _abi.status_string(_abi.FA_ERR_UNSUPPORTED_HEAD_DIM)
    assert "16-byte" in _abi.status_string(_abi.FA_ERR_MISALIGNED)
    assert "timed out" in _abi.status_string(_abi.FA_ERR_DEVICE_TIMEOUT)
    assert "out of device memory" in _abi.status_string(_abi.FA_ERR_OUT_OF_MEMORY)
    assert _abi.status_string(_abi.FA_ERR_CUDA)  # CUDA's text once a call recorded one


def _strides():
    return (ctypes.c_int64 * 3)(4096, 1024, 64)


@pytest.mark.parametrize("name", ["fa_fwd", "fa_fwd_bf16"])
@pytest.mark.parametrize("d,expect", [(48, _abi.FA_ERR_UNSUPPORTED_HEAD_DIM), (256, _abi.FA_ERR_UNSUPPORTED_HEAD_DIM)])
def test_rejects_head_dim_before_any_cuda_call(name, d, expect):
    s = _strides()
    rc = getattr(_abi.lib(), name)(16, 16, 16, 16, 16, 1, 1, 1, 8, 8, d, s, s, s, s, 0.1, 1, 0, 0, None)
    assert rc == expect


@pytest.mark.parametrize("shape", [(0, 1, 1, 8, 8), (1, 3, 2, 8, 8), (1, 1, 1, 0, 8), (1, 1, 1, 8, -1)])
def test_rejects_bad_shapes(shape):
    b, hq, hkv, nq, nk = shape
    s = _strides()
    rc = _abi.lib().fa_fwd(16, 16, 16, 16, 16, b, hq, hkv, nq, nk, 64, s, s, s, s, 0.1, 1, 0, 0, None)
    assert rc == _abi.FA_ERR_BAD_SHAPE


def test_rejects_misaligned_output_and_nonfinite_scale():
    s = _strides()
    lib = _abi.lib()
    assert lib.fa_fwd(16, 16, 16, 18, 16, 1, 1, 1, 8, 8, 64, s, s, s, s, 0.1, 1, 0, 0, None) == _abi.FA_ERR_MISALIGNED
    assert lib.fa_fwd(16, 16, 16, 16, 16, 1, 1, 1, 8, 8, 64, s, s, s, s, float("inf"), 1, 0, 0, None) \
        == _abi.FA_ERR_BAD_SHAPE
    odd = (ctypes.c_int64 * 3)(4096, 1024, 63)
    assert lib.fa_bwd_delta(16, 16, 16, 1, 1, 8, 64, odd, s, None) == _abi.FA_ERR_MISALIGNED


def test_fused_backward_validation_without_cuda():
    """The fused backward serves D = 32, 64 and 128 and wants a 16-byte
    aligned fp32 dQ accumulator; other head dims and a misaligned
    accumulator are refused before any CUDA call."""
    s = _strides()
    lib = _abi.lib()
    for name in ("fa_bwd_fused", "fa_bwd_fused_bf16"):
        for d in (48, 96, 256):
            rc = getattr(lib, name)(16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 1, 1, 8, 8, d, s, s, s, s, s, s,
                                    0.1, 1, 0, 0, 0, None)
            assert rc == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM, d
    assert lib.fa_bwd_preprocess(16, 16, 16, 18, 1, 1, 8, 64, s, s, None) == _abi.FA_ERR_MISALIGNED
    assert lib.fa_bwd_dq_convert(18, 16, 1, 1, 8, 64, s, None) == _abi.FA_ERR_MISALIGNED
    assert lib.fa_bwd_dq_convert(16, 16, 1, 1, 8, 48, s, None) == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM


def test_varlen_and_paged_entry_points_reject_before_any_cuda_call():
    lib = _abi.lib()
    p = 16  # a non-null, 16-byte aligned stand-in pointer; nothing is dereferenced on these paths
    # fa_fwd_varlen(q, k, v, o, lse, cu_q, cu_k, B, Hq, Hkv, max_q, max_k, total_q, total_k, D, scale, causal,
    #               window, stream)
    assert lib.fa_fwd_varlen(p, p, p, p, p, p, p, 2, 4, 2, 64, 64, 100, 100, 48, 0.1, 1, 0, None) \
        == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM
    assert lib.fa_fwd_varlen(p, p, p, p, p, p, p, 0, 4, 2, 64, 64, 100, 100, 64, 0.1, 1, 0, None) \
        == _abi.FA_ERR_BAD_SHAPE
    assert lib.fa_fwd_varlen(p, p, p, p, p, None, p, 2, 4, 2, 64, 64, 100, 100, 64, 0.1, 1, 0, None) \
        == _abi.FA_ERR_BAD_SHAPE
    assert lib.fa_fwd_varlen(p, p, p, p, p, p, p, 2, 4, 3, 64, 64, 100, 100, 64, 0.1, 1, 0, None) \
        == _abi.FA_ERR_BAD_SHAPE
    # a sliding window needs the causal mask and a non-negative size
    assert lib.fa_fwd_varlen(p, p, p, p, p, p, p, 2, 4, 2, 64, 64, 100, 100, 64, 0.1, 0, 16, None) \
        == _abi.FA_ERR_BAD_SHAPE
    assert lib.fa_fwd_varlen(p, p, p, p, p, p, p, 2, 4, 2, 64, 64, 100, 100, 64, 0.1, 1, -1, None) \
        == _abi.FA_ERR_BAD_SHAPE
    # fa_bwd_varlen: the fused pass (D = 64, deterministic = 0) needs the dQ accumulator
    assert lib.fa_bwd_varlen(p, p, p, p, p, p, p, p, p, p, None, p, p, 2, 4, 2, 64, 64, 100, 100, 64,
                             0.1, 1, 0, 0, None) == _abi.FA_ERR_BAD_SHAPE
    # fa_fwd_paged(q, kc, vc, o, lse, cu_q, seqlens_k, table, B, Hq, Hkv, max_q, max_k, total_q,
    #              num_pages, page_size, max_pages_per_seq, D, scale, causal, window, stream)
    for page in (12, 8, 0, 48):
        assert lib.fa_fwd_paged(p, p, p, p, p, p, p, p, 2, 4, 2, 1, 300, 2, 10, page, 5, 64, 0.1, 1, 0, None) \
            == _abi.FA_ERR_BAD_SHAPE, page
    assert lib.fa_fwd_paged(p, p, p, p, p, p, p, p, 2, 4, 2, 1, 300, 2, 10, 64, 5, 96, 0.1, 1, 0, None) \
        == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM
    # fa_fwd_paged_split(q, kc, vc, o_part, lse_part, cu_q, seqlens_k, table, B, Hq, Hkv, max_q, max_k,
    #                    total_q, num_pages, page_size, max_pages_per_seq, D, scale, causal, splits, stream):
    # 300 keys are 3 key tiles, so at most 3 ranges; splitting needs GQA packing
    for splits in (0, 4, 65):
        assert lib.fa_fwd_paged_split(p, p, p, p, p, p, p, p, 2, 4, 2, 1, 300, 2, 10, 64, 5, 64, 0.1, 1, splits,
                                      None) == _abi.FA_ERR_BAD_SHAPE, splits
    assert lib.fa_fwd_paged_split(p, p, p, p, p, p, p, p, 2, 4, 4, 1, 300, 2, 10, 64, 5, 64, 0.1, 1, 2, None) \
        == _abi.FA_ERR_BAD_SHAPE
    assert lib.fa_fwd_paged_split(p, p, p, p, p, p, p, p, 2, 4, 2, 1, 300, 2, 10, 64, 5, 96, 0.1, 1, 2, None) \
        == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM
    # fa_combine_splits(o_part, lse_part, o, lse, splits, total_q, H, D, stream)
    assert lib.fa_combine_splits(p, p, p, p, 0, 2, 4, 64, None) == _abi.FA_ERR_BAD_SHAPE
    assert lib.fa_combine_splits(p, p, p, p, 65, 2, 4, 64, None) == _abi.FA_ERR_BAD_SHAPE
    assert lib.fa_combine_splits(p, p, p, p, 2, 2, 4, 48, None) == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM
    assert lib.fa_combine_splits(p, p, 18, p, 2, 2, 4, 64, None) == _abi.FA_ERR_MISALIGNED
