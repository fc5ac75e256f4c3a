"""fa_bwd_fused_noalloc: the fused backward for callers that cannot allocate
device memory (engines and plugin hosts that plan every byte up front and
forbid allocation while running, thin FFI bindings without a device
allocator).  It keeps Delta and the fp32 dQ accumulator in the library's own
32 MiB __device__ array instead of caller scratch.

The GPU test calls it through the C ABI twice in a row on the same inputs and
compares both results with the allocating path (fa_bwd_preprocess +
fa_bwd_fused + fa_bwd_dq_convert with torch-allocated scratch).  The second
call starts with the first call's accumulator still in the array, so it also
checks that every call re-zeroes it.  dK and dV come from the same kernel on
the same inputs and must match bitwise; dQ is summed with fp32 reduce-adds in
schedule order, so it may differ by rounding: max |a - b| <= 1e-3 + 1e-2 |b|,
the fused-backward bar for fp16.

This file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import triton_flash_attention_b200 as fa
from triton_flash_attention_b200 import _abi


def _noalloc(q, k, v, o, do, lse, causal, scale):
    b, hq, nq, d = q.shape
    hkv, nk = k.shape[1], k.shape[2]
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
    rc = _abi.lib().fa_bwd_fused_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, hq, hkv, nq, nk, d,
        _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(o), _abi.strides3(do),
        _abi.strides3(dq), _abi.strides3(dk), _abi.strides3(dv), float(scale), 1 if causal else 0, stream)
    _abi.check(rc, "fa_bwd_fused_noalloc")
    return dq, dk, dv


CASES = [
    # b, hq, hkv, nq, nk, d, causal
    (2, 4, 2, 300, 300, 64, True),
    (1, 6, 3, 1000, 1000, 32, False),
    (1, 16, 16, 4096, 4096, 64, True),  # 17 MB of the 32 MiB array
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_noalloc_matches_allocating_path_twice(case):
    b, hq, hkv, nq, nk, d, causal = case
    g = torch.Generator(device="cpu").manual_seed(1000 + nq + d)
    q = torch.randn(b, hq, nq, d, generator=g).half().cuda()
    k = torch.randn(b, hkv, nk, d, generator=g).half().cuda()
    v = torch.randn(b, hkv, nk, d, generator=g).half().cuda()
    do = torch.randn(b, hq, nq, d, generator=g).half().cuda()
    scale = d ** -0.5
    o, lse = fa.attention_forward(q, k, v, causal, scale)
    ref_dq, ref_dk, ref_dv = fa.attention_backward_fused(q, k, v, o, do, lse, causal, scale)
    torch.cuda.synchronize()
    bound = 1e-3 + 1e-2 * ref_dq.float().abs()
    for _ in range(2):
        dq, dk, dv = _noalloc(q, k, v, o, do, lse, causal, scale)
        torch.cuda.synchronize()
        assert _abi.device_status() == 0
        assert torch.equal(dk, ref_dk)
        assert torch.equal(dv, ref_dv)
        diff = (dq.float() - ref_dq.float()).abs()
        assert bool((diff <= bound).all()), float(diff.max())


def test_noalloc_rejects_calls_beyond_the_scratch_limit():
    """Sizes past the array are refused before any CUDA call (runs without a
    GPU): B*Hq*Nq*(D + 1) fp32 values must fit in 32 MiB."""
    s = (ctypes.c_int64 * 3)(16 * 8192 * 64, 8192 * 64, 64)
    lib = _abi.lib()
    # 1 x 16 x 8192 x 64: 8.5 M floats > 8 M
    rc = lib.fa_bwd_fused_noalloc(16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 16, 16, 8192, 8192, 64,
                                  s, s, s, s, s, s, s, s, 0.125, 1, None)
    assert rc == _abi.FA_ERR_SCRATCH_LIMIT
    assert "FA_NOALLOC_SCRATCH_BYTES" in _abi.status_string(rc)
    # D = 128 has no fused kernel
    rc = lib.fa_bwd_fused_noalloc(16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 1, 1, 64, 64, 128,
                                  s, s, s, s, s, s, s, s, 0.125, 1, None)
    assert rc == _abi.FA_ERR_UNSUPPORTED_HEAD_DIM
