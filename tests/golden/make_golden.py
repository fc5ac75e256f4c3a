"""Generate golden vectors by running the reference's own Triton kernels on CPU.

The reference (AmanPandey28/triton-flash-attention) is pure Python + Triton.
Its kernels run here under Triton's interpreter (``TRITON_INTERPRET=1``), with
no GPU: this script imports ``triton_flash_attention.attention`` from the
reference checkout, launches ``_attn_fwd`` (attention.py:90), the Delta
preprocess (attention.py:237) and ``_attn_bwd`` (attention.py:377) with one
fixed entry of the reference's own autotune tables (attention.py:82-87,
353-374; autotuning itself needs a GPU benchmarker), and mirrors the launch
arguments of ``TritonAttention.forward/backward`` (attention.py:676-771).

Usage (in a checkout that has the reference at REF_ROOT):
    python tests/golden/make_golden.py REF_ROOT   (the reference checkout; required)
writes ``tests/golden/golden.npz``.  Inputs follow the reference's CUDA test
(tests/test_cuda_correctness.py:26-60): q/k/v = 0.5 * randn, dO = 0.1 * randn,
fp16, with the seeds listed in CASES.
"""

from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

# (name, B, Hq, Hkv, N, D, causal, seed, fwd BLOCK_M/BLOCK_N, bwd MACRO/MICRO)
CASES = [
    ("n17_d32_causal", 1, 2, 2, 17, 32, True, 123, (64, 32), (64, 16)),
    ("n17_d32_full", 1, 2, 2, 17, 32, False, 123, (64, 32), (64, 16)),
    ("n129_d64_causal", 1, 2, 2, 129, 64, True, 123, (128, 32), (128, 32)),
    ("n129_d64_full", 1, 2, 2, 129, 64, False, 123, (64, 32), (64, 32)),
    ("gqa_n65_d64_causal", 1, 4, 2, 65, 64, True, 123, (64, 32), (64, 16)),
    ("n7_d32_b2h4_causal", 2, 4, 4, 7, 32, True, 0, (64, 32), (64, 16)),
    ("gqa_n11_d32_causal", 1, 4, 2, 11, 32, True, 1, (64, 32), (64, 16)),
    ("n96_d128_causal", 1, 1, 1, 96, 128, True, 7, (64, 32), (64, 16)),
    ("n200_d128_full", 1, 1, 1, 200, 128, False, 9, (64, 32), (64, 16)),
]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch
    import triton
    from triton_flash_attention import attention as A

    out = {}
    for name, b, hq, hkv, n, d, causal, seed, (bm, bn), (bma, bmi) in CASES:
        torch.manual_seed(seed)
        q = (torch.randn(b, hq, n, d, dtype=torch.float16) * 0.5).contiguous()
        k = (torch.randn(b, hkv, n, d, dtype=torch.float16) * 0.5).contiguous()
        v = (torch.randn(b, hkv, n, d, dtype=torch.float16) * 0.5).contiguous()
        do = (torch.randn(b, hq, n, d, dtype=torch.float16) * 0.1).contiguous()
        scale = d ** -0.5
        o = torch.empty_like(q)
        lse = torch.empty((b, hq, n), dtype=torch.float32)
        A._attn_fwd.fn[(triton.cdiv(n, bm), b * hq)](
            Q=q, K=k, V=v, sm_scale=scale, LSE=lse, Out=o,
            stride_q_batch=q.stride(0), stride_q_head=q.stride(1),
            stride_q_seq=q.stride(2), stride_q_dim=q.stride(3),
            stride_k_batch=k.stride(0), stride_k_head=k.stride(1),
            stride_k_seq=k.stride(2), stride_k_dim=k.stride(3),
            stride_v_batch=v.stride(0), stride_v_head=v.stride(1),
            stride_v_seq=v.stride(2), stride_v_dim=v.stride(3),
            stride_o_batch=o.stride(0), stride_o_head=o.stride(1),
            stride_o_seq=o.stride(2), stride_o_dim=o.stride(3),
            NUM_Q_HEADS=hq, NUM_KV_HEADS=hkv, N_CTX=n, HEAD_DIM=d,
            BLOCK_M=bm, BLOCK_N=bn, CAUSAL=causal)
        delta = torch.empty_like(lse)
        A._attn_bwd_preprocess[(triton.cdiv(n, 128), b * hq)](
            Out=o, dO=do, Delta=delta, N_CTX=n, HEAD_DIM=d, BLOCK_M=128)
        dq = torch.empty_like(q)
        dk = torch.zeros_like(k)
        dv = torch.zeros_like(v)
        A._attn_bwd.fn[(triton.cdiv(n, bma), b * hq)](
            Q_ptr=q, K_ptr=k, V_ptr=v, dO_ptr=do, dQ_ptr=dq, dK_ptr=dk, dV_ptr=dv,
            LSE_ptr=lse, Delta_ptr=delta, sm_scale=scale,
            NUM_Q_HEADS=hq, NUM_KV_HEADS=hkv, N_CTX=n, HEAD_DIM=d, CAUSAL=causal,
            BLOCK_MACRO=bma, BLOCK_MICRO=bmi)
        meta = np.array([b, hq, hkv, n, d, int(causal), seed, bm, bn, bma, bmi], np.int64)
        for key, val in (("q", q), ("k", k), ("v", v), ("do", do), ("o", o), ("lse2", lse),
                         ("delta", delta), ("dq", dq), ("dk", dk), ("dv", dv)):
            out[f"{name}/{key}"] = val.numpy()
        out[f"{name}/meta"] = meta
        print(f"{name}: done")
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <root of the reference checkout>")
    main(sys.argv[1])
