"""The forward+backward step through the public API captures into a CUDA
graph (torch.cuda.graph) and replays to the eager results (GPU only).

Launch overhead matters for short attention calls; the library's launches
are plain stream-ordered kernel launches on the current stream, host-side
tensor-map encoding, and attribute lookups cached on first use, so a warm
step captures.  Replay must match eager: O, dK, dV bitwise (same kernels,
same inputs), dQ within fp32 reduce-order rounding (the fused backward's
reduce-adds), 1e-3 + 1e-2 |dQ|.
"""

from __future__ import annotations

import pytest
import torch

import triton_flash_attention_b200 as fa

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d", [64, 128])
def test_fwd_bwd_step_captures_and_replays(d):
    g = torch.Generator(device="cpu").manual_seed(d)
    q, k, v, do = (torch.randn(2, 4, 640, d, generator=g).half().cuda() for _ in range(4))
    q.requires_grad_()
    k.requires_grad_()
    v.requires_grad_()

    def step():
        o = fa.scaled_dot_product_attention(q, k, v, is_causal=True)
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), do)
        return o.detach(), dq, dk, dv

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        eager = step()  # warm-up: first-use lookups happen outside the capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = step()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    o, dq, dk, dv = static_out
    assert torch.equal(o, eager[0])
    assert torch.equal(dk, eager[2]) and torch.equal(dv, eager[3])
    diff = (dq.float() - eager[1].float()).abs()
    assert bool((diff <= 1e-3 + 1e-2 * eager[1].float().abs()).all()), float(diff.max())
    assert fa._abi.device_status() == 0
