"""Ring context parallelism on the GPU: the CUDA block operations with
global position offsets, the LSE merge kernel and the fp32 gradient
accumulation, checked against the dense kernels; plus the ring itself over
NCCL when two GPUs are present (the 2-rank case is skipped on 1-GPU boxes)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import triton_flash_attention_b200 as fa

pytestmark = pytest.mark.gpu


def _rand(*shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).half().cuda()


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("d,hq,hkv", [(64, 4, 4), (128, 4, 2)])
def test_block_decomposition_matches_full(causal, d, hq, hkv):
    """Keys split into 4 chunks with global offsets; partial forwards merged by
    LSE and block backwards accumulated in fp32 equal the full kernels."""
    import triton_flash_attention_b200.ring as ring
    n, c = 1024, 256
    q, do = _rand(1, hq, n, d, seed=1), _rand(1, hq, n, d, seed=2)
    k, v = _rand(1, hkv, n, d, seed=3), _rand(1, hkv, n, d, seed=4)
    scale = d ** -0.5
    ops = ring.cuda_block_ops()
    o_full, lse_full = fa.attention_forward(q, k, v, causal, scale)
    o_acc = torch.zeros(1, hq, n, d, device="cuda")
    lse_acc = torch.full((1, hq, n), float("-inf"), device="cuda")
    for j in range(n // c):
        kj, vj = k[:, :, j * c:(j + 1) * c], v[:, :, j * c:(j + 1) * c]
        o_p, lse_p = ops.fwd(q, kj, vj, causal, scale, 0, j * c)
        ops.merge(o_acc, lse_acc, o_p, lse_p)
    assert float((o_acc - o_full.float()).abs().max()) <= 2e-3
    assert float((lse_acc - lse_full).abs().max()) <= 1e-3
    delta = fa.attention_delta(o_full, do)
    dq_full = fa.attention_backward_dq(q, k, v, do, lse_full, delta, causal, scale)
    dk_full, dv_full = fa.attention_backward_dkdv(q, k, v, do, lse_full, delta, causal, scale)
    dq_acc = torch.zeros(1, hq, n, d, device="cuda")
    dk_acc = torch.zeros(1, hkv, n, d, device="cuda")
    dv_acc = torch.zeros(1, hkv, n, d, device="cuda")
    for j in range(n // c):
        sl = slice(j * c, (j + 1) * c)
        ops.bwd_dq(q, k[:, :, sl], v[:, :, sl], do, lse_full, delta, causal, scale, dq_acc, 0, j * c)
        ops.bwd_dkdv(q, k[:, :, sl], v[:, :, sl], do, lse_full, delta, causal, scale, dk_acc[:, :, sl],
                     dv_acc[:, :, sl], 0, j * c)
    for acc, full in ((dq_acc, dq_full), (dk_acc, dk_full), (dv_acc, dv_full)):
        assert float((acc - full.float()).abs().max()) <= 1e-2
    # the fused block op (one pass per block: dQ reduce-added, dK/dV added)
    dq_acc.zero_(), dk_acc.zero_(), dv_acc.zero_()
    for j in range(n // c):
        sl = slice(j * c, (j + 1) * c)
        ops.bwd_fused(q, k[:, :, sl], v[:, :, sl], do, lse_full, delta, causal, scale, dq_acc, dk_acc[:, :, sl],
                      dv_acc[:, :, sl], 0, j * c)
    for acc, full in ((dq_acc, dq_full), (dk_acc, dk_full), (dv_acc, dv_full)):
        assert float((acc - full.float()).abs().max()) <= 1e-2
    assert fa._abi.device_status() == 0


def test_single_rank_ring_equals_kernel():
    import triton_flash_attention_b200.ring as ring
    q, k, v, do = (_rand(1, 4, 512, 64, seed=s) for s in range(4))
    qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))
    o = ring.ring_scaled_dot_product_attention(qc, kc, vc, is_causal=True)
    grads = torch.autograd.grad(o, (qc, kc, vc), do)
    q2, k2, v2 = (t.clone().requires_grad_() for t in (q, k, v))
    o2 = fa.scaled_dot_product_attention(q2, k2, v2, is_causal=True)
    grads2 = torch.autograd.grad(o2, (q2, k2, v2), do)
    assert float((o - o2).abs().max()) <= 2e-3
    for a, b in zip(grads, grads2):
        assert float((a - b).abs().max()) <= 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import triton_flash_attention_b200.ring as ring
        g = torch.Generator().manual_seed(11)
        n, d = 2048, 128
        full = [torch.randn(1, h, n, d, generator=g).half() for h in (8, 2, 2, 8)]
        q, k, v, do = (ring.zigzag_shard(t, world, rank).cuda() for t in full)
        q.requires_grad_(); k.requires_grad_(); v.requires_grad_()
        o = ring.ring_scaled_dot_product_attention(q, k, v, is_causal=True)
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), do)
        torch.cuda.synchronize()
        torch.save({x: t.cpu() for x, t in (("o", o.detach()), ("dq", dq), ("dk", dk), ("dv", dv))},
                   os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_ring_nccl(tmp_path):
    import triton_flash_attention_b200.ring as ring
    world = 2
    mp.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    parts = [torch.load(os.path.join(tmp_path, f"r{r}.pt")) for r in range(world)]
    g = torch.Generator().manual_seed(11)
    n, d = 2048, 128
    q, k, v, do = (torch.randn(1, h, n, d, generator=g).half().cuda() for h in (8, 2, 2, 8))
    qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))
    o = fa.scaled_dot_product_attention(qc, kc, vc, is_causal=True, enable_gqa=True)
    ref = dict(zip(("o", "dq", "dk", "dv"), (o.detach(),) + torch.autograd.grad(o, (qc, kc, vc), do)))
    for key in ("o", "dq", "dk", "dv"):
        got = ring.zigzag_unshard([p[key] for p in parts]).cuda()
        tol = 2e-3 if key == "o" else 1e-2
        assert float((got.float() - ref[key].float()).abs().max()) <= tol, key
