"""Ring context parallelism on CPU ranks (gloo, world size 2 and 3).

The ring schedule of ``triton_flash_attention_b200.ring`` -- zig-zag layout,
K/V rotation with P2P sends, LSE merges, the reverse pass with travelling
fp32 dK/dV accumulators -- runs with block operations from the float64
oracle, and the gathered result must equal dense attention over the whole
sequence.  No GPU is involved; the CUDA block operations are tested in
tests/test_ring_cuda.py."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fa2_oracle as orc


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_ops():
    import triton_flash_attention_b200.ring as ring

    def fwd(q, k, v, causal, scale, q_off, k_off):
        o, lse2 = orc.attention_block(q.numpy(), k.numpy(), v.numpy(), causal=causal, scale=scale,
                                      q_offset=q_off, k_offset=k_off)
        return torch.from_numpy(o), torch.from_numpy(lse2)

    def merge(o_acc, lse_acc, o, lse):
        mx = torch.maximum(lse_acc, lse)
        safe = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
        wa = torch.exp2(lse_acc - safe)
        wb = torch.exp2(lse - safe)
        tot = wa + wb
        o_acc.copy_(torch.where(tot[..., None] > 0, (o_acc * wa[..., None] + o.to(o_acc.dtype) * wb[..., None])
                                / torch.where(tot > 0, tot, torch.ones_like(tot))[..., None], o_acc))
        lse_acc.copy_(torch.where(tot > 0, safe + torch.log2(torch.where(tot > 0, tot, torch.ones_like(tot))),
                                  torch.full_like(tot, float("-inf"))))

    def delta(o, do):
        return (o.double() * do.double()).sum(-1)

    def bwd_dq(q, k, v, do, lse, dl, causal, scale, dq_acc, q_off, k_off):
        dq, _, _ = orc.attention_block_grads(q.numpy(), k.numpy(), v.numpy(), do.numpy(), lse.numpy(), dl.numpy(),
                                             causal=causal, scale=scale, q_offset=q_off, k_offset=k_off)
        dq_acc += torch.from_numpy(dq).to(dq_acc.dtype)

    def bwd_dkdv(q, k, v, do, lse, dl, causal, scale, dk_acc, dv_acc, q_off, k_off):
        _, dk, dv = orc.attention_block_grads(q.numpy(), k.numpy(), v.numpy(), do.numpy(), lse.numpy(),
                                              dl.numpy(), causal=causal, scale=scale, q_offset=q_off,
                                              k_offset=k_off)
        dk_acc += torch.from_numpy(dk).to(dk_acc.dtype)
        dv_acc += torch.from_numpy(dv).to(dv_acc.dtype)

    return ring.BlockOps(fwd=fwd, merge=merge, delta=delta, bwd_dq=bwd_dq, bwd_dkdv=bwd_dkdv)


def _worker(rank, world, port, causal, hq, hkv, n, d, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import triton_flash_attention_b200.ring as ring
        g = torch.Generator().manual_seed(7)
        q = torch.randn(1, hq, n, d, generator=g, dtype=torch.float64)
        k = torch.randn(1, hkv, n, d, generator=g, dtype=torch.float64)
        v = torch.randn(1, hkv, n, d, generator=g, dtype=torch.float64)
        do = torch.randn(1, hq, n, d, generator=g, dtype=torch.float64)
        shard = lambda x: ring.zigzag_shard(x, world, rank).contiguous()
        ql, kl, vl, dol = (shard(x).requires_grad_(x is not do) for x in (q, k, v, do))
        ops = _oracle_ops()
        o = ring.ring_scaled_dot_product_attention(ql, kl, vl, is_causal=causal, scale=d ** -0.5, ops=ops)
        dq, dk, dv = torch.autograd.grad(o, (ql, kl, vl), dol)
        torch.save({"o": o.detach(), "dq": dq, "dk": dk, "dv": dv}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,causal,hq,hkv", [(2, True, 2, 2), (2, False, 2, 1), (3, True, 4, 2)])
def test_ring_matches_dense(tmp_path, world, causal, hq, hkv):
    n, d = 12 * world, 16
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, causal, hq, hkv, n, d, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    import triton_flash_attention_b200.ring as ring
    parts = [torch.load(os.path.join(tmp_path, f"r{r}.pt")) for r in range(world)]
    g = torch.Generator().manual_seed(7)
    q = torch.randn(1, hq, n, d, generator=g, dtype=torch.float64)
    k = torch.randn(1, hkv, n, d, generator=g, dtype=torch.float64)
    v = torch.randn(1, hkv, n, d, generator=g, dtype=torch.float64)
    do = torch.randn(1, hq, n, d, generator=g, dtype=torch.float64)
    ref = orc.sdpa_reference(q.numpy(), k.numpy(), v.numpy(), causal=causal, scale=d ** -0.5, do=do.numpy())
    for key in ("o", "dq", "dk", "dv"):
        full = ring.zigzag_unshard([p[key] for p in parts]).numpy()
        assert np.abs(full - ref[key]).max() < 1e-10, key


def test_zigzag_roundtrip_and_balance():
    import triton_flash_attention_b200.ring as ring
    x = torch.arange(2 * 4 * 5).reshape(1, 1, 40, 1).float()
    shards = [ring.zigzag_shard(x, 4, r) for r in range(4)]
    assert torch.equal(ring.zigzag_unshard(shards), x)
    # causal work per rank per ring step: 2 full chunk pairs after step 0
    for r in range(4):
        for step in range(1, 4):
            pairs = ring.visible_pairs(4, r, (r - step) % 4, True)
            assert len(pairs) == 2 and not any(diag for _, _, diag in pairs)
        first = ring.visible_pairs(4, r, r, True)
        assert sorted(d for _, _, d in first) == [False, True, True]
