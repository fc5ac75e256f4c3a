"""Ring context parallelism for long sequences (no counterpart in the
reference, which runs on one GPU).

Layout ("zig-zag"): the global sequence of length N is cut into 2P equal
chunks of C = N / 2P positions; rank r holds chunks r and 2P-1-r of Q, K, V
(and dO), concatenated in that order along the sequence axis.  Under a causal
mask every rank then does the same amount of work: at ring step 0 a rank
attends its own two chunks (two diagonal blocks and one full block), at every
later step exactly two full chunk pairs.

Forward: P steps.  At step s rank r holds the K/V block of rank
src = (r - s) mod P.  It posts the send of that block to rank r+1 and the
receive of the next one from rank r-1 (NCCL P2P through torch.distributed,
overlapping the transfer with compute), runs the B200 forward kernel for each
visible (query chunk, key chunk) pair with the chunks' global positions as
offsets, and merges the partial (O, LSE) into fp32 accumulators by their
base-2 log-sum-exp (``fa_merge_partial``).

Backward: the same ring in the same direction.  dQ accumulates locally in
fp32; each K/V block travels with fp32 dK/dV accumulators that every rank adds
its contribution to (one ``fa_bwd_fused`` pass per chunk pair with
``accumulate_fp32``, or under deterministic algorithms ``fa_bwd_dq`` and
``fa_bwd_dkdv``), using the merged global LSE and Delta = rowsum(dO * O).  After P steps each
accumulator is one hop away from its owner and is sent home.

The block-level operations are injectable (``BlockOps``) so the ring schedule
can be tested on CPU ranks (gloo) with a reference implementation; the
default ops are the CUDA kernels.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


# --------------------------------------------------------------------------- layout
def zigzag_shard(x: torch.Tensor, world: int, rank: int, dim: int = 2) -> torch.Tensor:
    """This rank's two chunks (r and 2P-1-r) of a global sequence tensor."""
    n = x.shape[dim]
    if n % (2 * world) != 0:
        raise ValueError(f"sequence length {n} must be divisible by 2 * world size ({2 * world})")
    c = n // (2 * world)
    a = x.narrow(dim, rank * c, c)
    b = x.narrow(dim, (2 * world - 1 - rank) * c, c)
    return torch.cat([a, b], dim=dim)


def zigzag_unshard(shards: list[torch.Tensor], dim: int = 2) -> torch.Tensor:
    """Inverse of ``zigzag_shard`` given every rank's shard, in rank order."""
    world = len(shards)
    c = shards[0].shape[dim] // 2
    chunks = [None] * (2 * world)
    for r, s in enumerate(shards):
        chunks[r] = s.narrow(dim, 0, c)
        chunks[2 * world - 1 - r] = s.narrow(dim, c, c)
    return torch.cat(chunks, dim=dim)


def _chunk_ids(world: int, rank: int) -> tuple[int, int]:
    return rank, 2 * world - 1 - rank


def visible_pairs(world: int, rank: int, src: int, causal: bool):
    """(local query chunk slot, key chunk slot, causal-diagonal?) triples a
    rank computes when holding the K/V block of rank ``src``; the chunk slots
    index the two chunks held locally (0: early chunk, 1: late chunk)."""
    out = []
    qa = _chunk_ids(world, rank)
    kb = _chunk_ids(world, src)
    for i, a in enumerate(qa):
        for j, b in enumerate(kb):
            if not causal:
                out.append((i, j, False))
            elif b < a:
                out.append((i, j, False))
            elif b == a:
                out.append((i, j, True))
    return out


# --------------------------------------------------------------------------- block ops
@dataclass
class BlockOps:
    """Block-level operations the ring is built from.

    fwd(q, k, v, causal, scale, q_off, k_off) -> (o, lse2)
    merge(o_acc, lse_acc, o, lse2) -> None            (in place, o_acc fp32)
    delta(o, do) -> delta
    bwd_dq(q, k, v, do, lse, delta, causal, scale, dq_acc, q_off, k_off)      (in place)
    bwd_dkdv(q, k, v, do, lse, delta, causal, scale, dk_acc, dv_acc, q_off, k_off)  (in place)
    bwd_fused(q, k, v, do, lse, delta, causal, scale, dq_acc, dk_acc, dv_acc, q_off, k_off)
        (optional, in place: both of the above in one pass)
    """

    fwd: Callable
    merge: Callable
    delta: Callable
    bwd_dq: Callable
    bwd_dkdv: Callable
    bwd_fused: Callable | None = None


def cuda_block_ops() -> BlockOps:
    """The B200 kernels (the product path)."""
    from . import _abi
    from .attention import attention_backward_dkdv, attention_backward_dq, attention_delta, attention_forward

    def fwd(q, k, v, causal, scale, q_off, k_off):
        return attention_forward(q, k, v, causal, scale, q_offset=q_off, k_offset=k_off)

    def merge(o_acc, lse_acc, o, lse):
        b, h, n, d = o.shape
        if not (o_acc.is_contiguous() and o.is_contiguous() and lse_acc.is_contiguous() and lse.is_contiguous()):
            raise ValueError("merge operands must be contiguous")
        rc = _abi.entry("fa_merge_partial", o.dtype)(o_acc.data_ptr(), lse_acc.data_ptr(), o.data_ptr(),
                                                     lse.data_ptr(), b, h, n, d,
                                                     torch.cuda.current_stream(o.device).cuda_stream)
        _abi.check(rc, "fa_merge_partial")

    def bwd_dq(q, k, v, do, lse, delta, causal, scale, dq_acc, q_off, k_off):
        attention_backward_dq(q, k, v, do, lse, delta, causal, scale, dq=dq_acc, q_offset=q_off, k_offset=k_off)

    def bwd_dkdv(q, k, v, do, lse, delta, causal, scale, dk_acc, dv_acc, q_off, k_off):
        attention_backward_dkdv(q, k, v, do, lse, delta, causal, scale, dk=dk_acc, dv=dv_acc,
                                q_offset=q_off, k_offset=k_off)

    def bwd_fused(q, k, v, do, lse, delta, causal, scale, dq_acc, dk_acc, dv_acc, q_off, k_off):
        # one pass: dQ reduce-added into the chunk's fp32 accumulator, dK/dV
        # added into the travelling fp32 accumulators (fa_bwd_fused)
        b, hq, nq, d = q.shape
        hkv, nk = k.shape[1], k.shape[2]
        rc = _abi.entry("fa_bwd_fused", q.dtype)(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(), delta.data_ptr(),
            dq_acc.data_ptr(), dk_acc.data_ptr(), dv_acc.data_ptr(), b, hq, hkv, nq, nk, d,
            _abi.strides3(q), _abi.strides3(k), _abi.strides3(v), _abi.strides3(do), _abi.strides3(dk_acc),
            _abi.strides3(dv_acc), float(scale), 1 if causal else 0, int(q_off), int(k_off), 1,
            torch.cuda.current_stream(q.device).cuda_stream)
        _abi.check(rc, "fa_bwd_fused")

    return BlockOps(fwd=fwd, merge=merge, delta=attention_delta, bwd_dq=bwd_dq, bwd_dkdv=bwd_dkdv,
                    bwd_fused=bwd_fused)


# --------------------------------------------------------------------------- P2P
def _exchange(tensors, group, world, rank):
    """Send ``tensors`` to rank+1 and receive same-shaped tensors from
    rank-1 (asynchronously); returns (received buffers, works)."""
    nxt = (rank + 1) % world
    prv = (rank - 1) % world
    recv = [torch.empty_like(t) for t in tensors]
    ops = []
    for t, r in zip(tensors, recv):
        ops.append(dist.P2POp(dist.isend, t, dist.get_global_rank(group, nxt) if group is not None else nxt, group))
        ops.append(dist.P2POp(dist.irecv, r, dist.get_global_rank(group, prv) if group is not None else prv, group))
    works = dist.batch_isend_irecv(ops)
    return recv, works


def _wait(works):
    for w in works:
        w.wait()


def _chunk(x, slot, c):
    return x.narrow(2, slot * c, c)


def _acc_dtype(x: torch.Tensor) -> torch.dtype:
    # fp32 accumulators for the fp16 kernels; float64 stays float64 (CPU checks)
    return torch.float64 if x.dtype == torch.float64 else torch.float32


# --------------------------------------------------------------------------- ring passes
def ring_forward(q, k, v, *, causal: bool, scale: float, group=None, ops: BlockOps | None = None):
    """Forward over the ring; q, k, v are this rank's zig-zag shards
    (B, H, 2C, D).  Returns (o, lse2) for the local queries."""
    ops = ops or cuda_block_ops()
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    c = q.shape[2] // 2
    b, h, _, d = q.shape
    qa = _chunk_ids(world, rank)
    acc = _acc_dtype(q)
    o_acc = [torch.zeros(b, h, c, d, device=q.device, dtype=acc) for _ in range(2)]
    lse_acc = [torch.full((b, h, c), float("-inf"), device=q.device, dtype=acc) for _ in range(2)]
    kv = (k.contiguous(), v.contiguous())
    for step in range(world):
        src = (rank - step) % world
        works = None
        if step + 1 < world:
            nxt_kv, works = _exchange(kv, group, world, rank)
        kb = _chunk_ids(world, src)
        for i, j, diag in visible_pairs(world, rank, src, causal):
            o_p, lse_p = ops.fwd(_chunk(q, i, c), _chunk(kv[0], j, c), _chunk(kv[1], j, c), diag, scale,
                                 qa[i] * c, kb[j] * c)
            ops.merge(o_acc[i], lse_acc[i], o_p, lse_p)
        if works is not None:
            _wait(works)
            kv = tuple(nxt_kv)
    o = torch.cat(o_acc, dim=2).to(q.dtype)
    lse = torch.cat(lse_acc, dim=2)
    return o, lse


def ring_backward(q, k, v, o, lse, do, *, causal: bool, scale: float, group=None, ops: BlockOps | None = None):
    """Backward over the ring; returns (dq, dk, dv) for this rank's shards."""
    ops = ops or cuda_block_ops()
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    c = q.shape[2] // 2
    qa = _chunk_ids(world, rank)
    do = do.contiguous()
    delta = ops.delta(o.contiguous(), do)
    acc = _acc_dtype(q)
    dq_acc = [torch.zeros(_chunk(q, i, c).shape, device=q.device, dtype=acc) for i in range(2)]
    lse_c = [_chunk(lse.unsqueeze(-1), i, c).squeeze(-1).contiguous() for i in range(2)]
    delta_c = [_chunk(delta.unsqueeze(-1), i, c).squeeze(-1).contiguous() for i in range(2)]
    q_c = [_chunk(q, i, c) for i in range(2)]
    do_c = [_chunk(do, i, c) for i in range(2)]
    k_cur, v_cur = k.contiguous(), v.contiguous()
    # one fused pass per chunk pair (dQ, dK, dV from one visit), unless
    # deterministic algorithms ask for the bitwise-reproducible split kernels
    fused = ops.bwd_fused is not None and not torch.are_deterministic_algorithms_enabled()
    # The running fp32 dK/dV sums of the block held at step s arrive from
    # rank - 1 while this rank computes its own contribution into fresh
    # accumulators; the two are added and sent on to rank + 1 at the end of
    # the step, so each hand-off overlaps the next step's compute.  After the
    # last step every rank receives its own block's complete sums.
    gworks = None
    g_in = g_out = None  # buffers of the hand-off in flight (kept alive until it completes)
    for step in range(world):
        src = (rank - step) % world
        kb = _chunk_ids(world, src)
        works = None
        if step + 1 < world:  # K/V for the next step travel while this one computes
            nxt_kv, works = _exchange((k_cur, v_cur), group, world, rank)
        dk_cur = torch.zeros(k_cur.shape, device=k.device, dtype=acc)
        dv_cur = torch.zeros(v_cur.shape, device=v.device, dtype=acc)
        for i, j, diag in visible_pairs(world, rank, src, causal):
            kj, vj = _chunk(k_cur, j, c), _chunk(v_cur, j, c)
            dk_j = _chunk(dk_cur, j, c)
            dv_j = _chunk(dv_cur, j, c)
            if fused:
                ops.bwd_fused(q_c[i], kj, vj, do_c[i], lse_c[i], delta_c[i], diag, scale, dq_acc[i], dk_j, dv_j,
                              qa[i] * c, kb[j] * c)
                continue
            ops.bwd_dq(q_c[i], kj, vj, do_c[i], lse_c[i], delta_c[i], diag, scale, dq_acc[i], qa[i] * c, kb[j] * c)
            ops.bwd_dkdv(q_c[i], kj, vj, do_c[i], lse_c[i], delta_c[i], diag, scale, dk_j, dv_j,
                         qa[i] * c, kb[j] * c)
        # this block's running sums (from rank - 1) plus this rank's part move
        # on with the block; the last hop returns them to their owner
        if gworks is not None:
            _wait(gworks)
            dk_cur += g_in[0]
            dv_cur += g_in[1]
        if world > 1:
            g_out = (dk_cur, dv_cur)
            g_in, gworks = _exchange(g_out, group, world, rank)
        if works is not None:
            _wait(works)
            k_cur, v_cur = nxt_kv
    if gworks is not None:
        _wait(gworks)
        dk_cur, dv_cur = g_in
    del g_out
    dq = torch.cat(dq_acc, dim=2).to(q.dtype)
    return dq, dk_cur.to(k.dtype), dv_cur.to(v.dtype)


class RingAttention(torch.autograd.Function):
    """Autograd Function over the ring; inputs are this rank's zig-zag
    shards."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale, group, ops):
        o, lse = ring_forward(q, k, v, causal=bool(causal), scale=float(scale), group=group, ops=ops)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale, ctx.group, ctx.ops = bool(causal), float(scale), group, ops
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = ring_backward(q, k, v, o, lse, do, causal=ctx.causal, scale=ctx.scale, group=ctx.group,
                                   ops=ctx.ops)
        return dq, dk, dv, None, None, None, None


def ring_scaled_dot_product_attention(query, key, value, *, is_causal: bool = False, scale: float | None = None,
                                      group=None, ops: BlockOps | None = None) -> torch.Tensor:
    """Attention over a sequence sharded zig-zag across the ranks of
    ``group`` (see ``zigzag_shard``).  Inputs are (B, H, 2C, D) shards; GQA is
    allowed (Hq a multiple of Hkv)."""
    if query.shape[2] % 2 or key.shape[2] != query.shape[2]:
        raise ValueError("ring attention expects equal-length zig-zag shards of even length")
    if query.shape[1] % key.shape[1]:
        raise ValueError("the number of query heads must be divisible by the number of key/value heads")
    sc = float(scale) if scale is not None else query.shape[-1] ** -0.5
    return RingAttention.apply(query.contiguous(), key.contiguous(), value.contiguous(), is_causal, sc, group, ops)
