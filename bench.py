"""Benchmark of the attention hot path (driver contract: one JSON line).

Metric: causal fp16 forward+backward algorithmic TFLOP/s at
B=4, H=16, N=4096, D=64 (config C2), the FLOP convention of the reference's
benchmark (benchmarks/benchmark_attention.py:46-53): fwd+bwd = 3.5 x
4*B*H*N(N+1)/2*D = 4.8115e11 FLOP per step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

* ``value``: one step = forward + backward on device-resident synthetic
  inputs (seeded N(0,1) fp16), K steps timed with CUDA events, max over
  ranks.  The backward is the product's default at D = 64: preprocess
  (Delta, zeroed fp32 dQ accumulator), the fused dK/dV + dQ kernel, and the
  dQ cast; ``--deterministic`` times the bitwise-reproducible path instead
  (Delta, dQ kernel, dK/dV kernel).  The per-step working set (q, k, v, o, dO, dq, dk, dv =
  256 MiB) exceeds the 126 MB L2, so no flush is inserted.
* ``e2e``: the same metric through the public API
  (``scaled_dot_product_attention`` + autograd backward) with pinned host
  buffers: each step copies q, k, v, dO host->device and O, dQ, dK, dV
  device->host inside the timed region; the copies of neighbouring steps
  overlap the compute (two copy streams, double-buffered device inputs).
* ``roofline``: the dominant kernel (the fused backward; dK/dV under
  ``--deterministic``) -- its GEMM FLOPs per launch over its CUDA-event
  duration against the measured dense bf16/fp16 peak.
* ``graph``: the same step captured once in a CUDA graph (torch.cuda.graph)
  and replayed -- the launch gaps between the four kernels removed; an extra
  key, the metric stays the eager ``value``.
* ``cpu_baseline``: the reference's own CPU path (``backend="auto"`` on CPU
  fp16 tensors, which the reference sends to PyTorch's SDPA) from the
  unmodified install in baseline/_ref, timed on every host core on a bounded
  sample (whole C2 batch elements); the oracle's float32 restatement stands
  in when the reference is not installed (``kind: "port"``).
* ``per_rank``: every rank's mean, median and slowest step; the timed region
  is enqueued while the stream is held by a bounded spin, so a host stall
  cannot open a gap in it, and one clock sampler runs per node.
* comparators (1 GPU): the same step through the reference's own Triton
  kernel (``reference_triton_ms``), PyTorch's SDPA (``torch_sdpa_ms``,
  ``cudnn_sdpa_ms``) and this build's public API (``api_ms_per_step``), with
  each one's max-abs error against fp32 on two heads.
* ``ring``: C5 (B1 Hq32 Hkv8 N131072 D128 causal) with ring context
  parallelism over the job's GPUs -- its ms per step, and a parity check of
  the ring against the single-GPU kernels and fp32 at N 16384.
* Multi-GPU (torchrun): weak scaling -- every rank runs its own C2-sized
  batch shard; no collective touches the data path.
* ``--impl reference``: the reference's CPU path as above, on the host
  cores; rank 0 only.
* ``--workload sweep``: the parity/measurement configurations C3 (non-causal,
  B4 H16, D in {32,64,128} x N in {512,...,8192}) and C4 (GQA causal), forward
  and forward+backward through the public API, one JSON line per
  configuration, with the reference's Triton kernel (``backend="triton"``,
  from baseline/_ref) timed beside it when installed.  Informational; the
  metric line is the default workload.
* ``--workload varlen``: a packed batch of 16 causal sequences of ragged
  lengths through ``scaled_dot_product_attention_varlen``, beside the same
  sequences padded and run dense.  Informational.
* ``--workload decode``: one query per sequence over a paged K/V cache
  (``scaled_dot_product_attention_paged``), HBM roofline.  Informational.
* ``--workload masked``: boolean ``attn_mask`` forms (key padding, all
  true, random) and ``dropout_p`` at the C2 shape beside the unmasked call.
  Informational.
* ``--workload kernels --shape B,Hq,Hkv,N,D``: each kernel alone through the
  C ABI (forward, preprocess, Delta, fused backward, dQ, dK/dV); the command
  the kernel profiles are captured with.  Informational.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

B, H, N, D = 4, 16, 4096, 64
CAUSAL = True
WORKLOAD = "C2: MHA causal fp16 fwd+bwd B4 H16 N4096 D64"
# ncu dram__bytes_read.sum + dram__bytes_write.sum of one C2 launch (--set full capture of this command)
DKDV_TRAFFIC_BYTES = 191_409_664 + 38_601_472
FUSED_TRAFFIC_BYTES = 684_556_544 + 343_758_848


def flops_step() -> int:
    from triton_flash_attention_b200.flops import attention_flops
    return attention_flops(batch=B, query_heads=H, sequence=N, head_dim=D, causal=CAUSAL, mode="forward-backward")


def read_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": float(p["bf16_tflops"]), "hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons of the given GPUs during
    the timed region.  One sampler per node (the caller starts it on local
    rank 0 only), so the ranks' timed loops do not share the host with one
    nvidia-smi process each."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices, active: bool = True, period_ms: int = 200):
        self.indices = list(indices)
        self.active = active
        self.period_ms = period_ms
        self.proc = None
        self.lines = []

    def __enter__(self):
        if self.active:
            try:
                ids = ",".join(str(i) for i in self.indices)
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={ids}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                     "-lms", str(self.period_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except Exception:
                self.proc = None
            time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self) -> dict | None:
        if not self.active:
            return None
        sm, mx, reasons, gpus = [], None, set(), set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                gpus.add(f[0])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "gpus": len(gpus)}


def hold_stream(ms: float = 50.0) -> None:
    """Occupies the current stream for about ``ms`` milliseconds (torch's
    bounded clock spin) before a timed region, so that the host enqueues the
    whole region while the GPU is still busy: a host-side stall (scheduler,
    an nvidia-smi query, the interpreter) then cannot open a gap inside the
    timed region.  The spin runs before the start event and is not timed."""
    import torch
    torch.cuda._sleep(int(ms * 1e-3 * 2.0e9))


# ------------------------------------------------------------------ CPU baseline
def _reference_pkg():
    """The unmodified reference package installed in baseline/_ref, or None."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "triton_flash_attention")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        import triton_flash_attention as ref
    except Exception:
        return None
    return ref


def reference_cpu_run(steps: int, warmup: int, batch: int = 1) -> dict:
    """The reference's own CPU path -- ``scaled_dot_product_attention(...,
    backend="auto")`` on CPU fp16 tensors, which the reference dispatches to
    PyTorch's SDPA (attention.py:774-786, 832-839) -- forward + backward on
    ``batch`` of C2's batch elements (all 16 heads, N 4096, D 64) per step,
    on every host core.  Falls back to the oracle's float32 restatement of
    that path when the reference is not installed."""
    import torch

    from triton_flash_attention_b200.flops import attention_flops

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ref = _reference_pkg()
    fl = attention_flops(batch=batch, query_heads=H, sequence=N, head_dim=D, causal=CAUSAL, mode="forward-backward")
    times = []
    if ref is not None:
        g = torch.Generator().manual_seed(0)
        q, k, v, do = (torch.randn(batch, H, N, D, generator=g).half() for _ in range(4))
        q, k, v = (t.requires_grad_() for t in (q, k, v))

        def step():
            o = ref.scaled_dot_product_attention(q, k, v, is_causal=CAUSAL, backend="auto")
            torch.autograd.grad(o, (q, k, v), do)

        decision = ref.explain_dispatch(q, k, v)
        kind, what = "reference", (f"triton_flash_attention (unmodified, baseline/_ref), "
                                   f"backend='auto' -> {decision.backend} ({decision.reason})")
    else:
        import numpy as np

        from oracle import fa2_oracle as orc
        rng = np.random.default_rng(0)
        qn, kn, vn, don = (rng.standard_normal((N, D)).astype(np.float16) for _ in range(4))

        def step():
            for _ in range(batch * H):
                orc.sdpa_head_fwd_bwd_fp32(qn, kn, vn, don, causal=CAUSAL, scale=D ** -0.5)

        kind, what = "port", "the oracle's float32 numpy restatement of the reference's CPU path"
    for _ in range(warmup):
        step()
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"value": fl / sec / 1e12, "unit": "TFLOP/s", "cores": int(torch.get_num_threads()), "kind": kind,
            "sec_per_step": sec,
            "sample": f"each step = fwd+bwd of {batch} of C2's {B} batch elements (B{batch} H{H} N{N} D{D}, causal, "
                      f"fp16 CPU tensors), median of {steps} steps after {warmup} warm-up; {what}"}


def cpu_baseline(max_seconds: float = 15.0) -> dict:
    """The reference's CPU path timed on the host cores on a bounded sample
    of C2 (whole batch elements, about ``max_seconds`` of work)."""
    probe = reference_cpu_run(steps=1, warmup=1)
    steps = max(3, min(20, int(max_seconds / max(probe["sec_per_step"], 1e-3))))
    r = reference_cpu_run(steps=steps, warmup=0)
    r.pop("sec_per_step", None)
    return r


# ------------------------------------------------------------------ distributed plumbing
def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def gpu_local_cpus(dev) -> set[int] | None:
    """The host CPUs on the GPU's NUMA node (sysfs ``local_cpulist`` of its
    PCI function), restricted to those this process may run on; None when
    unknown."""
    import torch

    try:
        pr = torch.cuda.get_device_properties(dev)
        path = f"/sys/bus/pci/devices/{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0/local_cpulist"
        cpus = set()
        with open(path) as f:
            for part in f.read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except (OSError, ValueError, AttributeError):
        return None


def barrier_max(world: int, value: float) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_floats(world: int, values: list[float]) -> list[list[float]]:
    """Every rank's ``values`` (same length on every rank), in rank order."""
    if world == 1:
        return [list(values)]
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, device="cuda", dtype=torch.float64)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [p.tolist() for p in parts]


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def timed_loop(fn, steps: int, warmup: int, world: int = 1, per_step: bool = False):
    """Runs ``fn`` warmup times, then times ``steps`` calls on the current
    stream with CUDA events (barrier + synchronize on both sides, the stream
    held while the host enqueues).  Returns (ms per step on this rank,
    sorted per-step ms or None)."""
    import torch
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)] if per_step else []
    torch.cuda.synchronize()
    barrier(world)
    hold_stream()
    start.record(stream)
    for i in range(steps):
        if per_step:
            evs[i][0].record(stream)
        fn()
        if per_step:
            evs[i][1].record(stream)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end) / steps
    return ms, (sorted(a.elapsed_time(b) for a, b in evs) if per_step else None)


# ------------------------------------------------------------------ comparators (1 GPU)
def comparators(args, q, k, v, do) -> dict:
    """The same C2 step through (a) the reference's own Triton kernel,
    unmodified, from baseline/_ref (backend="triton"), (b) PyTorch's SDPA
    (its default backend, and cuDNN forced), and (c) this build's public API
    (scaled_dot_product_attention + autograd), all with device-resident
    inputs in this process; plus the max-abs errors of the reference kernel
    and of this build against fp32 math on two heads."""
    import torch
    import torch.nn.functional as F

    import triton_flash_attention_b200 as fa

    fl = flops_step()
    steps = max(3, min(args.steps, 20))
    out = {}
    qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))
    impls = [("api", lambda a, b_, c: fa.scaled_dot_product_attention(a, b_, c, is_causal=CAUSAL))]
    ref = _reference_pkg()
    if ref is not None:
        impls.append(("reference_triton",
                      lambda a, b_, c: ref.scaled_dot_product_attention(a, b_, c, is_causal=CAUSAL, backend="triton")))
    impls.append(("torch_sdpa", lambda a, b_, c: F.scaled_dot_product_attention(a, b_, c, is_causal=CAUSAL)))

    def cudnn(a, b_, c):
        from torch.nn.attention import SDPBackend, sdpa_kernel
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            return F.scaled_dot_product_attention(a, b_, c, is_causal=CAUSAL)

    impls.append(("cudnn_sdpa", cudnn))
    # fp32 math on two heads, the error reference
    q32, k32, v32 = (t[:1, :2].detach().float().requires_grad_() for t in (q, k, v))
    o32 = F.scaled_dot_product_attention(q32, k32, v32, is_causal=CAUSAL)
    g32 = (o32.detach(),) + torch.autograd.grad(o32, (q32, k32, v32), do[:1, :2].float())
    for name, fn in impls:
        try:
            def step():
                o = fn(qc, kc, vc)
                torch.autograd.grad(o, (qc, kc, vc), do)

            ms, _ = timed_loop(step, steps, max(args.warmup, 3))
            qs, ks, vs = (t[:1, :2].detach().clone().requires_grad_() for t in (q, k, v))
            o = fn(qs, ks, vs)
            got = (o.detach(),) + torch.autograd.grad(o, (qs, ks, vs), do[:1, :2])
            errs = {n: round(float((a.float() - r).abs().max()), 6) for n, a, r in zip(("o", "dq", "dk", "dv"), got, g32)}
            out[name] = {"ms_per_step": round(ms, 4), "tflops": round(fl / ms / 1e9, 2), "max_abs_err_vs_fp32": errs}
        except Exception as exc:  # reported, not fatal
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:200]}
    return out


# ------------------------------------------------------------------ ring section (C5)
RING_B, RING_HQ, RING_HKV, RING_N, RING_D = 1, 32, 8, 131072, 128
RING_CHECK_N, RING_CHECK_HQ, RING_CHECK_HKV = 16384, 8, 2


def ring_parity(world: int, rank: int, dev) -> dict | None:
    """The ring (zig-zag shards over the ranks, NCCL P2P) at a reduced
    length, B1 Hq8 Hkv2 N16384 D128 causal: its O, dQ, dK, dV gathered and
    un-sharded on rank 0 and compared with (a) the single-GPU kernels on the
    whole sequence and (b) fp32 math on the first GQA group (4 query heads,
    1 K/V head).  Returns the max-abs differences on rank 0."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    import triton_flash_attention_b200 as fa
    import triton_flash_attention_b200.ring as ring

    n, hq, hkv, d = RING_CHECK_N, RING_CHECK_HQ, RING_CHECK_HKV, RING_D
    scale = d ** -0.5
    group = dist.group.WORLD if world > 1 else None
    g = torch.Generator(device=dev).manual_seed(4242)
    full = [torch.randn(1, h, n, d, device=dev, dtype=torch.float16, generator=g) for h in (hq, hkv, hkv, hq)]
    q, k, v, do = (ring.zigzag_shard(t, world, rank).contiguous() for t in full)
    o, lse = ring.ring_forward(q, k, v, causal=True, scale=scale, group=group)
    dq, dk, dv = ring.ring_backward(q, k, v, o, lse, do, causal=True, scale=scale, group=group)

    def gathered(t):
        if world == 1:
            return t
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        return ring.zigzag_unshard(parts)

    got = dict(zip(("o", "dq", "dk", "dv"), (gathered(t) for t in (o, dq, dk, dv))))
    if rank != 0:
        return None
    fq, fk, fv, fdo = full
    qc, kc, vc = (t.clone().requires_grad_() for t in (fq, fk, fv))
    o1 = fa.scaled_dot_product_attention(qc, kc, vc, is_causal=True, enable_gqa=True)
    single = dict(zip(("o", "dq", "dk", "dv"), (o1.detach(),) + torch.autograd.grad(o1, (qc, kc, vc), fdo)))
    grp = hq // hkv
    q32 = fq[:, :grp].float().requires_grad_()
    k32, v32 = (t[:, :1].float().requires_grad_() for t in (fk, fv))
    o32 = F.scaled_dot_product_attention(q32, k32.expand(1, grp, n, d).contiguous(),
                                         v32.expand(1, grp, n, d).contiguous(), is_causal=True)
    ref32 = dict(zip(("o", "dq", "dk", "dv"), (o32.detach(),) + torch.autograd.grad(o32, (q32, k32, v32),
                                                                                     fdo[:, :grp].float())))
    heads = {"o": grp, "dq": grp, "dk": 1, "dv": 1}
    vs_single = {x: round(float((got[x].float() - single[x].float()).abs().max()), 6) for x in got}
    vs_fp32 = {x: round(float((got[x][:, :heads[x]].float() - ref32[x]).abs().max()), 6) for x in got}
    single_fp32 = {x: round(float((single[x][:, :heads[x]].float() - ref32[x]).abs().max()), 6) for x in got}
    ok = all(vs_fp32[x] <= (2e-3 if x == "o" else 1e-2) for x in vs_fp32)
    return {"config": f"B1 Hq{hq} Hkv{hkv} N{n} D{d} causal, zig-zag over {world} rank(s)",
            "max_abs_vs_single_gpu": vs_single, "max_abs_vs_fp32_group0": vs_fp32,
            "single_gpu_max_abs_vs_fp32_group0": single_fp32,
            "tolerance": {"o": 2e-3, "grads": 1e-2}, "within_tolerance": ok}


def ring_timing(args, world: int, rank: int, local: int, dev, ring_seq: int = 0) -> dict:
    """C5 fwd+bwd (B1 Hq32 Hkv8 N131072 D128, causal) with ring context
    parallelism over the ranks (strong scaling: the sequence is split
    zig-zag into 2P chunks); each rank generates its own chunks from
    per-chunk seeds.  CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist

    import triton_flash_attention_b200 as fa
    import triton_flash_attention_b200.ring as ring

    n = ring_seq or RING_N
    c = n // (2 * world)

    def chunked(heads, tag):
        parts = []
        for cid in (rank, 2 * world - 1 - rank):
            g = torch.Generator(device=dev).manual_seed(100003 * tag + cid)
            parts.append(torch.randn(RING_B, heads, c, RING_D, device=dev, dtype=torch.float16, generator=g))
        return torch.cat(parts, dim=2)

    q, k, v, do = chunked(RING_HQ, 1), chunked(RING_HKV, 2), chunked(RING_HKV, 3), chunked(RING_HQ, 4)
    scale = RING_D ** -0.5
    group = dist.group.WORLD if world > 1 else None

    def step():
        o, lse = ring.ring_forward(q, k, v, causal=True, scale=scale, group=group)
        ring.ring_backward(q, k, v, o, lse, do, causal=True, scale=scale, group=group)

    steps = max(2, min(args.ring_steps, args.steps))
    with ClockSampler(range(world), active=local == 0) as clk:
        ms_local, _ = timed_loop(step, steps, 1, world)
    ms = barrier_max(world, ms_local)
    fl = fa.attention_flops(batch=RING_B, query_heads=RING_HQ, sequence=n, head_dim=RING_D, causal=True,
                            mode="forward-backward")
    per_rank = gather_floats(world, [ms_local])
    return {"workload": f"C5: GQA causal B{RING_B} Hq{RING_HQ} Hkv{RING_HKV} N{n} D{RING_D}, ring context "
                        f"parallel over {world} GPU(s), zig-zag chunks of {c}",
            "ms_per_step": round(ms, 3), "value": round(fl / ms / 1e9, 2), "unit": "TFLOP/s", "steps": steps,
            "scaling": "strong", "per_rank_ms": [round(x[0], 3) for x in per_rank],
            "parallelism": f"ring-cp x{world} (NCCL P2P)" if world > 1 else "ring-cp x1 (no peer)",
            "clocks": clk.summary()}


# ------------------------------------------------------------------ our arm
def run_ours(args) -> None:
    import torch

    import triton_flash_attention_b200 as fa

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks = read_peaks()
    scale = D ** -0.5
    fl = flops_step()
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q, k, v, do = (torch.randn(B, H, N, D, device=dev, dtype=torch.float16, generator=g) for _ in range(4))
    stream = torch.cuda.current_stream(dev)

    ev_kv = []
    if args.deterministic:
        torch.use_deterministic_algorithms(True)
    fused = fa.fused_backward_enabled(D)
    if fused:
        # the fused kernel alone, bracketed by events, for the roofline line
        from triton_flash_attention_b200 import _abi
        dq_acc = torch.empty(B, H, N, D, device=dev, dtype=torch.float32)
        delta_buf = torch.empty(B, H, N, device=dev, dtype=torch.float32)
        dk_buf, dv_buf = torch.empty_like(q), torch.empty_like(q)
    kv_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(max(args.steps, 1))]

    def step(record: bool):
        o, lse = fa.attention_forward(q, k, v, CAUSAL, scale)
        if fused:
            sh = torch.cuda.current_stream(dev).cuda_stream  # the capture stream under torch.cuda.graph
            _abi.check(_abi.lib().fa_bwd_preprocess(o.data_ptr(), do.data_ptr(), delta_buf.data_ptr(),
                                                    dq_acc.data_ptr(), B, H, N, D, _abi.strides3(o),
                                                    _abi.strides3(do), sh), "fa_bwd_preprocess")
            if record:
                e0, e1 = kv_ev[len(ev_kv)]
                e0.record(stream)
            _abi.check(_abi.lib().fa_bwd_fused(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
                                               lse.data_ptr(), delta_buf.data_ptr(), dq_acc.data_ptr(),
                                               dk_buf.data_ptr(), dv_buf.data_ptr(), B, H, H, N, N, D,
                                               _abi.strides3(q), _abi.strides3(k), _abi.strides3(v),
                                               _abi.strides3(do), _abi.strides3(dk_buf), _abi.strides3(dv_buf),
                                               scale, 1 if CAUSAL else 0, 0, 0, 0, sh), "fa_bwd_fused")
            if record:
                e1.record(stream)
                ev_kv.append((e0, e1))
            dq = torch.empty_like(q)
            _abi.check(_abi.lib().fa_bwd_dq_convert(dq_acc.data_ptr(), dq.data_ptr(), B, H, N, D,
                                                    _abi.strides3(dq), sh), "fa_bwd_dq_convert")
            return
        delta = fa.attention_delta(o, do)
        fa.attention_backward_dq(q, k, v, do, lse, delta, CAUSAL, scale)
        if record:
            e0, e1 = kv_ev[len(ev_kv)]
            e0.record(stream)
        fa.attention_backward_dkdv(q, k, v, do, lse, delta, CAUSAL, scale)
        if record:
            e1.record(stream)
            ev_kv.append((e0, e1))

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    with ClockSampler(range(world), active=local == 0) as clk:
        ms_local, per_step = timed_loop(lambda: step(True), args.steps, 0, world, per_step=True)

    # per-step distribution, as the reference's benchmark reports it
    # (benchmarks/benchmark_attention.py:153-158): median, p20, p80
    def pct(p):
        return per_step[min(len(per_step) - 1, int(round(p * (len(per_step) - 1))))]
    ms = barrier_max(world, ms_local)
    per_rank = gather_floats(world, [ms_local, pct(0.5), per_step[-1]])
    kv_ms = statistics.mean(a.elapsed_time(b) for a, b in ev_kv)
    value = world * fl / (ms * 1e-3) / 1e12
    status = fa._abi.device_status()

    # ---------------- the same step captured once in a CUDA graph and replayed
    # (launch gaps removed; the kernels and their work are the same)
    graph_info = None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(False)
        gms_local, _ = timed_loop(graph.replay, args.steps, args.warmup, world)
        gms = barrier_max(world, gms_local)
        graph_info = {"ms_per_step": round(gms, 4), "value": round(world * fl / (gms * 1e-3) / 1e12, 2),
                      "note": "the same step captured in one CUDA graph (torch.cuda.graph) and replayed"}
        del graph
    except Exception as exc:  # reported, not fatal: the eager number above is the metric
        graph_info = {"error": f"{type(exc).__name__}: {exc}"[:200]}
        barrier(world)

    # ---------------- end to end through the public API, host buffers
    # Every step copies its q, k, v, dO from pinned host memory and its O,
    # dQ, dK, dV back, and runs forward + backward through
    # scaled_dot_product_attention / autograd.  The copies of neighbouring
    # steps overlap the compute (input copies on one stream into two device
    # buffers, output copies on another), as a data pipeline would run it.
    # The pinned buffers are allocated, and the section runs, on the GPU's
    # NUMA node, as a NUMA-aware loader would place them (the process's
    # previous CPU set is restored afterwards).
    prev_cpus = os.sched_getaffinity(0)
    local_cpus = gpu_local_cpus(dev)
    if local_cpus:
        os.sched_setaffinity(0, local_cpus)
    hq, hk, hv, hdo = (t.cpu().pin_memory() for t in (q, k, v, do))
    outs = [torch.empty(B, H, N, D, dtype=torch.float16).pin_memory() for _ in range(4)]
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hdo))
    d2h = sum(t.numel() * t.element_size() for t in outs)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    bufs = [[torch.empty(B, H, N, D, device=dev, dtype=torch.float16) for _ in range(4)] for _ in range(2)]
    for bset in bufs:
        for t in bset[:3]:
            t.requires_grad_()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]

    def h2d_into(b):
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[b])  # the step that last read these buffers is done
            with torch.no_grad():
                for dst, src in zip(bufs[b], (hq, hk, hv, hdo)):
                    dst.copy_(src, non_blocking=True)
            ev_in[b].record(s_in)

    def e2e_run(n):
        for b in range(2):
            ev_used[b].record(stream)
        h2d_into(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                h2d_into(1 - b)
            stream.wait_event(ev_in[b])
            qd, kd, vd, dod = bufs[b]
            o = fa.scaled_dot_product_attention(qd, kd, vd, is_causal=CAUSAL)
            res = (o, *torch.autograd.grad(o, (qd, kd, vd), dod))
            ev_used[b].record(stream)
            s_out.wait_stream(stream)
            with torch.cuda.stream(s_out):
                for dst, src in zip(outs, res):
                    src.record_stream(s_out)
                    dst.copy_(src.detach(), non_blocking=True)
        stream.wait_stream(s_out)

    e2e_steps = max(4, min(args.steps, 20))
    e2e_run(max(args.warmup, 3))
    torch.cuda.synchronize()
    barrier(world)
    s2 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    e2e_run(e2e_steps)
    e2.record(stream)
    torch.cuda.synchronize()
    e2e_ms = barrier_max(world, s2.elapsed_time(e2) / e2e_steps)
    e2e_value = world * fl / (e2e_ms * 1e-3) / 1e12
    del bufs, outs, hq, hk, hv, hdo
    os.sched_setaffinity(0, prev_cpus)
    e2e_host = {"numa_local_cpus": len(local_cpus) if local_cpus else None, "process_cpus": len(prev_cpus)}

    # ---------------- the same step through other implementations (1 GPU)
    comp = None
    if world == 1 and not args.no_comparators:
        comp = comparators(args, q, k, v, do)

    # ---------------- C5 ring context parallelism: parity and timing
    ring_info = None
    if not args.no_ring:
        del q, k, v, do
        if fused:
            del dq_acc, delta_buf, dk_buf, dv_buf
        torch.cuda.empty_cache()
        try:
            ring_info = {"parity": ring_parity(world, rank, dev)}
            torch.cuda.empty_cache()
            ring_info.update(ring_timing(args, world, rank, local, dev))
        except Exception as exc:  # reported, not fatal: the C2 line above is the metric
            ring_info = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()

    # The forward's 2 GEMMs are 4*pairs*D FLOPs per (b, h); the dK/dV kernel
    # runs 4 GEMMs of 2*pairs*D (2x the forward), the fused kernel 5 (2.5x).
    fwd_flops = fa.attention_flops(batch=B, query_heads=H, sequence=N, head_dim=D, causal=CAUSAL, mode="forward")
    kv_flops = fwd_flops * 5 // 2 if fused else 2 * fwd_flops
    achieved = kv_flops / (kv_ms * 1e-3) / 1e12
    # ncu dram__bytes_read.sum + dram__bytes_write.sum of one C2 launch of
    # the kernel, from a --set full capture of this command
    traffic = FUSED_TRAFFIC_BYTES if fused else DKDV_TRAFFIC_BYTES
    rl_kernel = "fa_bwd_fused_kernel<64>" if fused else "fa_bwd_dkdv_wide_kernel<64>"
    if rank == 0:
        line = {
            "metric": "causal fp16 fwd+bwd TFLOP/s, B4 H16 N4096 D64; % of B200 FP16 tensor peak",
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "step_ms_quantiles": {"p20": round(pct(0.2), 4), "p50": round(pct(0.5), 4), "p80": round(pct(0.8), 4)},
            "per_rank": {"ms_mean": [round(x[0], 4) for x in per_rank], "ms_p50": [round(x[1], 4) for x in per_rank],
                         "ms_max_step": [round(x[2], 4) for x in per_rank]},
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp16",
            "data": "synthetic: seeded N(0,1) q, k, v, dO (no dataset involved)",
            "config": {"workload": WORKLOAD, "global_batch": B * world, "heads": H, "seq_len": N,
                       "head_dim": D, "causal": CAUSAL, "parallelism": f"batch-shard x{world} (no collective)",
                       "l2": "per-step working set 256 MiB > 126 MB L2; no flush",
                       "timing": "CUDA events on the launching stream; the stream is held by a bounded spin "
                                 "while the host enqueues the timed steps (not timed)"},
            "pct_of_peak": round(100.0 * value / world / peaks["bf16_tflops"], 2),
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4), "host": e2e_host,
                    "copies": "pinned host buffers; copies of neighbouring steps overlap the compute"},
            "backward": "fused dK/dV + dQ (dQ summed by fp32 reduce-adds)" if fused
                        else "deterministic: separate dQ and dK/dV kernels",
            "roofline": {"kernel": rl_kernel, "bound": "tensor", "achieved": round(achieved, 2),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops"], 4), "traffic": traffic,
                         "peak_source": peaks["source"], "launch_ms": round(kv_ms, 4)},
            "graph": graph_info,
            "cpu_baseline": cpu,
            "gpu_launches": 4 * args.steps,
            "clocks": clk.summary(),
            "device_status": status,
        }
        if comp is not None:
            line["comparators"] = comp
            for key, name in (("api_ms_per_step", "api"), ("reference_triton_ms", "reference_triton"),
                              ("torch_sdpa_ms", "torch_sdpa"), ("cudnn_sdpa_ms", "cudnn_sdpa")):
                line[key] = comp.get(name, {}).get("ms_per_step")
        if ring_info is not None:
            line["ring"] = ring_info
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------------------ ring workload (C5)
def run_ring(args) -> None:
    """C5 alone (``--workload ring``): the ring's parity check and its
    timing, as the ``ring`` key of the default line reports them."""
    import torch

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    info = {"parity": None if args.no_ring_parity else ring_parity(world, rank, dev)}
    torch.cuda.empty_cache()
    info.update(ring_timing(args, world, rank, local, dev, ring_seq=args.ring_seq))
    if rank == 0:
        line = {"metric": "causal fp16 fwd+bwd TFLOP/s, ring context parallel (C5)", "value": info["value"],
                "unit": "TFLOP/s", "n_gpus": world, "steps": info["steps"], "warmup": 1,
                "ms_per_step": info["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "fp16", "data": "synthetic: seeded N(0,1) per zig-zag chunk",
                "config": {"workload": info["workload"], "parallelism": info["parallelism"]},
                "clocks": info["clocks"], "ring": info}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------------------ reference arm
def run_reference(args) -> None:
    """The reference's own CPU path (``backend="auto"`` on CPU tensors, which
    the reference sends to PyTorch's SDPA) on every host core, rank 0 only;
    each step is forward + backward of one of C2's four batch elements."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    r = reference_cpu_run(steps=args.steps, warmup=args.warmup)
    value = r["value"]
    line = {
        "impl": "reference",
        "metric": "causal fp16 fwd+bwd TFLOP/s, B4 H16 N4096 D64; % of B200 FP16 tensor peak",
        "value": round(value, 5),
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(r["sec_per_step"] * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic: seeded N(0,1) q, k, v, dO",
        "config": {"workload": WORKLOAD, "global_batch": B, "heads": H, "seq_len": N, "head_dim": D,
                   "causal": CAUSAL, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": r["cores"], "kind": r["kind"],
                         "sample": r["sample"]},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_gpu(args) -> None:
    """Informational: the reference's own Triton kernel (backend="triton"),
    unmodified, from its pip install in baseline/_ref, timed on this GPU at C2
    beside this build's kernels, with both implementations' max-abs errors
    against fp32 math on two heads.  Not the driver's reference arm (that is
    the CPU path, --impl reference)."""
    import torch

    import triton_flash_attention_b200 as fa

    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "triton_flash_attention")):
        print(json.dumps({"impl": "reference-gpu", "unavailable": "baseline/_ref is not installed"}))
        return
    sys.path.insert(0, ref_dir)
    import triton_flash_attention as ref

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1234)
    q, k, v, do = (torch.randn(B, H, N, D, device=dev, dtype=torch.float16, generator=g) for _ in range(4))
    fl = flops_step()
    out = {}
    for name, sdpa, kw in (("reference_triton", ref.scaled_dot_product_attention, {"backend": "triton"}),
                           ("b200", fa.scaled_dot_product_attention, {})):
        qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))

        def step():
            o = sdpa(qc, kc, vc, is_causal=CAUSAL, **kw)
            o.backward(do)

        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            step()
        s1.record()
        torch.cuda.synchronize()
        ms = s0.elapsed_time(s1) / args.steps
        qs, ks, vs = (t[:1, :2].detach().clone().requires_grad_() for t in (q, k, v))
        o = sdpa(qs, ks, vs, is_causal=CAUSAL, **kw)
        grads = torch.autograd.grad(o, (qs, ks, vs), do[:1, :2])
        q32, k32, v32 = (t[:1, :2].detach().float().requires_grad_() for t in (q, k, v))
        o32 = torch.nn.functional.scaled_dot_product_attention(q32, k32, v32, is_causal=CAUSAL)
        g32 = torch.autograd.grad(o32, (q32, k32, v32), do[:1, :2].float())
        errs = [float((o.float() - o32).abs().max())] + [float((a.float() - b).abs().max()) for a, b in zip(grads, g32)]
        out[name] = {"ms_per_step": round(ms, 4), "tflops": round(fl / ms / 1e9, 2),
                     "max_abs_err_vs_fp32": dict(zip(("o", "dq", "dk", "dv"), (round(e, 6) for e in errs)))}
    print(json.dumps({"impl": "reference-gpu", "metric": "causal fp16 fwd+bwd TFLOP/s, B4 H16 N4096 D64",
                      "unit": "TFLOP/s", "steps": args.steps, "results": out,
                      "speedup_b200_over_reference_triton": round(out["reference_triton"]["ms_per_step"]
                                                                  / out["b200"]["ms_per_step"], 3)}), flush=True)


def run_kernels(args) -> None:
    """Individual kernels through the C ABI at one shape (``--shape
    B,Hq,Hkv,N,D``, causal unless ``--full``): the forward, the backward
    preprocess (Delta + zeroing the fp32 dQ accumulator), Delta alone, the
    fused backward, and the separate dQ and dK/dV kernels; median of 20
    launches each, CUDA events.  GEMM kernels report TFLOP/s of the work they
    are credited with (forward 1x, fused backward 2.5x, dQ 1.5x, dK/dV 2x of
    the forward count), the memory-bound ones GB/s of their algorithmic
    bytes.  Informational, one JSON line; the command the kernel profiles
    under profiles/ are captured with."""
    import torch

    import triton_flash_attention_b200 as fa
    from triton_flash_attention_b200 import _abi

    b, hq, hkv, n, d = (int(x) for x in args.shape.split(","))
    causal = not args.full
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    q, do = (torch.randn(b, hq, n, d, device=dev, dtype=torch.float16, generator=g) for _ in range(2))
    k, v = (torch.randn(b, hkv, n, d, device=dev, dtype=torch.float16, generator=g) for _ in range(2))
    sc = d ** -0.5
    st = torch.cuda.current_stream().cuda_stream
    lib = _abi.lib()
    o, lse = fa.attention_forward(q, k, v, causal, sc)
    delta = torch.empty(b, hq, n, device=dev, dtype=torch.float32)
    acc = torch.empty(b, hq, n, d, device=dev, dtype=torch.float32)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    S = _abi.strides3
    fwd_fl = fa.attention_flops(batch=b, query_heads=hq, sequence=n, head_dim=d, causal=causal, mode="forward")
    row_bytes = b * hq * n

    def fwd():
        _abi.check(lib.fa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), b, hq, hkv, n,
                              n, d, S(q), S(k), S(v), S(o), sc, int(causal), 0, 0, st), "fa_fwd")

    def pre():
        _abi.check(lib.fa_bwd_preprocess(o.data_ptr(), do.data_ptr(), delta.data_ptr(), acc.data_ptr(), b, hq, n, d,
                                          S(o), S(do), st), "fa_bwd_preprocess")

    def dlt():
        _abi.check(lib.fa_bwd_delta(o.data_ptr(), do.data_ptr(), delta.data_ptr(), b, hq, n, d, S(o), S(do), st),
                   "fa_bwd_delta")

    def fused():
        _abi.check(lib.fa_bwd_fused(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                    delta.data_ptr(), acc.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, hq, hkv, n, n,
                                    d, S(q), S(k), S(v), S(do), S(dk), S(dv), sc, int(causal), 0, 0, 0, st),
                   "fa_bwd_fused")

    def dqk():
        _abi.check(lib.fa_bwd_dq(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                 delta.data_ptr(), dq.data_ptr(), b, hq, hkv, n, n, d, S(q), S(k), S(v), S(do),
                                 S(dq), sc, int(causal), 0, 0, 0, st), "fa_bwd_dq")

    def dkdv():
        _abi.check(lib.fa_bwd_dkdv(q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                   delta.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, hq, hkv, n, n, d, S(q), S(k),
                                   S(v), S(do), S(dk), S(dv), sc, int(causal), 0, 0, 0, st), "fa_bwd_dkdv")

    kernels = {
        "fwd": (fwd, "TFLOP/s", fwd_fl),
        "preprocess": (pre, "GB/s", 4 * row_bytes * d + 4 * row_bytes + 4 * row_bytes * d),
        "delta": (dlt, "GB/s", 4 * row_bytes * d + 4 * row_bytes),
        "fused": (fused, "TFLOP/s", fwd_fl * 5 // 2),
        "dq": (dqk, "TFLOP/s", fwd_fl * 3 // 2),
        "dkdv": (dkdv, "TFLOP/s", 2 * fwd_fl),
    }
    pre()
    torch.cuda.synchronize()
    out = {}
    for name in args.kernels.split(","):
        fn, unit, work = kernels[name]
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(20)]
        for e0, e1 in evs:
            e0.record()
            fn()
            e1.record()
        torch.cuda.synchronize()
        us = statistics.median(a.elapsed_time(b_) for a, b_ in evs) * 1e3
        rate = work / (us * 1e-6) / (1e12 if unit == "TFLOP/s" else 1e9)
        out[name] = {"us": round(us, 1), unit: round(rate, 1)}
    print(json.dumps({"workload": "kernels", "shape": {"B": b, "Hq": hq, "Hkv": hkv, "N": n, "D": d,
                                                       "causal": causal},
                      "dtype": "fp16", "data": "synthetic: seeded N(0,1)", "results": out,
                      "device_status": _abi.device_status()}), flush=True)


SWEEP = ([("C3", 4, 16, 16, n, d, False) for d in (32, 64, 128) for n in (512, 1024, 2048, 2049, 4096, 8192)]
         + [("C4", 2, 32, 8, 8191, 128, True)])


def run_sweep(args) -> None:
    """C3 / C4: forward-only and forward+backward TFLOP/s through the public
    API (this build, and the reference's Triton kernel when baseline/_ref is
    installed), CUDA events, one JSON line per configuration."""
    import torch

    import triton_flash_attention_b200 as fa

    impls = [("b200", fa.scaled_dot_product_attention, {})]
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not args.no_comparators and os.path.isdir(os.path.join(ref_dir, "triton_flash_attention")):
        sys.path.insert(0, ref_dir)
        import triton_flash_attention as ref

        impls.append(("reference_triton", ref.scaled_dot_product_attention, {"backend": "triton"}))
    dev = torch.device("cuda", 0)
    steps = max(1, min(args.steps, 20))

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    for name, b, hq, hkv, n, d, causal in SWEEP:
        g = torch.Generator(device=dev).manual_seed(7 + n + d)
        q = torch.randn(b, hq, n, d, device=dev, dtype=torch.float16, generator=g)
        k, v = (torch.randn(b, hkv, n, d, device=dev, dtype=torch.float16, generator=g) for _ in range(2))
        do = torch.randn(b, hq, n, d, device=dev, dtype=torch.float16, generator=g)
        fl_f = fa.attention_flops(batch=b, query_heads=hq, sequence=n, head_dim=d, causal=causal, mode="forward")
        fl_fb = fa.attention_flops(batch=b, query_heads=hq, sequence=n, head_dim=d, causal=causal, mode="forward-backward")
        row = {"workload": "sweep", "config": name, "B": b, "Hq": hq, "Hkv": hkv, "N": n, "D": d, "causal": causal,
               "unit": "TFLOP/s", "steps": steps}
        for tag, sdpa, kw in impls:
            qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))
            gqa = hq != hkv
            with torch.no_grad():
                ms_f = timed(lambda: sdpa(qc, kc, vc, is_causal=causal, enable_gqa=gqa, **kw))

            def fwd_bwd():
                o = sdpa(qc, kc, vc, is_causal=causal, enable_gqa=gqa, **kw)
                o.backward(do)

            ms_fb = timed(fwd_bwd)
            row[tag] = {"fwd_ms": round(ms_f, 4), "fwd_tflops": round(fl_f / ms_f / 1e9, 1),
                        "fwd_bwd_ms": round(ms_fb, 4), "fwd_bwd_tflops": round(fl_fb / ms_fb / 1e9, 1)}
            del qc, kc, vc
        print(json.dumps(row), flush=True)
        del q, k, v, do
        torch.cuda.empty_cache()


VARLEN_SEQS, VARLEN_H, VARLEN_D, VARLEN_MAX = 16, 16, 64, 4096


def run_varlen(args) -> None:
    """Packed variable-length batch (no counterpart in the reference): 16
    causal sequences of seeded random lengths in [256, 4096] (H16, D64,
    fp16), forward and forward+backward through
    ``scaled_dot_product_attention_varlen``, beside the same sequences padded
    to the longest and run dense.  FLOPs count each sequence's own pairs
    (the reference's convention per sequence); informational, one JSON line."""
    import numpy as np
    import torch

    import triton_flash_attention_b200 as fa

    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(2024)
    lens = rng.integers(256, VARLEN_MAX + 1, size=VARLEN_SEQS)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    total, mx = int(lens.sum()), int(lens.max())
    g = torch.Generator(device=dev).manual_seed(3)
    q, k, v, do = (torch.randn(total, VARLEN_H, VARLEN_D, device=dev, dtype=torch.float16, generator=g)
                   for _ in range(4))
    fl_f = sum(fa.attention_flops(batch=1, query_heads=VARLEN_H, sequence=int(n), head_dim=VARLEN_D, causal=True,
                                  mode="forward") for n in lens)
    fl_fb = sum(fa.attention_flops(batch=1, query_heads=VARLEN_H, sequence=int(n), head_dim=VARLEN_D, causal=True,
                                   mode="forward-backward") for n in lens)
    steps = max(1, min(args.steps, 20))

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    qc, kc, vc = (t.clone().requires_grad_() for t in (q, k, v))
    with torch.no_grad():
        ms_f = timed(lambda: fa.scaled_dot_product_attention_varlen(qc, kc, vc, cu, cu, mx, mx, is_causal=True))

    def fwd_bwd():
        fa.scaled_dot_product_attention_varlen(qc, kc, vc, cu, cu, mx, mx, is_causal=True).backward(do)

    ms_fb = timed(fwd_bwd)
    # the same sequences padded to the longest, dense (B, H, N, D)
    pad = lambda t: torch.stack([torch.nn.functional.pad(t[int(a):int(b)], (0, 0, 0, 0, 0, mx - int(b - a)))
                                 for a, b in zip(cu[:-1].tolist(), cu[1:].tolist())]).transpose(1, 2).contiguous()
    qp, kp, vp, dop = (pad(t) for t in (q, k, v, do))
    qp, kp, vp = (t.requires_grad_() for t in (qp, kp, vp))
    with torch.no_grad():
        ms_pf = timed(lambda: fa.scaled_dot_product_attention(qp, kp, vp, is_causal=True))

    def fwd_bwd_pad():
        fa.scaled_dot_product_attention(qp, kp, vp, is_causal=True).backward(dop)

    ms_pfb = timed(fwd_bwd_pad)
    print(json.dumps({
        "workload": "varlen", "sequences": VARLEN_SEQS, "heads": VARLEN_H, "head_dim": VARLEN_D, "causal": True,
        "dtype": "fp16", "total_tokens": total, "max_seqlen": mx, "unit": "TFLOP/s", "steps": steps,
        "data": "synthetic: seeded N(0,1), seeded random lengths in [256, 4096]",
        "varlen": {"fwd_ms": round(ms_f, 4), "fwd_tflops": round(fl_f / ms_f / 1e9, 1),
                   "fwd_bwd_ms": round(ms_fb, 4), "fwd_bwd_tflops": round(fl_fb / ms_fb / 1e9, 1)},
        "padded_dense": {"fwd_ms": round(ms_pf, 4), "fwd_bwd_ms": round(ms_pfb, 4),
                         "note": "same sequences padded to max_seqlen; TFLOP/s counts only the real pairs",
                         "fwd_tflops": round(fl_f / ms_pf / 1e9, 1), "fwd_bwd_tflops": round(fl_fb / ms_pfb / 1e9, 1)},
    }), flush=True)


def run_masked(args) -> None:
    """Dense boolean masks and attention dropout (no counterpart in the
    reference): the C2 shape (B4 H16 N4096 D64, fp16), forward and
    forward+backward through ``scaled_dot_product_attention`` with no mask,
    a key-padding mask (B, 1, 1, N) hiding each batch's last 512 * (b + 1)
    keys, a mask with every bit set, a seeded random (B, 1, N, N) mask of
    density 0.7, and dropout at p = 0.1, each bidirectional and causal; plus
    the pack kernel alone on the random mask.  The masked times include
    packing the mask (once per forward); dropout runs the split backward.
    Informational, one JSON line."""
    import torch

    import triton_flash_attention_b200 as fa

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    q, k, v, do = (torch.randn(B, H, N, D, device=dev, dtype=torch.float16, generator=g) for _ in range(4))
    q, k, v = (t.requires_grad_() for t in (q, k, v))
    padding = torch.ones(B, 1, 1, N, dtype=torch.bool, device=dev)
    for b in range(B):
        padding[b, ..., N - 512 * (b + 1):] = False
    masks = {
        "none": None,
        "key_padding": padding,
        "all_true": torch.ones(N, N, dtype=torch.bool, device=dev),
        "random_0.7": torch.rand(B, 1, N, N, generator=g, device=dev) < 0.7,
        "dropout_0.1": None,
    }
    steps = max(1, min(args.steps, 20))

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    rows = {}
    for causal in (False, True):
        for name, m in masks.items():
            p = 0.1 if name.startswith("dropout") else 0.0

            def fwd():
                with torch.no_grad():
                    fa.scaled_dot_product_attention(q, k, v, is_causal=causal, attn_mask=m, dropout_p=p)

            def fwd_bwd():
                o = fa.scaled_dot_product_attention(q, k, v, is_causal=causal, attn_mask=m, dropout_p=p)
                torch.autograd.grad(o, (q, k, v), do)

            rows[f"{'causal' if causal else 'bidirectional'}/{name}"] = {
                "fwd_ms": round(timed(fwd), 4), "fwd_bwd_ms": round(timed(fwd_bwd), 4)}
    pack_ms = timed(lambda: fa.pack_attention_mask(masks["random_0.7"], B, H, N, N))
    print(json.dumps({
        "workload": "masked", "batch": B, "heads": H, "seq_len": N, "head_dim": D, "dtype": "fp16",
        "data": "synthetic: seeded N(0,1); seeded masks", "steps": steps, "times": rows,
        "pack_random_mask_ms": round(pack_ms, 4),
        "pack_random_mask_gbs": round(B * N * N / (pack_ms * 1e-3) / 1e9, 1),
        "note": "masked times include fa_mask_pack; key_padding hides 512..2048 trailing keys per batch",
    }), flush=True)


DECODE_B, DECODE_HQ, DECODE_HKV, DECODE_D, DECODE_CTX, DECODE_PAGE = 16, 32, 8, 128, 8192, 64


def run_decode(args) -> None:
    """Decode over a paged K/V cache (no counterpart in the reference): 16
    sequences of 8,192 cached tokens, one new query each, GQA 32/8, D128,
    page 64, fp16, through ``scaled_dot_product_attention_paged`` (the GQA
    group's 4 query heads share a query tile, so each K/V page is read once
    per group).  Decode is bound by reading the cache: the line reports the
    achieved HBM bandwidth (unique K/V bytes / time) against the measured
    copy peak.  The ``few_sequences`` key times 2 sequences of 65,536 cached
    tokens (the same 512 MiB of cache), whose 16 (sequence, K/V head) units
    leave most SMs idle, so the call splits each unit's keys (split-KV, count
    from ``varlen.kv_splits``); both keys also time the call with
    ``num_splits=1``.  Informational, one JSON line."""
    import numpy as np
    import torch

    import triton_flash_attention_b200 as fa
    from triton_flash_attention_b200 import varlen

    dev = torch.device("cuda", 0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    steps = max(1, min(args.steps, 50))
    peaks = read_peaks()

    def measure(n_seq, ctx):
        pages_per = ctx // DECODE_PAGE
        n_pages = n_seq * pages_per
        rng = np.random.default_rng(5)
        table = torch.tensor(rng.permutation(n_pages).reshape(n_seq, pages_per), dtype=torch.int32, device=dev)
        g = torch.Generator(device=dev).manual_seed(6)
        kc, vc = (torch.randn(n_pages, DECODE_PAGE, DECODE_HKV, DECODE_D, device=dev, dtype=torch.float16,
                              generator=g) for _ in range(2))
        q = torch.randn(n_seq, DECODE_HQ, DECODE_D, device=dev, dtype=torch.float16, generator=g)
        cu = torch.arange(n_seq + 1, dtype=torch.int32, device=dev)
        sk = torch.full((n_seq,), ctx, dtype=torch.int32, device=dev)

        def timed(num_splits):
            def step():
                fa.scaled_dot_product_attention_paged(q, kc, vc, table, cu, sk, 1, ctx, is_causal=True,
                                                      enable_gqa=True, num_splits=num_splits)

            with torch.no_grad():
                for _ in range(args.warmup):
                    step()
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(steps):
                    step()
                e1.record()
                torch.cuda.synchronize()
            return e0.elapsed_time(e1) / steps

        ms, ms_unsplit = timed(None), timed(1)
        kv_bytes = 2 * n_seq * ctx * DECODE_HKV * DECODE_D * 2
        gbs = kv_bytes / (ms * 1e-3) / 1e9
        return {"sequences": n_seq, "context": ctx, "ms_per_step": round(ms, 4),
                "kv_splits": varlen.kv_splits(n_seq * DECODE_HKV, ctx // 128, sms),
                "unsplit_ms_per_step": round(ms_unsplit, 4), "kv_bytes_per_step": kv_bytes,
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"]}}

    main_cfg = measure(DECODE_B, DECODE_CTX)
    few = measure(2, DECODE_CTX * DECODE_B // 2)
    print(json.dumps({
        "workload": "decode", "query_heads": DECODE_HQ, "kv_heads": DECODE_HKV,
        "head_dim": DECODE_D, "page_size": DECODE_PAGE, "dtype": "fp16",
        "data": "synthetic: seeded N(0,1) cache and queries, shuffled page table", **main_cfg,
        "few_sequences": few,
        "note": "L2 (126 MB) is smaller than either case's 512 MiB cache; no flush needed",
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--deterministic", action="store_true",
                    help="time the bitwise-reproducible backward (separate dQ and dK/dV kernels)")
    ap.add_argument("--workload", choices=["c2", "ring", "sweep", "varlen", "decode", "masked", "kernels"],
                    default="c2",
                    help="c2: the metric's configuration (default); ring: C5 ring context parallelism; "
                         "sweep: C3/C4 forward and forward+backward beside the reference's Triton kernel; "
                         "varlen: a packed batch of ragged sequences beside its padded dense equivalent; "
                         "decode: one query per sequence over a paged K/V cache; "
                         "masked: boolean attn_mask forms and dropout at the C2 shape; "
                         "kernels: individual kernels through the C ABI at --shape")
    ap.add_argument("--shape", default="4,16,16,4096,64", help="kernels workload: B,Hq,Hkv,N,D")
    ap.add_argument("--kernels", default="fwd,preprocess,delta,fused,dq,dkdv",
                    help="kernels workload: which kernels to time")
    ap.add_argument("--full", action="store_true", help="kernels workload: bidirectional instead of causal")
    ap.add_argument("--ring-seq", type=int, default=0, help="override C5's sequence length (ring workload)")
    ap.add_argument("--ring-steps", type=int, default=3, help="timed C5 steps (the ring key / ring workload)")
    ap.add_argument("--no-ring", action="store_true", help="skip the C5 ring key of the default line")
    ap.add_argument("--no-ring-parity", action="store_true", help="ring workload: skip the parity check")
    ap.add_argument("--no-comparators", action="store_true",
                    help="skip the reference-kernel / PyTorch SDPA / public-API keys of the default line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-gpu":
        run_reference_gpu(args)
    elif args.workload == "ring":
        run_ring(args)
    elif args.workload == "sweep":
        run_sweep(args)
    elif args.workload == "varlen":
        run_varlen(args)
    elif args.workload == "decode":
        run_decode(args)
    elif args.workload == "masked":
        run_masked(args)
    elif args.workload == "kernels":
        run_kernels(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
