"""Benchmark of the 720p refinement BSA call on B200 (metric: BSA ms/call and sparse
TFLOP/s = 4*B*H*S*k*64*D / t, as a fraction of bf16 tensor peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config config2] [--impl ours|reference]

One step = one full BSA call on synthetic config inputs already resident in HBM: Q and K block
pooling, routing (bf16 pair split, tcgen05 approximate score keys, per-row selection with exact fp32
scores in the threshold band, the exact fallback for unsettled rows) and the sparse tcgen05 attention,
through the engine's forward entry (6 kernel launches: the bf16 pair split of the routing runs inside
the two pool kernels).
At N > 1 (torchrun, one rank per GPU, NCCL) every rank holds a sequence shard of Q/K/V for all
32 heads; a step is the sequence -> heads exchange, the BSA call on its 32/N heads and the
exchange back, pipelined over head groups (ulysses_bsa_attention).
The problem is fixed as N grows (strong scaling).  Inputs (2.1 GB at config 2) exceed the 126 MB
L2, so no flush is needed between steps.

`--impl reference` times the CPU restatement of the reference's Tier A path (oracle/, the
reference itself is MLX-only and cannot run here) on the host cores: each step is a bounded
sample (one head of the config: routing + sparse attention), reported in the same unit.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "longcat-video-mlx_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "BSA sparse TFLOP/s (4*B*H*S*k*64*D per call) at the 720p refinement shape"
UNIT = "TFLOP/s"
# DRAM bytes (read + write) of one attention launch per (batch, head) at the config-2 shape: ncu
# dram__bytes_read.sum + dram__bytes_write.sum of one launch on 4 heads of config 2 (inputs 265 MB, above
# the L2), 339.0 + 77.7 MB; the traffic is per head.
ATTN_DRAM_BYTES_PER_HEAD = {"config2": (338.954496e6 + 77.703936e6) / 4}
# L2 -> shared-memory rate of TMA tensor gathers alone: 148 CTAs, each keeping 192 KB of random 16 KB K+V
# blocks (two 64 x 64 bf16 boxes each, 128B swizzle) of one head's 44 MB working set in flight and
# releasing every block as it lands; 13.1-14.7 TB/s on two boxes, whatever the map's rank (2-D, 3-D or
# 5-D).  Plain loads go faster (1-D bulk copies 18.6, LDG.128 20.2 TB/s) but cannot produce the swizzled
# operand layout the MMA reads.  The ceiling of the attention kernel's K/V gather.
TMA_GATHER_CEILING_TBS = 13.4


def attn_gather_bytes(cfg, world: int = 1) -> float:
    """Algorithmic L2 -> shared-memory bytes of one attention call on one rank: every (q-block, selected
    kv-block) pair brings its own 64-token K and V tiles."""
    import torch

    elt = torch.empty((), dtype=cfg.dtype).element_size() if cfg.dtype != torch.float32 else 2  # f32 runs f16 attention
    nb = cfg.S // 64
    return float(cfg.B * (cfg.H // world) * nb * cfg.topk * 2 * 64 * cfg.D * elt)


def _peaks():
    """(bf16 burst TFLOP/s, bf16 sustained TFLOP/s, HBM GB/s, "measured" | "fallback")."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        burst = float(p["bf16_tflops"])
        return burst, float(p.get("bf16_tflops_sustained", burst)), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


# ------------------------------------------------------------------------------- clocks
class NullSampler:
    """Stand-in for ranks other than 0, whose clock summaries are not printed."""

    def mark(self, on):
        pass

    def summary(self):
        return None


class ClockSampler:
    """SM clock and throttle reasons of one GPU, polled through NVML every few milliseconds by a host thread
    (falling back to `nvidia-smi -lms 200` when NVML is unavailable).  `mark(True/False)` brackets the timed
    region; the summary covers only the samples taken inside it."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int, interval_s: float = 0.005):
        self.gpu = gpu_index
        self.interval = interval_s
        self.samples = []  # (t, sm_mhz, max_mhz, reasons)
        self.window = [None, None]
        self._stop = threading.Event()
        self._t = None
        self.proc = None
        self.lines = []
        self.error = None
        self._nv = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:
            props = torch.cuda.get_device_properties(self.gpu)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def _sample(self):
        nv, h = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        bits = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}
        try:
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            r = get_reasons(h)
            self.samples.append((time.monotonic(), float(sm), float(mx), {n for n, b in bits.items() if r & b}))
        except Exception as e:  # keep the first error for the record
            self.error = self.error or f"{type(e).__name__}: {e}"

    def _poll(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.interval)

    def __enter__(self):
        self.error = None
        self._nv = None
        try:
            self._nv = self._nvml_handle()
            self._sample()
            if not self.samples:
                raise RuntimeError(self.error or "NVML returned no sample")
            self._t = threading.Thread(target=self._poll, daemon=True)
            self._t.start()
        except Exception as e:
            self.error = f"{type(e).__name__}: {e}"
            self._nv = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                     "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self._t = threading.Thread(target=self._read, daemon=True)
                self._t.start()
            except Exception:
                self.proc = None
        return self

    def mark(self, start: bool):
        """Bracket the timed region; a reading is also taken right here (so the region has samples even if
        the polling thread is starved of the interpreter lock)."""
        if start:
            self.window[0] = time.monotonic()
        if self._nv is not None:
            self._sample()
        if not start:
            self.window[1] = time.monotonic()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self._t:
            self._t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        t0, t1 = self.window
        for t, s_, m_, r in self.samples:
            if t0 is not None and t < t0 or t1 is not None and t > t1:
                continue
            sm.append(s_)
            mx = m_
            reasons |= r
        for ln in self.lines:  # nvidia-smi fallback
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(self.NAMES, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        else:
            out = {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                   "sm_mhz_min": min(sm)}
        if getattr(self, "error", None):
            out["sampler_error"] = self.error
        return out


# ------------------------------------------------------------------------------- CPU sample
def cpu_sample(cfg, heads=1, qblocks=None, seed=0):
    """Time the oracle (CPU restatement of Tier A, sparse gather form) on `heads` heads of the
    config: routing (pool, scores, top-k) + sparse attention.  Returns (seconds, flops, desc)."""
    import numpy as np
    import torch

    from oracle import bsa_oracle as orc

    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    shape_h = (1, heads, cfg.S, cfg.D)
    xs = []
    for _ in range(3):
        x = torch.randn(shape_h, generator=g) * (0.5 if cfg.kind == "offset" else 1.0)
        if cfg.kind == "offset":
            x = (x.view(1, heads, cfg.nb, 64, cfg.D) + torch.randn((1, heads, cfg.nb, 1, cfg.D), generator=g)).view(shape_h)
        xs.append(x.to(cfg.dtype).float().numpy())
    q, k, v = xs
    nq = cfg.nb if qblocks is None else qblocks
    t0 = time.perf_counter()
    qb = orc.mean_pool_blocks_3d(q, cfg.shape, cfg.chunk)
    kb = orc.mean_pool_blocks_3d(k, cfg.shape, cfg.chunk)
    idx, _ = orc.topk_block_indices(orc.block_routing_scores(qb[:, :, :nq], kb), topk=cfg.topk)
    full_idx = np.zeros((1, heads, cfg.nb, cfg.topk), np.int32)
    full_idx[:, :, :nq] = idx
    orc.bsa_sparse_attention(q, k, v, full_idx, cfg.shape, cfg.chunk, qblocks=list(range(nq)), dtype=np.float32)
    dt = time.perf_counter() - t0
    flops = 4.0 * heads * nq * 64 * cfg.topk * 64 * cfg.D
    return dt, flops, f"{heads} head(s) x {nq} q-blocks of {cfg.name}: routing + sparse attention, numpy fp32"


def run_reference(args, cfg):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(cores)
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    times, flops, desc = [], 0.0, ""
    for i in range(args.warmup + args.steps):
        dt, flops, desc = cpu_sample(cfg, heads=1, qblocks=args.ref_qblocks)
        if i >= args.warmup:
            times.append(dt)
    t = statistics.median(times)
    value = flops / t / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config shapes)", "impl": "reference",
        "config": {"workload": cfg.name, "B": cfg.B, "H": cfg.H, "S": cfg.S, "D": cfg.D, "topk": cfg.topk,
                   "block": 64, "sample": desc},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- GPU arm
def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    from longcat_video import _native
    from longcat_video.context_parallel import ulysses_bsa_attention
    from longcat_video.models.block_sparse_attention import bsa_attention
    from longcat_video.models.rope_3d import RopeTables
    from longcat_video.workloads import make_qkv

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    if cfg.H % world or cfg.S % world:
        raise SystemExit("heads and tokens must split evenly over the ranks")
    peak_tf, peak_tf_sus, peak_hbm, peak_kind = _peaks()

    # inputs: the full problem is generated identically on every rank; each rank keeps its
    # sequence shard (all heads, S/world tokens)
    q, k, v = make_qkv(cfg, dev, seed=0)
    Sl = cfg.S // world
    if world > 1:
        q, k, v = (t[:, :, rank * Sl:(rank + 1) * Sl].contiguous() for t in (q, k, v))
    torch.cuda.synchronize()
    rope = RopeTables(cfg.grid, cfg.D, dev) if cfg.rope else None
    rope_args = rope.native_args() if rope else None
    Hl = cfg.H // world
    B, D, S = cfg.B, cfg.D, cfg.S
    nb = cfg.nb
    scale = 1.0 / math.sqrt(D)
    out_h = torch.empty((B, Hl, S, D), device=dev, dtype=cfg.dtype)
    idx = torch.empty((B, Hl, nb, cfg.topk), device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]

    scratch_by_heads = {}

    def local_call(qh, kh, vh, i=None):
        """One BSA call on whole-sequence heads through the engine's forward entry (the path of
        bsa_attention), with events before it, between routing and attention (the engine's phase-event
        hook) and after it."""
        heads = int(qh.shape[1])
        if heads not in scratch_by_heads:
            nbytes = int(_native.lib().bsa_forward_scratch_bytes(B, heads, S, D, *cfg.chunk))
            scratch_by_heads[heads] = torch.empty((nbytes,), device=dev, dtype=torch.uint8)
        if i is not None:
            ev[i][0].record(stream)
            _native.set_phase_event(ev[i][1])
        try:
            o = _native.forward(qh, kh, vh, cfg.shape, cfg.chunk, cfg.topk, scale, rope=rope_args, out=out_h[:, :heads],
                                block_indices=idx[:, :heads], scratch=scratch_by_heads[heads])
        finally:
            if i is not None:
                _native.set_phase_event(None)
        if i is not None:
            ev[i][2].record(stream)
        return o

    def step(i=None):
        if world > 1:
            # sequence shards in, sequence shards out: head-group pipelined all-to-all around the call
            return ulysses_bsa_attention(q, k, v, cfg.shape, chunk_thw=cfg.chunk, topk=cfg.topk, rope=rope,
                                         sm_reserve=args.sm_reserve, head_groups=args.head_groups,
                                         exchange=args.exchange)
        return local_call(q, k, v, i)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # rank 0 samples its GPU's clocks (its summary is the one printed); the other ranks do not poll NVML
    with (ClockSampler(local) if rank == 0 else contextlib.nullcontext(NullSampler())) as clk:
        time.sleep(0.02)  # the sampler's first reading lands before the timed region
        clk.mark(True)  # (rank 0 reads NVML here: before the ranks line up, so that read is not timed)
        if world > 1:
            # the ranks left the sampler's start-up at different times: line them up again, so the first
            # step's barrier does not count one rank's start-up skew as exchange time
            dist.barrier()
            torch.cuda.synchronize()
        t_start.record(stream)
        for i in range(args.steps):
            step_ev[i].record(stream)
            step(i)
        t_end.record(stream)
        torch.cuda.synchronize()
        clk.mark(False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    total_ms = t_start.elapsed_time(t_end)
    bounds = step_ev + [t_end]
    steps_ms = [bounds[i].elapsed_time(bounds[i + 1]) for i in range(args.steps)]
    rank_totals = [total_ms]
    if world > 1:
        # per step, the slowest rank; and every rank's total (the reported value takes the largest)
        st = torch.tensor(steps_ms + [total_ms], device=dev, dtype=torch.float64)
        gathered = [torch.empty_like(st) for _ in range(world)]
        dist.all_gather(gathered, st)
        steps_ms = torch.stack(gathered)[:, :-1].max(dim=0).values.tolist()
        rank_totals = [float(g[-1]) for g in gathered]
    per_step = sorted(steps_ms)
    pct = lambda q: per_step[min(len(per_step) - 1, int(q * (len(per_step) - 1) + 0.5))]
    if world > 1:
        # kernel breakdown for the roofline: the same local call on this rank's H/P whole-sequence
        # heads, timed after (outside) the timed region
        qh, kh, vh = make_qkv(cfg, dev, seed=0, heads=Hl)
        for _ in range(2):
            local_call(qh, kh, vh)
        for i in range(args.steps):
            local_call(qh, kh, vh, i)
        torch.cuda.synchronize()
        del qh, kh, vh
    route_ms = [ev[i][0].elapsed_time(ev[i][1]) for i in range(args.steps)]
    attn_ms = [ev[i][1].elapsed_time(ev[i][2]) for i in range(args.steps)]
    if world > 1:
        tt = torch.tensor([total_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms = float(tt.item())
    err = _native.device_error(clear=True)
    if err:
        raise SystemExit(f"device error code {err}")
    ms_per_step = total_ms / args.steps
    value = cfg.sparse_flops() / (ms_per_step * 1e-3) / 1e12

    # ---- host time per call of the library path: the Python API down to the C ABI (argument checks,
    # tensor maps, launches), enqueue only; the GPU runs behind
    host_us = None
    if world == 1:
        scratch = torch.empty((int(_native.lib().bsa_forward_scratch_bytes(B, cfg.H, S, D, *cfg.chunk)),),
                              device=dev, dtype=torch.uint8)
        fwd = lambda: _native.forward(q, k, v, cfg.shape, cfg.chunk, cfg.topk, scale, rope=rope_args, out=out_h,
                                      block_indices=idx, scratch=scratch)
        fwd()
        torch.cuda.synchronize()
        n_host = 20
        th0 = time.perf_counter()
        for _ in range(n_host):
            fwd()
        host_us = (time.perf_counter() - th0) / n_host * 1e6
        torch.cuda.synchronize()
        del scratch

    # ---- end to end through the public API with host buffers (pinned), per rank
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(tuple(q.shape), dtype=cfg.dtype).pin_memory()

    def e2e_step():
        if world > 1:
            dq, dk, dv = (h.to(dev, non_blocking=True) for h in (hq, hk, hv))
            o = ulysses_bsa_attention(dq, dk, dv, cfg.shape, chunk_thw=cfg.chunk, topk=cfg.topk, rope=rope,
                                      sm_reserve=args.sm_reserve, head_groups=args.head_groups,
                                      exchange=args.exchange)
            hout.copy_(o, non_blocking=True)
        else:
            # host tensors in, host tensor out: the API streams head groups through the GPU
            o = bsa_attention(hq, hk, hv, cfg.shape, chunk_thw=cfg.chunk, topk=cfg.topk, rope=rope)
            assert o.device.type == "cpu"

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    h2d = sum(h.numel() * h.element_size() for h in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()

    line = None
    if rank == 0:
        attn_avg = statistics.mean(attn_ms)
        route_avg = statistics.mean(route_ms)
        flops_local = cfg.sparse_flops() / world
        achieved = flops_local / (attn_avg * 1e-3) / 1e12
        per_head = ATTN_DRAM_BYTES_PER_HEAD.get(cfg.name)
        gbytes = attn_gather_bytes(cfg, world)
        traffic = per_head * cfg.B * (cfg.H // world) if per_head else None
        cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            import torch as _t

            _t.set_num_threads(cores)
            dt, fl, desc = cpu_sample(cfg, heads=1, qblocks=args.ref_qblocks)
            cpu = {"value": fl / dt / 1e12, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "ms_per_step_stats": {"median": pct(0.5), "p10": pct(0.1), "p90": pct(0.9), "min": per_step[0],
                                  "max": per_step[-1], "ranks": "max over ranks per step",
                                  "rank_totals_ms": [round(t, 3) for t in rank_totals]},
            "vs_baseline": None, "dtype": {"torch.bfloat16": "bf16", "torch.float16": "f16",
                      "torch.float32": "f32 I/O and routing, f16 attention"}[str(cfg.dtype)],
            "data": "synthetic (seeded; config-2 style per-block offsets)",
            "config": {"workload": cfg.name, "B": cfg.B, "H": cfg.H, "S": S, "D": D, "topk": cfg.topk, "block": 64,
                       "blocks": "contiguous 64-token", "rope_fused": cfg.rope,
                       "parallelism": f"ulysses-heads{world}" if world > 1 else "single-gpu",
                       "exchange": args.exchange if world > 1 else None,
                       "l2": "inputs 2.1 GB > 126 MB L2, no flush"},
            "pct_bf16_peak": value / peak_tf,
            "kernel_ms": {"routing(pool+route)": route_avg, "attention": attn_avg},
            "host_us_per_call": host_us,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "traffic": traffic, "peak_kind": f"{peak_kind} bf16 burst",
                         "frac_of_sustained": achieved / peak_tf_sus, "kernel": "bsa_attn_kernel",
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch on 4 "
                                           "heads of config 2, scaled per head" if traffic else None,
                         # the resource the kernel actually runs against: the K/V tile gather from L2
                         "gather": {"unit": "TB/s", "bytes": gbytes, "achieved": gbytes / (attn_avg * 1e-3) / 1e12,
                                    "ceiling": TMA_GATHER_CEILING_TBS,
                                    "frac": gbytes / (attn_avg * 1e-3) / 1e12 / TMA_GATHER_CEILING_TBS,
                                    "ceiling_kind": "measured TMA tensor gather of 16 KB K+V blocks from L2 alone"}},
            "e2e": {"value": cfg.sparse_flops() / (e2e_ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            # per step: pool Q, pool K, pair split, score keys, select, fallback, attention
            "gpu_launches": 6 * args.steps,
            "clocks": clk.summary(),
        }
        if cpu:
            line["cpu_baseline"] = cpu
    if world > 1:
        from longcat_video.context_parallel import close_exchanges

        close_exchanges()
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="config2")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--ref-qblocks", type=int, default=256,
                    help="q blocks of one head in each CPU sample (bounds the CPU run time)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sm-reserve", type=int, default=None,
                    help="N>1: SMs kept free of the attention kernel for the exchange (default: library default)")
    ap.add_argument("--exchange", default="auto", choices=["auto", "copy_engine", "messages"],
                    help="N>1: all-to-all implementation (default: copy engines where they apply)")
    ap.add_argument("--head-groups", type=int, default=None,
                    help="N>1: head groups of the pipelined exchange (default: library default)")
    ap.add_argument("--copy-streams", type=int, default=None,
                    help="N>1: copy streams per direction of the copy-engine exchange (default: library default)")
    ap.add_argument("--heads", type=int, default=None,
                    help="override the head count (small cases for profiling; not a bench line)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    from longcat_video.workloads import CONFIGS

    cfg = CONFIGS[args.config]
    if args.heads:
        import dataclasses

        cfg = dataclasses.replace(cfg, H=args.heads)
    if args.copy_streams:
        from longcat_video import context_parallel

        context_parallel.COPY_STREAMS = args.copy_streams
    if args.impl == "reference":
        return run_reference(args, cfg)
    return run_ours(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
