"""Benchmark of the fused attention layer core on B200 (one JSON line on rank 0).

Workload (default): LLaMA-3-8B-shaped attention layer, bf16, B=4, H=32,
S=8192, D=128, causal, RoPE (theta 500000) on Q and K before attention.
One step = RoPE(Q), RoPE(K), attention forward, attention backward with the
RoPE backward of dQ and dK fused into it; with N GPUs the heads are sharded (H/N per rank)
and the per-rank output shards are all-gathered over NCCL and reassembled
into [B, S, H, D] (the merged-heads layout) on every rank.

Metric: attention fwd+bwd TFLOP/s, FlashAttention convention
(fwd 4*B*H*S^2*D, bwd 2.5x fwd, causal halves both: 7*B*H*S^2*D), whole job.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl haelixe|reference]

`--workload block_stack` instead times a context workload, not the headline:
one training step of an 8-block TransformerBlock language model (d_model
2048, 16 heads x 128, GELU MLP 8192, final RMSNorm, vocab 32000, batch 2 x
seq 4096, causal, bf16 storage with f32 master weights, AdamW), every op
through the library (attention kernels, cuBLAS GEMMs, element kernels).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "attn fwd+bwd TFLOP/s and % of BF16 tensor peak at 1/2/4/8 B200 vs host-CPU ref"
UNIT = "TFLOP/s"
# Peak used for roofline.frac: the pool's measured cuBLAS bf16 figures. The
# burst figure applies to a timed region shorter than SUSTAINED_AFTER_S (the
# GPU has not yet settled under its power cap); the sustained figure to a
# longer one.
FALLBACK_PEAK_TFLOPS = 1590.0
SUSTAINED_AFTER_S = 2.0


def choose_peak(peaks, timed_s):
    """(peak TFLOP/s, source) for a timed region of `timed_s` seconds."""
    if not peaks:
        return FALLBACK_PEAK_TFLOPS, "fallback (1590 TF/s burst)"
    if timed_s >= SUSTAINED_AFTER_S and peaks.get("bf16_tflops_sustained"):
        return float(peaks["bf16_tflops_sustained"]), \
            f"measured cuBLAS bf16, sustained (timed region {timed_s:.2f} s >= {SUSTAINED_AFTER_S:g} s)"
    if peaks.get("bf16_tflops"):
        return float(peaks["bf16_tflops"]), \
            f"measured cuBLAS bf16, burst (timed region {timed_s:.2f} s < {SUSTAINED_AFTER_S:g} s)"
    return FALLBACK_PEAK_TFLOPS, "fallback (1590 TF/s burst)"
# DRAM bytes (read + write) per launch of the dominant kernel (the tcgen05
# backward) at B4 H32 S8192 D128: an ncu capture of the same kernel at B1
# H32 S8192 D128 (414.0 MB read + 225.6 MB written) scaled by 4, since the
# heads are independent and the traffic grows with B*H. Valid for the
# default workload only; other shapes report None.
DOMINANT_KERNEL_TRAFFIC_BYTES = 4 * (414.047232e6 + 225.557248e6)
TRAFFIC_WORKLOAD = (4, 32, 8192, 128)


def traffic_per_launch(dom, B, H, S, D):
    """DRAM bytes per launch of the dominant kernel on this rank, scaled from
    the captured workload by the number of (batch, head) slices it processes."""
    b0, h0, s0, d0 = TRAFFIC_WORKLOAD
    if dom != "bwd" or (S, D) != (s0, d0):
        return None
    return DOMINANT_KERNEL_TRAFFIC_BYTES * (B * H) / (b0 * h0)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["haelixe", "reference"], default="haelixe")
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--seq", type=int, default=8192)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--no-causal", action="store_true")
    p.add_argument("--dtype", choices=["bf16", "f32"], default="bf16",
                   help="operand dtype of the attention workload; f32 runs on the tensor cores as bf16 "
                        "hi/lo planes, three MMAs per product")
    p.add_argument("--rope-theta", type=float, default=500000.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--e2e-steps", type=int, default=20)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", choices=["attention", "block_stack", "linear"], default="attention")
    p.add_argument("--linear-shape", default="8192,2048,8192",
                   help="linear workload: rows,in_features,out_features of y = x W + b")
    p.add_argument("--gemm-backend", choices=["tcgen05", "cublas"], default="tcgen05",
                   help="block_stack workload: the bf16 Linear GEMMs on this library's kernel or on cuBLAS")
    p.add_argument("--rope-launches", type=int, choices=[1, 2], default=2,
                   help="rotate Q and K in two launches (hx_rope_fwd) or in one (hx_rope_fwd_qk)")
    p.add_argument("--head-layout", choices=["bhsd", "bshd"], default="bhsd",
                   help="memory of Q, K, V, dO, O and the gradients: [B, H, S, D], or [B, S, H, D] (the "
                        "projection rows of the multi-head layer, heads as strided views); with N > 1 the "
                        "latter lets the head merge run as copy-engine copies")
    p.add_argument("--compute-priority", choices=["default", "high"], default="default",
                   help="run the attention step on a high-priority stream, so its CTAs are scheduled "
                        "ahead of the exchange's (N > 1)")
    p.add_argument("--exchange-flags", type=int, default=1,
                   help="hx_group flags of the N>1 exchange: 1 register, 2 symmetric window, 4 copy engines")
    return p.parse_args()


def attn_flops(B, H, S, D, causal):
    f = 14.0 * B * H * S * S * D  # fwd 4 + bwd 10
    return f * 0.5 if causal else f


def workload_name(a):
    return (f"attention layer core B{a.batch} H{a.heads} S{a.seq} D{a.head_dim} "
            f"{'causal' if not a.no_causal else 'full'} {a.dtype}, RoPE theta {a.rope_theta:g} on Q/K")


def config_of(a, n):
    op_mb = a.batch * a.heads * a.seq * a.head_dim * (4 if a.dtype == "f32" else 2) / 1e6
    return {
        "workload": workload_name(a),
        "batch": a.batch, "heads": a.heads, "seq_len": a.seq, "head_dim": a.head_dim,
        "causal": not a.no_causal, "rope_theta": a.rope_theta, "head_layout": a.head_layout,
        "parallelism": f"heads/{n} per GPU + NCCL all-gather of O" if n > 1 else "1 GPU, all heads",
        "l2": ("inputs larger than L2 (each operand %.0f MB > 126 MB)" if op_mb > 126 else
               "inputs smaller than L2 (each operand %.0f MB); no L2 flush") % op_mb,
        "seed": a.seed,
    }


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """SM clocks, power and clock-event (throttle) reasons sampled every 5 ms
    during the timed region through NVML (read-only queries); falls back to
    `nvidia-smi -lms 200` when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.stop_flag = threading.Event()
        self.sm, self.power, self.reasons, self.max_mhz = [], [], set(), None
        self.lines = []
        self.source = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            bits = [(name, getattr(pynvml, const)) for name, const in self.REASONS]

            def loop():
                while not self.stop_flag.is_set():
                    try:
                        self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                        self.power.append(pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0)
                        mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        for name, bit in bits:
                            if mask & bit:
                                self.reasons.add(name)
                    except Exception:
                        pass
                    time.sleep(0.005)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            self.source = "nvml 5 ms"
            return
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            self.source = "nvidia-smi 200 ms"
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.source is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        if self.proc is None:
            self.stop_flag.set()
            self.thread.join(timeout=1)
        else:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
            for ln in self.lines:
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    self.sm.append(float(parts[1]))
                    self.max_mhz = float(parts[2])
                    self.power.append(float(parts[3]))
                except ValueError:
                    continue
                for nm, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        self.reasons.add(nm)
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(self.sm) if self.sm else None,
                "power_w_median": statistics.median(self.power) if self.power else None,
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": self.source}


def cpu_baseline(q, k, v, do, scale, causal, budget_s=12.0, max_slices=32):
    """Oracle (C restatement of the reference's CPU path) on whole (b,h) slices."""
    from oracle import oracle as ora
    B, H, S, D = q.shape
    n, t_total = 0, 0.0
    while n < max_slices and (t_total < budget_s or n == 0):
        b, h = n % B, (n * 7) % H
        sl = [t[b, h].float().cpu().numpy()[None] for t in (q, k, v, do)]
        t0 = time.perf_counter()
        ora.attn_fwd(*sl[:3], scale, causal)
        ora.attn_bwd(*sl, scale, causal)
        t_total += time.perf_counter() - t0
        n += 1
    flops = attn_flops(1, 1, S, D, causal) * n
    return {"value": flops / t_total / 1e12, "unit": UNIT, "cores": ora.num_threads(),
            "kind": "port",
            "sample": f"{n} of {B * H} (b,h) slices (S={S}, D={D}), fwd+bwd with S x S "
                      f"matrices materialised as the reference does; {t_total:.1f} s"}


def run_reference(a):
    """Reference arm: the reference's CPU attention path (C restatement) on host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    from oracle import oracle as ora
    ora.build()
    causal = not a.no_causal
    S, D = a.seq, a.head_dim
    scale = 1.0 / math.sqrt(D)
    rng = np.random.default_rng(a.seed)
    sl = [ora.round_bf16(rng.standard_normal((1, S, D), dtype=np.float32)) for _ in range(4)]
    sl[0] = ora.rope_fwd(sl[0], a.rope_theta)
    sl[1] = ora.rope_fwd(sl[1], a.rope_theta)

    def step():
        ora.attn_fwd(*sl[:3], scale, causal)
        g = ora.attn_bwd(*sl, scale, causal)
        ora.rope_bwd(g[0], a.rope_theta)
        ora.rope_bwd(g[1], a.rope_theta)

    for _ in range(a.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        step()
    dt = (time.perf_counter() - t0) / a.steps
    value = attn_flops(1, 1, S, D, causal) / dt / 1e12
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), bf16-rounded)", "config": config_of(a, a.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": ora.num_threads(),
                         "kind": "port",
                         "sample": f"one (b,h) slice (S={S}, D={D}) per step: RoPE, fwd+bwd with "
                                   "S x S matrices materialised, RoPE bwd"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is Rust+wgpu and cannot be built or run here; this arm times the "
                "C restatement of its CPU kernels (oracle/) on all host cores",
    }
    print(json.dumps(out), flush=True)
    return 0


def run_haelixe(a):
    import torch
    import torch.distributed as dist

    import haelixe_b200 as hx
    from haelixe_b200 import _native as N

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if a.compute_priority == "high":
        torch.cuda.set_stream(torch.cuda.Stream(device=dev, priority=-1))
    group = None
    if world > 1:
        # Control (barriers, max over ranks) over gloo on the host; the data
        # path's only collective is the library's own NCCL group.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        from haelixe_b200.sharding import HeadGroup
        group = HeadGroup.bootstrap(local, flags=a.exchange_flags, timeout_ms=120000)
    B, H, S, D = a.batch, a.heads, a.seq, a.head_dim
    causal = not a.no_causal
    if H % world:
        raise SystemExit(f"heads {H} not divisible by {world} GPUs")
    Hl = H // world
    scale = 1.0 / math.sqrt(D)
    ctx = hx.context(local)
    dt = torch.float32 if a.dtype == "f32" else torch.bfloat16

    # Inputs for this rank's heads, generated from the global head index so a
    # head's data does not depend on the GPU count.
    def gen(which):
        if a.head_layout == "bshd":
            t = torch.empty(B, S, Hl, D, device=dev, dtype=dt).permute(0, 2, 1, 3)
        else:
            t = torch.empty(B, Hl, S, D, device=dev, dtype=dt)
        for hl in range(Hl):
            g = torch.Generator(device=dev).manual_seed(a.seed * 1000003 + which * 1009 + rank * Hl + hl)
            t[:, hl] = torch.randn(B, S, D, device=dev, generator=g).to(dt)
        return t

    q, k, v, do = (gen(i) for i in range(4))

    def buffers(q, k, v, do):
        """Device tensors of one step: inputs, intermediates and results."""
        e = torch.empty_like
        return dict(q=q, k=k, v=v, do=do, qr=e(q), kr=e(k), o=e(q), dv=e(q), dq0=e(q), dk0=e(q),
                    lse=torch.empty(B * Hl * S, device=dev, dtype=torch.float32))

    bufs0 = buffers(q, k, v, do)
    if world > 1:
        # The forward writes O straight into this rank's slot of the group's
        # gather buffer, so the all-gather runs in place.
        gbuf = group.gather_buffer((B, Hl, S, D), dt)
        bufs0["o"] = (gbuf[rank].view(B, S, Hl, D).permute(0, 2, 1, 3) if a.head_layout == "bshd"
                      else gbuf[rank])
        merged = torch.empty(B, S, H, D, device=dev, dtype=dt)
    qr, kr, o, lse = bufs0["qr"], bufs0["kr"], bufs0["o"], bufs0["lse"]
    dv, dq0, dk0 = bufs0["dv"], bufs0["dq0"], bufs0["dk0"]
    stream = torch.cuda.current_stream(dev)
    ev = {}

    def step(timed=False, b=None):
        b = bufs0 if b is None else b
        q, k, v, do, qr, kr, o, lse = (b[n] for n in ("q", "k", "v", "do", "qr", "kr", "o", "lse"))
        dv, dq0, dk0 = b["dv"], b["dq0"], b["dk0"]
        if timed:
            ev.setdefault("f0", []).append(torch.cuda.Event(enable_timing=True))
            ev.setdefault("f1", []).append(torch.cuda.Event(enable_timing=True))
            ev.setdefault("b1", []).append(torch.cuda.Event(enable_timing=True))
        if a.rope_launches == 1:
            hx.rope_forward_qk(q, k, a.rope_theta, out_q=qr, out_k=kr)
        else:
            hx.rope_forward(q, a.rope_theta, out=qr)
            hx.rope_forward(k, a.rope_theta, out=kr)
        if timed:
            ev["f0"][-1].record(stream)
        hx.attn_forward(qr, kr, v, scale, causal, out=o, lse=lse)
        if timed:
            ev["f1"][-1].record(stream)
        if world > 1:
            # NCCL all-gather + reassembly into [B, S, H, D] on the group's
            # side stream, after the forward and beside the backward.
            group.all_gather(o, merged, "bshd")
        # Backward with the rotary embedding's backward fused into the last
        # writes of dQ and dK: dq0, dk0 are the gradients of q, k before RoPE.
        hx.attn_backward(qr, kr, v, o, lse, do, scale, causal, dq=dq0, dk=dk0, dv=dv,
                         rope_base=a.rope_theta)
        if timed:
            ev["b1"][-1].record(stream)
        if world > 1:
            group.wait()  # the step ends with O gathered and merged on every rank

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        # Untimed check of the gathered output: this rank's heads of `merged`
        # are its own O, and every rank holds the same merged tensor.
        own = torch.equal(merged[:, :, rank * Hl:(rank + 1) * Hl], o.transpose(1, 2))
        cs = merged.float().sum(dtype=torch.float64).reshape(1).cpu()
        lo, hi = cs.clone(), cs.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        ok = torch.tensor([1 if (own and lo.item() == hi.item()) else 0])
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if ok.item() != 1:
            raise SystemExit(f"rank {rank}: gathered heads do not match (own slice {own})")
        dist.barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    launches0 = N.lib().hx_kernel_launches(ctx.handle)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_start.record(stream)
    for _ in range(a.steps):
        step(timed=True)
    t_end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    launches = N.lib().hx_kernel_launches(ctx.handle) - launches0
    ms = t_start.elapsed_time(t_end) / a.steps
    fwd_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(ev["f0"], ev["f1"]))
    bwd_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(ev["f1"], ev["b1"]))
    t = torch.tensor([ms, fwd_ms, bwd_ms], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_ms, bwd_ms = t.tolist()
    total_flops = attn_flops(B, H, S, D, causal)
    value = total_flops / (ms * 1e-3) / 1e12

    # End to end through the C ABI with host buffers: H2D of q, k, v, dO
    # from pinned memory, the step, D2H of o, dq, dk, dv every step.
    e2e = None
    if not a.no_e2e:
        bufs1 = buffers(*(torch.empty_like(q) for _ in range(4)))
        e2e = e2e_measure(a, ctx, N, torch, dev, world, [bufs0, bufs1], step, total_flops)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(qr, kr, v, do, scale, causal)

    peak, peak_src = choose_peak(measured_peaks(), ms * a.steps * 1e-3)
    dom = "bwd" if bwd_ms >= fwd_ms else "fwd"
    dom_flops = (10.0 if dom == "bwd" else 4.0) * B * Hl * S * S * D * (0.5 if causal else 1.0)
    dom_ms = bwd_ms if dom == "bwd" else fwd_ms
    achieved = dom_flops / (dom_ms * 1e-3) / 1e12
    # f32 runs three bf16 MMAs per product: the tensor pipe does 3x the
    # attention FLOPs, and that issued work is what the bf16 peak bounds.
    split = 3.0 if a.dtype == "f32" else 1.0
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": a.dtype, "data": "synthetic (seeded N(0,1))",
            "config": config_of(a, world),
            "roofline": {"bound": "tensor", "kernel": f"attention {dom} ({ctx.last_path})",
                         "achieved": achieved, "peak": peak, "peak_source": peak_src,
                         "unit": "TFLOP/s", "frac": achieved * split / peak,
                         "mma_flops_per_flop": split,
                         "traffic": traffic_per_launch(dom, B, Hl, S, D) if split == 1.0 else None},
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
            "fraction_of_peak": value / world / peak,
            "gpu_launches": int(launches),
            "kernel_path": ctx.last_path,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        group.close()
        dist.destroy_process_group()
    return 0


def e2e_measure(a, ctx, N, torch, dev, world, sets, step, total_flops):
    """The step with its inputs copied in from pinned host memory and its
    results copied back out every step, through hx_copy_*_async, pipelined as a
    training or serving loop runs: copies in on one stream, compute on the
    launch stream, copies out on a third, over two device buffer sets, so step
    i's results go out while step i+1's inputs come in (PCIe is full duplex)
    and the compute overlaps both. Every step moves all of its bytes inside the
    timed region. The timed window runs from the first step's first upload to
    the last step's last download, so it includes the pipeline's fill and
    drain (one un-overlapped upload and download); 20 steps keep those to a
    few percent of the window (about 0.5 s at the attention workload)."""
    import ctypes
    steps = max(2, a.e2e_steps)
    ins, outs = ("q", "k", "v", "do"), ("o", "dq0", "dk0", "dv")
    h_in = [torch.empty(sets[0][n].shape, dtype=sets[0][n].dtype, pin_memory=True) for n in ins]
    for h, n in zip(h_in, ins):
        h.copy_(sets[0][n])
    h_out = [[torch.empty(sets[0][n].shape, dtype=sets[0][n].dtype, pin_memory=True) for n in outs]
             for _ in sets]
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    in_done = [torch.cuda.Event() for _ in sets]
    comp_done = [torch.cuda.Event() for _ in sets]
    out_done = [torch.cuda.Event() for _ in sets]
    bi = sum(sets[0][n].numel() * sets[0][n].element_size() for n in ins)
    bo = sum(sets[0][n].numel() * sets[0][n].element_size() for n in outs)

    def copy(stream, dst, src, nbytes, h2d):
        ctx.use_stream(stream)
        fn = N.lib().hx_copy_h2d_async if h2d else N.lib().hx_copy_d2h_async
        N.check(fn(ctx.handle, ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes), ctx.handle)

    def run(n):
        for i in range(n):
            j = i % len(sets)
            b = sets[j]
            if i >= len(sets):
                s_in.wait_event(comp_done[j])  # step i-2 is done reading this set's inputs
            for h, name in zip(h_in, ins):
                t = b[name]
                copy(s_in, t.data_ptr(), h.data_ptr(), t.numel() * t.element_size(), True)
            in_done[j].record(s_in)
            comp.wait_event(in_done[j])
            if i >= len(sets):
                comp.wait_event(out_done[j])  # step i-2's results in this set are out
            with torch.cuda.stream(comp):
                step(b=b)
            comp_done[j].record(comp)
            s_out.wait_event(comp_done[j])
            for h, name in zip(h_out[j], outs):
                t = b[name]
                copy(s_out, h.data_ptr(), t.data_ptr(), t.numel() * t.element_size(), False)
            out_done[j].record(s_out)
        ctx.use_stream(comp)

    run(2)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    run(steps)
    s_out.wait_stream(comp)
    s_out.wait_stream(s_in)
    t1.record(s_out)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    t = torch.tensor([ms], dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = t.item()
    return {"value": total_flops / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms,
            "steps": steps, "pipelined": "H2D / compute / D2H on three streams, two buffer sets",
            "h2d_bytes_per_step": int(bi), "d2h_bytes_per_step": int(bo)}


def run_block_stack(a):
    """The block-stack training step (context workload, 1 GPU; under torchrun
    only rank 0 runs it)."""
    import torch

    import haelixe_b200 as hx
    from haelixe_b200 import _native as N

    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, S, Hd, H, L, V = 2, 4096, 2048, 16, 8, 32000
    model = hx.nn.BlockStack(V, Hd, H, L, device=dev, dtype=torch.bfloat16, rope_base=10000.0, causal=True,
                             init_std=0.02, seed=a.seed)
    params = model.parameters()
    opt = hx.optim.AdamW(1e-4)
    ctx = hx.context(local)
    N.check(N.lib().hx_set_gemm_backend(ctx.handle, 1 if a.gemm_backend == "cublas" else 0), ctx.handle)
    g = torch.Generator().manual_seed(a.seed)
    ids_h = torch.randint(0, V, (B, S), generator=g, dtype=torch.int32).pin_memory()
    tgt_h = torch.randint(0, V, (B * S,), generator=g, dtype=torch.int32).pin_memory()
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    ids = torch.empty_like(ids_h, device=dev)
    tgt = torch.empty_like(tgt_h, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        ids.copy_(ids_h, non_blocking=True)
        tgt.copy_(tgt_h, non_blocking=True)
        loss = model.loss(ids, tgt)
        loss.backward()
        opt.step([(q, q.grad) for q in params])
        for q in params:
            q.grad = None
        loss_h.copy_(loss, non_blocking=True)

    losses = []
    for _ in range(a.warmup):
        step()
        torch.cuda.synchronize()
        losses.append(float(loss_h.item()))
    sampler = ClockSampler(local)
    sampler.start()
    launches0 = N.lib().hx_kernel_launches(ctx.handle)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record(stream)
    for _ in range(a.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / a.steps
    n_lin = sum(q.numel() for q in params if q.dim() == 2 and q is not model.embed.weight)
    flops = 6.0 * n_lin * B * S + L * attn_flops(B, H, S, Hd // H, True)
    tok_s = B * S / (ms * 1e-3)
    print(json.dumps({
        "metric": "block-stack training step tokens/s (context workload)", "value": tok_s, "unit": "tokens/s",
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform token ids, N(0,0.02) init)",
        "config": {"workload": f"{L}-block TransformerBlock LM d{Hd} H{H}x{Hd // H} MLP {4 * Hd} vocab {V} "
                               f"B{B} S{S} causal, bf16 + f32 master, AdamW",
                   "parameters": int(sum(q.numel() for q in params)),
                   "gemm": a.gemm_backend,
                   "l2": "activations and weights far larger than L2"},
        "model_tflops": flops / (ms * 1e-3) / 1e12, "flops_per_step": flops,
        "loss_warmup": losses, "loss": float(loss_h.item()),
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": int(ids_h.numel() * 4 + tgt_h.numel() * 4),
                "d2h_bytes_per_step": 4, "note": "token ids in and the loss out every step, inside the timed region"},
        "gpu_launches": int(N.lib().hx_kernel_launches(ctx.handle) - launches0),
        "clocks": clocks,
    }), flush=True)
    return 0


def run_linear(a):
    """One bf16 Linear forward (y = x W + b, W [in, out]) through hx_linear_fwd:
    the GEMM of the block stack's projections, on the backend --gemm-backend
    selects (context workload, 1 GPU)."""
    import ctypes

    import torch

    import haelixe_b200 as hx
    from haelixe_b200 import _native as N

    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    M, K, Nn = (int(x) for x in a.linear_shape.split(","))
    g = torch.Generator(device=dev).manual_seed(a.seed)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(K, Nn, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
    b = torch.randn(Nn, device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty(M, Nn, device=dev, dtype=torch.bfloat16)
    ctx = hx.context(local)
    ctx.use_stream()
    L = N.lib()
    N.check(L.hx_set_gemm_backend(ctx.handle, 1 if a.gemm_backend == "cublas" else 0), ctx.handle)
    p = lambda t: ctypes.c_void_p(t.data_ptr())

    def step():
        N.check(L.hx_linear_fwd(ctx.handle, N.HX_BF16, p(x), p(w), p(b), p(y), M, K, Nn), ctx.handle)

    for _ in range(a.warmup):
        step()
    launches0 = L.hx_kernel_launches(ctx.handle)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(a.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / a.steps
    tf = 2.0 * M * K * Nn / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": "linear forward TFLOP/s (context workload)", "value": tf, "unit": "TFLOP/s", "n_gpus": 1,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": f"linear y = x W + b, rows {M}, in {K}, out {Nn}", "gemm": a.gemm_backend,
                   "gemm_path": {1: "cublas", 2: "tcgen05"}.get(L.hx_last_gemm_path(ctx.handle), "none")},
        "gpu_launches": int(L.hx_kernel_launches(ctx.handle) - launches0),
    }), flush=True)
    return 0


def main():
    a = parse()
    if a.workload == "linear":
        return run_linear(a)
    if a.workload == "block_stack":
        return run_block_stack(a)
    if a.impl == "reference":
        return run_reference(a)
    return run_haelixe(a)


if __name__ == "__main__":
    sys.exit(main())
