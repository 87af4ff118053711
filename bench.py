"""Benchmark of the B200 operator ladder (headline: causal flash-attention forward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extras]

One step = one flash_attention_fwd_fused forward over the benchmarked configuration on every GPU:
Q, K, V bf16 [B=16, H=32, S=8192, D=128], causal, scale 1/sqrt(128), O bf16 + lse fp32.
Weak scaling: each rank owns a full 16x32-head shard of a global batch of 16*N (the work shards
over batch x heads with no exchange, so there is no collective on the data path).  Time is
measured with CUDA events on the launching stream between barriers, max over ranks; rank 0 prints
one JSON line.  Inputs (3.2 GB per GPU) are larger than the 126 MB L2.

Extra keys of the JSON line:
  roofline     the flash-attention kernel against the measured dense bf16 peak
  e2e          the same metric through the C ABI's host-buffer entry point
               (hc_flash_attention_fwd_fused_host: pinned H2D copies, kernel, D2H copies, per step)
  cpu_baseline the reference golden (compiled from the reference sources into oracle/_ref) on the
               host cores, on a bounded sample (rank 0, N=1 only)
  ops          the other benchmarked configurations (non-causal attention, matmul_bias, layer_norm,
               rms_norm_rope_fused, elementwise_add) with their roofline fractions
  clocks       SM clocks and throttle reasons sampled with nvidia-smi during the timed region

--impl reference times the reference's own CPU implementation of the path (oracle/_ref, all host
threads) on the same metric and prints the same JSON line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "ascend-npu-harness_b200"
sys.path.insert(0, str(PKG))

FA_B, FA_H, FA_S, FA_D = 16, 32, 8192, 128
METRIC = "flash-attn fwd TFLOP/s (% BF16 peak); norm/RoPE GB/s (% HBM); 1/2/4/8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def fa_flops(B, H, S_q, S_k, D, causal) -> float:
    """4*D FLOPs per visible (query, key) pair (QK^T and PV); causal counts S(S+1)/2 pairs."""
    pairs = S_q * (S_q + 1) / 2 if causal else S_q * S_k
    return 4.0 * B * H * D * pairs


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# op -> the profiles/<file>.md that records its ncu capture (named for the kernel and workload)
PROFILE_FILES = {
    "flash_attention_fwd_causal": "flash_attention_fwd_causal_B16H32S8192D128",
    "matmul_bias": "matmul_bias_8192x8192x8192",
    "layer_norm": "layer_norm_16384x4096_bf16",
    "rms_norm_rope_fused": "rms_norm_rope_fused_8x4096x32x128_bf16",
    "elementwise_add": "elementwise_add_4096x8192_f16",
    "activation_gelu_silu": "activation_gelu_silu_16384x4096_bf16",
    "transpose_2d_4d": "transpose_2d_4d_8192x8192_bf16",
}


def profile_traffic(op: str):
    """Per-launch DRAM bytes recorded from an ncu capture ("traffic_bytes_per_launch: N" in its profile)."""
    name = PROFILE_FILES.get(op)
    if name is None:
        return None
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


# ------------------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid: str | None):
        self.uuid = device_uuid
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
        if self.uuid:
            cmd += ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
                power.append(float(parts[2]))
            except ValueError:
                continue
            for n, flag in zip(names, parts[4:8]):
                if flag.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "power_w_max": max(power),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------
# distributed plumbing (one process per GPU; no collective on the data path)
# ------------------------------------------------------------------------------------------------
class Dist:
    """One process per GPU (RANK / WORLD_SIZE / LOCAL_RANK from torchrun).  NCCL carries only the
    barrier and the max-over-ranks of the timed region; `backend="gloo"` runs the same logic on
    CPU ranks.  The process-group timeout is short so that ranks waiting for a rank that died end
    with an error instead of waiting for good."""

    def __init__(self, world: int, backend: str | None = None, timeout_s: float = 120.0):
        import datetime

        import torch
        import torch.distributed as dist

        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", str(world)))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = dist if self.world > 1 else None
        self.backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        self.device = "cuda" if self.backend == "nccl" else "cpu"
        if self.dist:
            timeout = datetime.timedelta(seconds=timeout_s)
            if self.backend == "nccl":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group(self.backend, timeout=timeout)

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if not self.dist:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_gather_into(self, out, t):
        """out[r] = rank r's `t` on every rank (out has shape (world, *t.shape)).  NCCL gathers into
        the one buffer; gloo, which has no single-buffer form, gathers into its slices."""
        if not self.dist:
            out[0].copy_(t)
            return
        if self.backend == "nccl":
            self.dist.all_gather_into_tensor(out, t.contiguous())
        else:
            self.dist.all_gather(list(out.unbind(0)), t.contiguous())

    def close(self):
        if self.dist:
            self.dist.barrier()
            self.dist.destroy_process_group()


def whole_job_rate(units_per_rank: float, world: int, ms_max: float) -> float:
    """Weak scaling: every rank processes `units_per_rank`; the job's rate is all ranks' units
    divided by the slowest rank's time (units per second)."""
    return world * units_per_rank / (ms_max * 1e-3)


# ------------------------------------------------------------------------------------------------
# timing helpers
# ------------------------------------------------------------------------------------------------
def time_launches(fn, steps: int, warmup: int, d: Dist, flush=None, spin: bool = True):
    """Returns (ms per launch averaged over `steps`, max over ranks).

    Without `flush` (every workload here reads more than the 126 MB L2 per launch) the `steps`
    launches run back to back between one pair of events; a spin kernel queued first keeps the
    GPU busy while the host enqueues them, so host launch overhead does not leave the GPU idle
    inside the timed region.  With `flush`, every launch is bracketed by its own events and an
    L2-flushing write runs between launches (outside them).  `spin=False` for host-synchronous
    steps (the e2e runner), whose own copies must start inside the timed region."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    if flush is None:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if spin:
            torch.cuda._sleep(max(2_000_000, 400_000 * steps))  # ~0.2 ms of spinning per queued launch
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / steps
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for s, e in evs:
            flush()
            s.record()
            fn()
            e.record()
        torch.cuda.synchronize()
        ms = sum(s.elapsed_time(e) for s, e in evs) / steps
    d.barrier()
    return d.max(ms)


# ------------------------------------------------------------------------------------------------
# the reference arm: the reference's own CPU golden on the host cores
# ------------------------------------------------------------------------------------------------
def cpu_fa_sample(threads: int, seconds_target: float = 0.0):
    """Times the reference golden (oracle/_ref) -- or, if it was not built, the oracle port -- on a
    bounded sample of the workload: `threads` heads of the causal S x S top-left corner (S=1024,
    D=128, N(0,1) inputs), one head per host thread.  Returns (TFLOP/s, seconds, info)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle as om

    o = om.Oracle()
    kind = "reference" if om.reference_available() else "port"
    S, D = 1024, FA_D
    heads = threads
    q = o.normal(heads * S * D, 0).reshape(1, heads, S, D)
    k = o.normal(heads * S * D, 1).reshape(1, heads, S, D)
    v = o.normal(heads * S * D, 2).reshape(1, heads, S, D)
    q, k, v = (o.from_bf16(o.to_bf16(a)) for a in (q, k, v))
    sc = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    t0 = time.perf_counter()
    if kind == "reference":
        om.Reference().flash_attention_fwd(q, k, v, sc, 1, threads=threads)
    else:
        o.flash_attention_fwd(q, k, v, sc, 1, threads=threads)
    dt = time.perf_counter() - t0
    flops = fa_flops(1, heads, S, S, D, True)
    info = {"kind": kind, "cores": threads,
            "sample": f"{heads} heads x causal top-left {S}x{S} corner, D={D} (one head per thread), "
                      f"{'reference golden compiled from its sources' if kind == 'reference' else 'oracle port'}"}
    return flops / dt / 1e12, dt, info


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return  # only rank 0 runs the CPU reference; the others exit without work
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_fa_sample(threads)
    rates, secs, info = [], [], None
    for _ in range(args.steps):
        r, s, info = cpu_fa_sample(threads)
        rates.append(r)
        secs.append(s)
    value = statistics.mean(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.mean(secs),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic: Q,K,V ~ N(0,1) (bf16-quantised, widened to fp32 for the golden)",
        "config": {"workload": f"flash_attention_fwd_fused causal D={FA_D}: reference CPU golden on a bounded sample",
                   "global_batch": FA_B * world, "seq_len": FA_S, "heads": FA_H, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", **info},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
def run_ours(args):
    import ctypes

    import torch

    d = Dist(args.gpus)
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    import hc

    lib = hc.load()  # raises if the CUDA library is missing: there is no CPU fallback
    peaks, peak_src = load_peaks()
    n = d.world
    fa_b = args.fa_batch

    # ---------------- headline: causal flash attention -----------------------------------------
    gens = [torch.Generator(device=dev).manual_seed(s + 3 * d.rank) for s in (0, 1, 2)]
    q, k, v = (torch.randn((fa_b, FA_H, FA_S, FA_D), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
               for g in gens)
    o = torch.empty_like(q)
    lse = torch.empty((fa_b, FA_H, FA_S), dtype=torch.float32, device=dev)
    step = lambda: hc.flash_attention_fwd(q, k, v, True, out=o, lse=lse)  # noqa: E731
    step()
    torch.cuda.synchronize()
    hc.check_device_error()
    if lib.hc_flash_attention_last_path() != 1:
        raise SystemExit("flash attention did not take the tcgen05 path")
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    d.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)  # let the sampler's first lines land inside the busy window
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(args.steps):
        step()
    e_ev.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    d.barrier()
    ms_local = s_ev.elapsed_time(e_ev) / args.steps
    hc.check_device_error()
    ms = d.max(ms_local)
    flops_rank = fa_flops(fa_b, FA_H, FA_S, FA_S, FA_D, True)
    value = whole_job_rate(flops_rank, n, ms) / 1e12
    achieved = flops_rank / (ms_local * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "peak_source": f"{peak_src} bf16_tflops (burst: the kernel is timed alone)",
                "traffic": profile_traffic("flash_attention_fwd_causal"),
                "algorithmic_flops_per_launch": flops_rank}

    # ---------------- optional: the sharded outputs gathered onto every rank (after timing) -----------
    gather = None
    if args.gather_outputs and n > 1:
        full = torch.empty((n,) + tuple(o.shape), dtype=o.dtype, device=dev)
        d.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        d.all_gather_into(full, o)
        g1.record()
        torch.cuda.synchronize()
        g_ms = d.max(g0.elapsed_time(g1))
        own_ok = 1.0 - d.max(0.0 if torch.equal(full[d.rank], o) else 1.0)  # 1 only if every rank's slice is its own O
        gather = {"what": f"O [{fa_b}, {FA_H}, {FA_S}, {FA_D}] bf16 of every rank onto every rank (NCCL all-gather)",
                  "bytes_per_rank": o.numel() * 2, "gathered_bytes": full.numel() * 2, "ms": g_ms,
                  "gb_per_s_in_per_rank": (n - 1) * o.numel() * 2 / (g_ms * 1e-3) / 1e9, "own_slices_equal": own_ok == 1.0}
        del full
    del o

    # ---------------- e2e through the host-buffer C entry point -----------------------------------
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        ho = torch.empty_like(hq).pin_memory()
        hl = torch.empty((fa_b, FA_H, FA_S), dtype=torch.float32).pin_memory()
        t = hc.FlashAttentionFwdFusedTiling(fa_b, FA_H, FA_S, FA_S, FA_D, FA_D, 1.0 / math.sqrt(FA_D), 1)
        ws = ctypes.c_size_t()
        hc.check(lib.hc_flash_attention_fwd_fused_host_workspace_size(ctypes.byref(t), hc.DT_BF16, ctypes.byref(ws)))
        work = torch.empty(ws.value, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream().cuda_stream

        def e2e_step():
            hc.check(lib.hc_flash_attention_fwd_fused_host(hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), ho.data_ptr(),
                                                           hl.data_ptr(), ctypes.byref(t), hc.DT_BF16, work.data_ptr(),
                                                           ws.value, stream))

        e2e_steps = max(2, min(args.steps, 5))
        e2e_ms = time_launches(e2e_step, e2e_steps, 1, d, spin=False)
        h2d = 3 * q.numel() * 2
        d2h = ho.numel() * 2 + hl.numel() * 4
        e2e = {"value": n * flops_rank / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "hc_flash_attention_fwd_fused_host (pinned host buffers, chunked copies overlapped with the kernel)"}
        del hq, hk, hv, ho, hl, work
    del q, k, v, lse
    torch.cuda.empty_cache()

    # ---------------- the other benchmarked configurations ------------------------------------
    ops = {} if args.no_extras else run_extras(hc, d, dev, peaks, args)

    # ---------------- CPU baseline (rank 0, N=1) --------------------------------------------------
    cpu = None
    if d.rank == 0 and n == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        rate, secs, info = cpu_fa_sample(threads)
        cpu = {"value": rate, "unit": "TFLOP/s", **info, "seconds": secs}

    if d.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: Q,K,V ~ N(0,1) from torch's seeded CUDA generator (seeds 0/1/2, +3 per rank), bf16",
            "config": {"workload": f"flash_attention_fwd_fused causal bf16 B{fa_b} H32 S8192 D128 per GPU (O bf16 + lse fp32)",
                       "global_batch": fa_b * n, "seq_len": FA_S, "heads": FA_H, "head_dim": FA_D, "causal": True,
                       "parallelism": f"dp{n}: batch x heads sharded, no collective",
                       "l2": "inputs 3.2 GB per GPU > 126 MB L2; no flush needed"},
            "gpu_launches": args.steps,
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks, "ops": ops,
            **({"gather": gather} if gather else {}),
            "device": torch.cuda.get_device_name(dev),
        }
        print(json.dumps(line), flush=True)
    d.close()


EXTRA_OPS = ("flash_attention_fwd_noncausal", "matmul_bias", "layer_norm", "rms_norm_rope_fused", "elementwise_add",
             "axpy_scalar_affine", "broadcast_binary", "activation_gelu_silu", "reduce_sum_lastdim", "transpose_2d_4d")
# The last five ops have no configuration of their own in the reference's benchmark list; they are
# timed on sized analogs of the layer_norm shape (134 MB of 16-bit input per launch), stated in
# each entry's "config".
ANALOG_OPS = EXTRA_OPS[5:]


def settle():
    """Each configuration after the headline starts from an idle GPU: after the 8192^3 GEMM's power
    burst the power controller holds the clock down for about a second, and the next kernel
    (layer_norm here) measured up to 10 points low when timed at once."""
    import torch

    torch.cuda.synchronize()
    time.sleep(1.0)


def run_extras(hc, d: Dist, dev, peaks, args, want=EXTRA_OPS) -> dict:
    """The other benchmarked configurations, each timed alone (W=3, 20 launches)."""
    import torch

    out = {}
    if not want:
        return out
    steps, warm = 20, 3
    # The bandwidth workloads below each read more than the 126 MB L2 per launch (layer_norm
    # 134 MB, rms_norm_rope 268 MB, elementwise_add 134 MB), so they run back to back without an
    # L2 flush; consecutive launches alternate between two independent buffer sets, so a launch
    # can neither re-read the previous launch's inputs nor rewrite its still-dirty outputs in L2.
    hbm = peaks["hbm_gbs"]
    flip = [0]

    def alternate(sets):
        def nxt():
            flip[0] ^= 1
            return sets[flip[0]]
        return nxt
    g = torch.Generator(device=dev).manual_seed(0)

    def bw_entry(name, bytes_, ms, launches=1):
        gbs = bytes_ / (ms * 1e-3) / 1e9
        out[name] = {"value": d.world * gbs, "unit": "GB/s", "per_gpu": gbs, "ms": ms,
                     "timing": f"after a 1 s idle pause, {steps} back-to-back launches alternating two buffer sets, "
                               "no L2 flush (each reads > 126 MB)",
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                                  "algorithmic_bytes_per_launch": bytes_, "traffic": profile_traffic(name)}}

    if "flash_attention_fwd_noncausal" in want:  # same shapes as the headline, no mask
        q, k, v = (torch.randn((FA_B, FA_H, FA_S, FA_D), generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
        o = torch.empty_like(q)
        lse = torch.empty((FA_B, FA_H, FA_S), dtype=torch.float32, device=dev)
        settle()
        ms = time_launches(lambda: hc.flash_attention_fwd(q, k, v, False, out=o, lse=lse), 5, warm, d)
        fl = fa_flops(FA_B, FA_H, FA_S, FA_S, FA_D, False)
        tf = fl / (ms * 1e-3) / 1e12
        out["flash_attention_fwd_noncausal"] = {
            "value": d.world * tf, "unit": "TFLOP/s", "per_gpu": tf, "ms": ms,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "algorithmic_flops_per_launch": fl}}
        del q, k, v, o, lse

    if "matmul_bias" in want:  # 8192^3 bf16, A, B ~ N(0,1)/sqrt(K), bias ~ N(0, 0.1)
        M = K = N = 8192
        A = (torch.randn((M, K), generator=g, device=dev) / math.sqrt(K)).to(torch.bfloat16)
        B = (torch.randn((K, N), generator=g, device=dev) / math.sqrt(K)).to(torch.bfloat16)
        bias = (torch.randn((N,), generator=g, device=dev) * 0.1).to(torch.bfloat16)
        C = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        settle()
        ms = time_launches(lambda: hc.matmul_bias(A, B, bias, out=C), steps, warm, d)
        fl = 2.0 * M * N * K
        tf = fl / (ms * 1e-3) / 1e12
        out["matmul_bias"] = {"value": d.world * tf, "unit": "TFLOP/s", "per_gpu": tf, "ms": ms,
                              "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"],
                                           "unit": "TFLOP/s", "frac": tf / peaks["bf16_tflops"],
                                           "algorithmic_flops_per_launch": fl,
                                           "algorithmic_bytes_per_launch": 3 * M * N * 2 + N * 2,
                                           "traffic": profile_traffic("matmul_bias")}}
        del A, B, bias, C

    if "layer_norm" in want:  # [16384, 4096] bf16, fp32 gamma/beta
        gamma = torch.rand((4096,), generator=g, device=dev) + 0.5
        beta = torch.rand((4096,), generator=g, device=dev) * 0.2 - 0.1
        sets = []
        for _ in range(2):
            x = torch.randn((16384, 4096), generator=g, device=dev).to(torch.bfloat16)
            sets.append((x, torch.empty_like(x)))
        nxt = alternate(sets)

        def ln_step():
            xx, yy = nxt()
            hc.layer_norm(xx, gamma, beta, 1e-5, y=yy)

        settle()
        ms = time_launches(ln_step, steps, warm, d)
        bw_entry("layer_norm", 2 * x.numel() * 2 + 2 * 4096 * 4, ms)
        del x, sets

    if "rms_norm_rope_fused" in want:  # [8, 4096, 32, 128] bf16, rotate-half, fp32 cos/sin [4096, 64]
        w = torch.rand((128,), generator=g, device=dev) + 0.5
        pos = torch.arange(4096, device=dev, dtype=torch.float32)[:, None]
        inv = 1.0 / (10000.0 ** (torch.arange(64, device=dev, dtype=torch.float32) * 2 / 128))
        cos, sin = torch.cos(pos * inv).contiguous(), torch.sin(pos * inv).contiguous()
        sets = []
        for _ in range(2):
            x = torch.randn((8, 4096, 32, 128), generator=g, device=dev).to(torch.bfloat16)
            sets.append((x, torch.empty_like(x)))
        nxt = alternate(sets)

        def rms_step():
            xx, yy = nxt()
            hc.rms_norm_rope_fused(xx, w, cos, sin, 128, 1e-6, heads=32, rope_style=1, out=yy)

        settle()
        ms = time_launches(rms_step, steps, warm, d)
        bw_entry("rms_norm_rope_fused", 2 * x.numel() * 2 + 128 * 4 + 2 * cos.numel() * 4, ms)
        del x, sets

    if "elementwise_add" in want:  # fp16 [4096, 8192], U[-1, 1]
        sets = []
        for _ in range(2):
            a = (torch.rand((4096, 8192), generator=g, device=dev) * 2 - 1).to(torch.float16)
            b = (torch.rand((4096, 8192), generator=g, device=dev) * 2 - 1).to(torch.float16)
            sets.append((a, b, torch.empty_like(a)))
        nxt = alternate(sets)
        settle()
        ms = time_launches(lambda: hc.elementwise_add(*nxt()), steps, warm, d)
        bw_entry("elementwise_add", 3 * a.numel() * 2, ms)
        del a, b, sets
    if any(op in want for op in ANALOG_OPS):
        out.update(run_analogs(hc, d, dev, peaks, want, steps, warm, alternate))
    torch.cuda.empty_cache()
    return out


def run_analogs(hc, d: Dist, dev, peaks, want, steps, warm, alternate) -> dict:
    """Sized analogs for the ops without a configuration of their own: bf16, 134 MB of input."""
    import torch

    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    hbm = peaks["hbm_gbs"]
    R, K = 16384, 4096  # the layer_norm shape

    def rnd(*shape):
        return torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)

    def entry(name, config, bytes_, make_set, run):
        sets = [make_set() for _ in range(2)]
        nxt = alternate(sets)
        settle()
        ms = time_launches(lambda: run(*nxt()), steps, warm, d)
        gbs = bytes_ / (ms * 1e-3) / 1e9
        out[name] = {"value": d.world * gbs, "unit": "GB/s", "per_gpu": gbs, "ms": ms, "config": config,
                     "timing": f"after a 1 s idle pause, {steps} back-to-back launches alternating two buffer sets, no L2 flush",
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                                  "algorithmic_bytes_per_launch": bytes_, "traffic": profile_traffic(name)}}

    n = R * K
    if "axpy_scalar_affine" in want:
        entry("axpy_scalar_affine", f"analog: bf16 [{R}, {K}], y = 0.5 x - 1", 2 * n * 2,
              lambda: (rnd(R, K), torch.empty((R, K), dtype=torch.bfloat16, device=dev)),
              lambda x, y: hc.axpy_scalar_affine(x, 0.5, -1.0, y=y))
    if "broadcast_binary" in want:
        B, Cc, H, W = 16, 256, 128, 128
        y_ = rnd(B, Cc)
        bias = rnd(Cc)
        entry("broadcast_binary", f"analog: bf16 x [{B}, {Cc}, {H}, {W}] NCHW, y [{B}, {Cc}], bias [{Cc}]",
              2 * n * 2 + (B * Cc + Cc) * 2,
              lambda: (rnd(B, Cc, H, W), torch.empty((B, Cc, H, W), dtype=torch.bfloat16, device=dev)),
              lambda x, z: hc.broadcast_binary(x, y_, bias, B, z=z))
    if "activation_gelu_silu" in want:
        entry("activation_gelu_silu", f"analog: bf16 [{R}, {K}], tanh-GELU", 2 * n * 2,
              lambda: (rnd(R, K), torch.empty((R, K), dtype=torch.bfloat16, device=dev)),
              lambda x, y: hc.activation_gelu_silu(x, "gelu", y=y))
    if "reduce_sum_lastdim" in want:
        entry("reduce_sum_lastdim", f"analog: bf16 [{R}, {K}] -> fp32 [{R}]", n * 2 + R * 4,
              lambda: (rnd(R, K), torch.empty((R,), dtype=torch.float32, device=dev)),
              lambda x, o: hc.reduce_sum_lastdim(x, out=o))
    if "transpose_2d_4d" in want:
        M = N = 8192
        entry("transpose_2d_4d", f"analog: bf16 [{M}, {N}] -> [{N}, {M}]", 2 * M * N * 2,
              lambda: (rnd(M, N), torch.empty((N, M), dtype=torch.bfloat16, device=dev)),
              lambda x, o: hc.transpose_2d_4d(x, 0, out=o))
    return out


def run_only(args):
    """One non-headline configuration alone (used for per-kernel profiling captures)."""
    import torch

    d = Dist(args.gpus)
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    import hc

    hc.load()
    peaks, _ = load_peaks()
    out = run_extras(hc, d, dev, peaks, args, want=(args.only,))
    hc.check_device_error()
    if d.rank == 0:
        print(json.dumps({"only": args.only, **out[args.only]}), flush=True)
    d.close()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip the non-headline configurations")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--gather-outputs", action="store_true",
                    help="with N > 1: all-gather every rank's attention output after the timed region and report it")
    ap.add_argument("--fa-batch", type=int, default=FA_B,
                    help="attention batch per GPU (default 16, the benchmarked size; smaller only for profiling captures)")
    ap.add_argument("--only", choices=EXTRA_OPS, default=None,
                    help="time one non-headline configuration alone and print its entry (profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3  # timing rule: at least 3 untimed warm-up steps
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.only:
        run_only(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
