"""Benchmark of the B200 operator ladder (headline: causal flash-attention forward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extras]

One step = one flash_attention_fwd_fused forward over the benchmarked configuration:
Q, K, V bf16 [B=16, H=32, S=8192, D=128], causal, scale 1/sqrt(128), O bf16 + lse fp32.
Strong scaling: the 16 x 32 = 512 (batch, head) pairs of the one fixed problem are split over the
N ranks (one process per GPU, torchrun), 512/N heads each; the work shards over batch x heads with
no exchange, so there is no collective on the data path.  Time is measured with CUDA events on the
launching stream between barriers, max over ranks; `value` is the whole problem's FLOPs divided by
that time.  Rank 0 prints one JSON line.  Inputs (3.2 GB at N=1) are larger than the 126 MB L2.

Extra keys of the JSON line:
  roofline     the flash-attention kernel against the measured dense bf16 peak
  accuracy     the headline output of the timed launches checked after timing: sampled heads of
               every rank against a torch fp32 reference on the device (max-abs / max-rel)
  e2e          the same metric through the C ABI's host-buffer entry point
               (hc_flash_attention_fwd_fused_host: pinned H2D copies, kernel, D2H copies, per step)
  cpu_baseline the reference golden (compiled from the reference sources into oracle/_ref) on the
               host cores, on a bounded sample (rank 0, N=1 only)
  weak         (N > 1) every rank running the full 512-head problem: the per-GPU-constant figure
  ops          the other benchmarked configurations, each split over the ranks like the headline,
               as {value, unit, frac, ms, max_abs, max_rel, pass}; the accuracy columns come from
               a sampled check of that op's output in the same run (torch fp32 reference on the
               device; bit-exact ops compare bits)
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

import specs  # noqa: E402  (per-operator B200 contracts: benchmark configurations and tolerances)

_FA = specs.bench_config("flash_attention_fwd_fused")
FA_B, FA_H, FA_S, FA_D = _FA["B"], _FA["H"], _FA["S_q"], _FA["D"]
FA_TOL = specs.tolerance("flash_attention_fwd_fused", "bfloat16")
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


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Strong scaling: rank `rank`'s contiguous share (start, count) of `total` independent units
    (attention heads, matrix rows, sequence positions, elements).  Shares differ by at most one
    unit and together cover every unit exactly once."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def fixed_job_rate(total_units: float, ms_max: float) -> float:
    """Strong scaling: the one fixed problem's units divided by the slowest rank's time."""
    return total_units / (ms_max * 1e-3)


def rel_err(expected, actual):
    """Element-wise relative error as the harness's accuracy::CompareArrays defines it
    (include/harness/accuracy.hpp:78-83): |e - a| / |e|, or / |a| when |e| <= 1e-12."""
    import torch

    e, a = expected.double(), actual.double()
    d = (e - a).abs()
    den = torch.where(e.abs() > 1e-12, e.abs(), a.abs())
    return torch.where(den > 1e-12, d / den.clamp_min(1e-300), torch.zeros_like(d))


def accuracy(expected, actual, abs_tol: float, rel_tol: float) -> dict:
    """Max-abs and max-rel error over all compared elements, and the CompareArrays verdict: an element
    fails only when it exceeds both tolerances."""
    d = (expected.double() - actual.double()).abs()
    r = rel_err(expected, actual)
    fails = int(((d > abs_tol) & (r > rel_tol)).sum().item())
    return {"max_abs": float(d.max().item()) if d.numel() else 0.0,
            "max_rel": float(r.max().item()) if r.numel() else 0.0, "pass": fails == 0}


def sig(x, n: int = 4):
    """Rounds floats to `n` significant digits (keeps the JSON line short)."""
    if isinstance(x, float) and math.isfinite(x) and x != 0.0:
        return round(x, n - 1 - int(math.floor(math.log10(abs(x)))))
    if isinstance(x, dict):
        return {k: sig(v, n) for k, v in x.items()}
    return x


# ------------------------------------------------------------------------------------------------
# timing helpers
# ------------------------------------------------------------------------------------------------
def time_launches(fn, steps: int, warmup: int, d: Dist, flush=None, spin: bool = True, local: bool = False):
    """Returns ms per launch averaged over `steps`: the max over ranks, or this rank's own figure
    with `local` (the barriers are the same either way).

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
    return ms if local else d.max(ms)


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
# torch fp32/fp64 references for the in-run accuracy checks (device-side; the oracle is not used)
# ------------------------------------------------------------------------------------------------
def fa_reference(q, k, v, causal: bool, scale: float):
    """O and lse of one head ([S, D] tensors) in float64 on the device: softmax(q k^T * scale) v."""
    import torch

    qd, kd, vd = q.double(), k.double(), v.double()
    s = (qd @ kd.transpose(0, 1)) * scale
    if causal:
        s = s.masked_fill(torch.ones_like(s, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ vd
    return o, lse


def check_fa_heads(q, k, v, o, lse, causal: bool, n_sample: int = 4) -> dict:
    """Sampled heads of this rank's shard ([1, h, S, D]) against fa_reference, with the spec's bf16
    tolerances (O max-abs 2e-2, lse 2e-3)."""
    import torch

    h = q.shape[1]
    heads = sorted({0, h - 1, *[int(i) for i in torch.linspace(0, h - 1, n_sample).round().tolist()]})
    scale = 1.0 / math.sqrt(q.shape[-1])
    worst = {"max_abs": 0.0, "max_rel": 0.0, "pass": True, "lse_max_abs": 0.0}
    for i in heads:
        o_ref, l_ref = fa_reference(q[0, i], k[0, i], v[0, i], causal, scale)
        acc = accuracy(o_ref, o[0, i], FA_TOL["abs"], FA_TOL["rel"])
        lerr = float((l_ref - lse[0, i].double()).abs().max().item())
        worst["max_abs"] = max(worst["max_abs"], acc["max_abs"])
        worst["max_rel"] = max(worst["max_rel"], acc["max_rel"])
        worst["lse_max_abs"] = max(worst["lse_max_abs"], lerr)
        worst["pass"] = worst["pass"] and acc["pass"] and lerr <= FA_TOL["lse_abs"]
    worst["heads_checked"] = len(heads)
    return worst


# Algorithmic FLOPs of the backward per visible (query, key) pair, as a multiple of the forward's
# 4*D: five products of 2*D each (S recomputed, dP, dV, dK, dQ).  The tensor-core kernels issue
# seven (S and dP are formed once for dQ and once for dK/dV); only the five count.
FA_BWD_FLOP_RATIO = 2.5
FA_BWD_TOL = 1e-2  # normwise ||got - exact|| / ||exact|| per gradient, bf16


def check_fa_bwd_heads(q, k, v, dout, grads, causal: bool, n_sample: int = 2) -> dict:
    """Sampled heads of the backward against fp32 gradients on the device (no TF32): dq, dk, dv
    each within FA_BWD_TOL normwise; max_abs/max_rel report the worst element."""
    import torch

    h = q.shape[1]
    heads = sorted({0, h - 1, *[int(i) for i in torch.linspace(0, h - 1, n_sample).round().tolist()]})
    scale = 1.0 / math.sqrt(q.shape[-1])
    worst = {"max_abs": 0.0, "max_rel": 0.0, "pass": True, "normwise": 0.0}
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for i in heads:
            qf, kf, vf, df = (t[0, i].float() for t in (q, k, v, dout))
            s = (qf @ kf.T) * scale
            if causal:
                s = s.masked_fill(torch.ones_like(s, dtype=torch.bool).triu(1), float("-inf"))
            p = torch.softmax(s, dim=-1)
            dp = df @ vf.T
            ds = p * (dp - (p * dp).sum(-1, keepdim=True))
            for ref, got in (((ds @ kf) * scale, grads[0][0, i]), ((ds.T @ qf) * scale, grads[1][0, i]),
                             (p.T @ df, grads[2][0, i])):
                acc = accuracy(ref, got, 0.0, 0.0)
                nw = float((got.double() - ref.double()).norm() / ref.double().norm())
                worst["max_abs"] = max(worst["max_abs"], acc["max_abs"])
                worst["max_rel"] = max(worst["max_rel"], acc["max_rel"])
                worst["normwise"] = max(worst["normwise"], nw)
                worst["pass"] &= nw <= FA_BWD_TOL
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return worst


def merge_acc(d: "Dist", acc: dict) -> dict:
    """Worst accuracy over the ranks (max of the errors, AND of the verdicts)."""
    out = dict(acc)
    for key in ("max_abs", "max_rel", "lse_max_abs", "normwise"):
        if key in acc:
            out[key] = d.max(acc[key])
    out["pass"] = d.max(0.0 if acc["pass"] else 1.0) == 0.0
    return out


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
def fa_inputs(dev, heads: int, seed_base: int):
    """Q, K, V bf16 [1, heads, S, D] ~ N(0,1) from torch's seeded CUDA generator."""
    import torch

    gens = [torch.Generator(device=dev).manual_seed(s + seed_base) for s in (0, 1, 2)]
    return [torch.randn((1, heads, FA_S, FA_D), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
            for g in gens]


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
    total_heads = args.fa_batch * FA_H
    h0, hn = shard_range(total_heads, n, d.rank)

    # ---------------- headline: causal flash attention, the fixed problem split over the ranks -------
    q, k, v = fa_inputs(dev, hn, 3 * d.rank)
    o = torch.empty_like(q)
    lse = torch.empty((1, hn, FA_S), dtype=torch.float32, device=dev)
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
    flops_total = fa_flops(1, total_heads, FA_S, FA_S, FA_D, True)
    flops_rank = fa_flops(1, hn, FA_S, FA_S, FA_D, True)
    value = fixed_job_rate(flops_total, ms) / 1e12
    achieved = flops_rank / (ms_local * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "peak_source": f"{peak_src} bf16_tflops (burst)",
                "traffic": profile_traffic("flash_attention_fwd_causal"),
                "algorithmic_flops_per_launch": flops_rank}
    acc = merge_acc(d, check_fa_heads(q, k, v, o, lse, True))

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
        gather = {"bytes_per_rank": o.numel() * 2, "ms": g_ms,
                  "gb_per_s_in_per_rank": (n - 1) * o.numel() * 2 / (g_ms * 1e-3) / 1e9, "own_slices_equal": own_ok == 1.0}
        del full
    del o

    # ---------------- e2e through the host-buffer C entry point -----------------------------------
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        ho = torch.empty_like(hq).pin_memory()
        hl = torch.empty((1, hn, FA_S), dtype=torch.float32).pin_memory()
        t = hc.FlashAttentionFwdFusedTiling(1, hn, FA_S, FA_S, FA_D, FA_D, 1.0 / math.sqrt(FA_D), 1)
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
        h2d = 3 * total_heads * FA_S * FA_D * 2
        d2h = total_heads * FA_S * (FA_D * 2 + 4)
        e2e = {"value": fixed_job_rate(flops_total, e2e_ms) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "hc_flash_attention_fwd_fused_host (pinned host buffers; bytes summed over ranks)"}
        del hq, hk, hv, ho, hl, work
    del q, k, v, lse
    torch.cuda.empty_cache()

    # ---------------- weak scaling (N > 1): every rank runs the whole 512-head problem ---------------
    weak = None
    if n > 1 and not args.no_weak:
        q, k, v = fa_inputs(dev, total_heads, 3 * d.rank)
        o = torch.empty_like(q)
        lse = torch.empty((1, total_heads, FA_S), dtype=torch.float32, device=dev)
        w_ms = time_launches(lambda: hc.flash_attention_fwd(q, k, v, True, out=o, lse=lse), max(3, args.steps // 4),
                             args.warmup, d)
        weak = {"value": whole_job_rate(flops_total, n, w_ms) / 1e12, "unit": "TFLOP/s", "ms_per_step": w_ms,
                "per_gpu_heads": total_heads}
        del q, k, v, o, lse
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
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: Q,K,V ~ N(0,1), torch CUDA generator seeds 0/1/2 (+3 per rank), bf16",
            "config": {"workload": f"flash_attention_fwd_fused causal bf16 B{args.fa_batch} H{FA_H} S{FA_S} D{FA_D}, "
                                   f"O bf16 + lse fp32; {total_heads} heads split over {n} GPU(s)",
                       "global_batch": args.fa_batch, "seq_len": FA_S, "heads": FA_H, "head_dim": FA_D,
                       "causal": True, "parallelism": f"dp{n}: batch x heads sharded, no collective",
                       "l2": "inputs > 126 MB L2 per GPU; no flush"},
            "gpu_launches": args.steps,
            "roofline": sig(roofline), "accuracy": sig(acc), "e2e": sig(e2e), "cpu_baseline": sig(cpu),
            "clocks": clocks,
            **({"weak": sig(weak)} if weak else {}),
            **({"gather": sig(gather)} if gather else {}),
            "ops": {k_: sig(v_) for k_, v_ in ops.items()},
        }
        print(json.dumps(line, separators=(",", ":")), flush=True)
    d.close()


EXTRA_OPS = ("flash_attention_fwd_noncausal", "flash_attention_bwd", "matmul_bias", "layer_norm", "rms_norm_rope_fused", "elementwise_add",
             "axpy_scalar_affine", "broadcast_binary", "activation_gelu_silu", "reduce_sum_lastdim", "transpose_2d_4d")
# The last five ops have no configuration of their own in the reference's benchmark list; they are
# timed on sized analogs of the layer_norm shape (134 MB of 16-bit input per launch); the shapes
# are listed in the design notes.
ANALOG_OPS = EXTRA_OPS[6:]


def settle():
    """Each configuration after the headline starts from an idle GPU: after the 8192^3 GEMM's power
    burst the power controller holds the clock down for about a second, and the next kernel
    (layer_norm here) measured up to 10 points low when timed at once."""
    import torch

    torch.cuda.synchronize()
    time.sleep(1.0)


def run_extras(hc, d: Dist, dev, peaks, args, want=EXTRA_OPS) -> dict:
    """The other benchmarked configurations, each split over the ranks like the headline and timed
    alone (W=3, 20 launches; 5 for attention).  Each entry: whole-job rate (total work / slowest
    rank's time), the kernel's roofline fraction on its shard, and the accuracy of that output
    against a device-side torch reference (sampled where the full check would dominate the run)."""
    import torch

    out = {}
    if not want:
        return out
    steps, warm = 20, 3
    n, r = d.world, d.rank
    # The bandwidth workloads below run back to back without an L2 flush; consecutive launches cycle
    # through independent buffer sets whose total exceeds twice the 126 MB L2 (two sets at N=1, where
    # each launch alone reads more than L2; more at N=8, where a 17-67 MB shard would fit), so a
    # launch can neither re-read a recent launch's inputs nor rewrite its still-dirty outputs in L2.
    hbm = peaks["hbm_gbs"]
    flip = [0]

    def alternate(sets):
        """Cycles through the buffer sets; flip[0] is the index of the set used last."""
        def nxt():
            flip[0] = (flip[0] + 1) % len(sets)
            return sets[flip[0]]
        return nxt

    def rotation(make_set, set_bytes):
        """Enough independent buffer sets that one cycle moves more than twice the 126 MB L2 (two at
        least): at N = 8 a single shard fits in L2, and back-to-back launches would otherwise re-read it."""
        count = max(2, min(32, math.ceil(2.2 * 126e6 / max(set_bytes, 1))))
        return [make_set() for _ in range(count)]
    g = torch.Generator(device=dev).manual_seed(100 + r)

    def entry(name, total_units, rank_units, unit_bytes_or_flops, ms_local, acc, bound):
        ms = d.max(ms_local)
        per = rank_units * unit_bytes_or_flops / (ms_local * 1e-3)
        acc = merge_acc(d, acc)
        if bound == "hbm":
            job = total_units * unit_bytes_or_flops / (ms * 1e-3) / 1e9
            e = {"value": job, "unit": "GB/s", "frac": per / 1e9 / hbm}
        else:
            job = total_units * unit_bytes_or_flops / (ms * 1e-3) / 1e12
            e = {"value": job, "unit": "TFLOP/s", "frac": per / 1e12 / peaks["bf16_tflops"]}
        e.update({"ms": ms, "max_abs": acc["max_abs"], "max_rel": acc["max_rel"], "pass": acc["pass"]})
        if "normwise" in acc:
            e["normwise"] = acc["normwise"]
        out[name] = e

    if "flash_attention_fwd_noncausal" in want:  # same shapes as the headline, no mask
        total = args.fa_batch * FA_H
        _, hn = shard_range(total, n, r)
        q, k, v = fa_inputs(dev, hn, 50 + 3 * r)
        o = torch.empty_like(q)
        lse = torch.empty((1, hn, FA_S), dtype=torch.float32, device=dev)
        settle()
        ms = time_launches(lambda: hc.flash_attention_fwd(q, k, v, False, out=o, lse=lse), 5, warm, d, local=True)
        acc = check_fa_heads(q, k, v, o, lse, False, n_sample=2)
        entry("flash_attention_fwd_noncausal", total, hn, fa_flops(1, 1, FA_S, FA_S, FA_D, False), ms, acc, "tensor")
        del q, k, v, o, lse

    if "flash_attention_bwd" in want:  # backward of the headline (same shapes, causal)
        total = args.fa_batch * FA_H
        _, hn = shard_range(total, n, r)
        q, k, v = fa_inputs(dev, hn, 70 + 3 * r)
        dout = fa_inputs(dev, hn, 80 + 3 * r)[0]
        o, lse = hc.flash_attention_fwd(q, k, v, True)
        grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(lse))
        settle()
        ms = time_launches(lambda: hc.flash_attention_bwd(q, k, v, o, lse, dout, True, out=grads), 5, warm, d,
                           local=True)
        acc = check_fa_bwd_heads(q, k, v, dout, grads, True)
        entry("flash_attention_bwd", total, hn, FA_BWD_FLOP_RATIO * fa_flops(1, 1, FA_S, FA_S, FA_D, True), ms, acc,
              "tensor")
        del q, k, v, dout, o, lse, grads

    if "matmul_bias" in want:  # 8192^3 bf16, M rows split over the ranks, B replicated
        cfg = specs.bench_config("matmul_bias")
        M, K, N = cfg["M"], cfg["K"], cfg["N"]
        _, mn = shard_range(M, n, r)
        A = (torch.randn((mn, K), generator=g, device=dev) / math.sqrt(K)).to(torch.bfloat16)
        B = (torch.randn((K, N), generator=g, device=dev) / math.sqrt(K)).to(torch.bfloat16)
        bias = (torch.randn((N,), generator=g, device=dev) * 0.1).to(torch.bfloat16)
        C = torch.empty((mn, N), dtype=torch.bfloat16, device=dev)
        settle()
        ms = time_launches(lambda: hc.matmul_bias(A, B, bias, out=C), steps, warm, d, local=True)
        rows = torch.unique(torch.cat([torch.tensor([0, mn - 1]), torch.randint(0, mn, (62,))])).to(dev)
        ref = A[rows].double() @ B.double() + bias.double()
        acc = accuracy(ref, C[rows], 0.0, 0.0)
        acc["pass"] = float((ref - C[rows].double()).abs().max() / ref.abs().max()) <= \
            specs.tolerance("matmul_bias", "bfloat16")["normwise_rel"]
        entry("matmul_bias", M, mn, 2.0 * N * K, ms, acc, "tensor")
        del A, B, bias, C, ref

    if "layer_norm" in want:  # [16384, 4096] bf16, fp32 gamma/beta, rows split over the ranks
        cfg = specs.bench_config("layer_norm")
        R, H, eps = cfg["rows"], cfg["lastDim"], cfg["eps"]
        _, rn = shard_range(R, n, r)
        gamma = torch.rand((H,), generator=g, device=dev) + 0.5
        beta = torch.rand((H,), generator=g, device=dev) * 0.2 - 0.1
        def ln_set():
            x = torch.randn((rn, H), generator=g, device=dev).to(torch.bfloat16)
            return x, torch.empty_like(x)
        sets = rotation(ln_set, 2 * rn * H * 2)
        nxt = alternate(sets)

        def ln_step():
            xx, yy = nxt()
            hc.layer_norm(xx, gamma, beta, eps, y=yy)

        settle()
        ms = time_launches(ln_step, steps, warm, d, local=True)
        x, y = sets[flip[0]]
        rows = torch.linspace(0, rn - 1, 64, device=dev).long()
        xd = x[rows].double()
        mean = xd.mean(-1, keepdim=True)
        var = ((xd - mean) ** 2).mean(-1, keepdim=True)
        ref = (xd - mean) / torch.sqrt(var + eps) * gamma.double() + beta.double()
        tol = specs.tolerance("layer_norm", "bfloat16")
        acc = accuracy(ref, y[rows], tol["abs"], tol["rel"])
        entry("layer_norm", R, rn, 2 * H * 2 + 2 * H * 4 / rn, ms, acc, "hbm")
        del x, y, sets

    if "rms_norm_rope_fused" in want:  # [8, 4096, 32, 128] bf16, rotate-half, positions split over the ranks
        cfg = specs.bench_config("rms_norm_rope_fused")
        Bb, S, Hh, D, eps, theta = cfg["B"], cfg["S"], cfg["heads"], cfg["H"], cfg["eps"], cfg["theta"]
        s0, sn = shard_range(S, n, r)
        w = torch.rand((D,), generator=g, device=dev) + 0.5
        pos = torch.arange(S, device=dev, dtype=torch.float32)[:, None]
        inv = 1.0 / (theta ** (torch.arange(D // 2, device=dev, dtype=torch.float32) * 2 / D))
        cos_all, sin_all = torch.cos(pos * inv), torch.sin(pos * inv)
        cos, sin = cos_all[s0:s0 + sn].contiguous(), sin_all[s0:s0 + sn].contiguous()
        def rms_set():
            x = torch.randn((Bb, sn, Hh, D), generator=g, device=dev).to(torch.bfloat16)
            return x, torch.empty_like(x)
        sets = rotation(rms_set, 2 * Bb * sn * Hh * D * 2)
        nxt = alternate(sets)

        def rms_step():
            xx, yy = nxt()
            hc.rms_norm_rope_fused(xx, w, cos, sin, D, eps, heads=Hh, rope_style=cfg["rope_style"], out=yy)

        settle()
        ms = time_launches(rms_step, steps, warm, d, local=True)
        x, y = sets[flip[0]]
        xs = x[:, :: max(1, sn // 16)].double()  # 16 positions of every batch, all heads
        ys = y[:, :: max(1, sn // 16)]
        cs, ss = cos[:: max(1, sn // 16)].double()[None, :, None], sin[:: max(1, sn // 16)].double()[None, :, None]
        xn = xs / torch.sqrt((xs * xs).mean(-1, keepdim=True) + eps) * w.double()
        lo, hi = xn[..., : D // 2], xn[..., D // 2:]
        ref = torch.cat([lo * cs - hi * ss, hi * cs + lo * ss], dim=-1)
        tol = specs.tolerance("rms_norm_rope_fused", "bfloat16")
        acc = accuracy(ref, ys, tol["abs"], tol["rel"])
        # per (position, head) row: x in and out, plus its share of the position's cos/sin row
        entry("rms_norm_rope_fused", Bb * S * Hh, Bb * sn * Hh, 2 * D * 2 + 2 * (D // 2) * 4 / (Bb * Hh), ms, acc, "hbm")
        del x, y, sets

    if "elementwise_add" in want:  # fp16 [4096, 8192], U[-1, 1], flat range split over the ranks
        total = math.prod(specs.bench_config("elementwise_add")["shape"])
        _, en = shard_range(total, n, r)
        def add_set():
            a = (torch.rand((en,), generator=g, device=dev) * 2 - 1).to(torch.float16)
            b = (torch.rand((en,), generator=g, device=dev) * 2 - 1).to(torch.float16)
            return a, b, torch.empty_like(a)
        sets = rotation(add_set, 3 * en * 2)
        nxt = alternate(sets)
        settle()
        ms = time_launches(lambda: hc.elementwise_add(*nxt()), steps, warm, d, local=True)
        a, b, z = sets[flip[0]]
        ref = a + b  # torch's fp16 add: fp32 sum, one round-to-nearest-even (the golden's arithmetic)
        acc = accuracy(ref, z, 0.0, 0.0)
        acc["pass"] = bool(torch.equal(ref.view(torch.int16), z.view(torch.int16)))  # bit-exact
        entry("elementwise_add", total, en, 3 * 2, ms, acc, "hbm")
        del a, b, z, sets
    if any(op in want for op in ANALOG_OPS):
        run_analogs(hc, d, dev, want, steps, warm, alternate, rotation, entry, flip)
    torch.cuda.empty_cache()
    return out


def run_analogs(hc, d: Dist, dev, want, steps, warm, alternate, rotation, entry, flip) -> None:
    """Sized analogs for the ops without a configuration of their own: bf16, 134 MB of input at
    N=1 (the layer_norm shape), rows split over the ranks."""
    import torch

    g = torch.Generator(device=dev).manual_seed(7 + d.rank)
    cfg = specs.bench_config("axpy_scalar_affine")
    R, K = cfg["rows"], cfg["lastDim"]  # the layer_norm shape
    _, rn = shard_range(R, d.world, d.rank)

    def rnd(*shape):
        return torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)

    def timed(make_set, run, set_bytes):
        sets = rotation(make_set, set_bytes)
        nxt = alternate(sets)
        settle()
        ms = time_launches(lambda: run(*nxt()), steps, warm, d, local=True)
        return ms, sets[flip[0]]

    def exact(ref, got):
        acc = accuracy(ref.float(), got.float(), 0.0, 0.0)
        acc["pass"] = bool(torch.equal(ref.view(torch.int16), got.view(torch.int16)))
        return acc

    if "axpy_scalar_affine" in want:  # y = 0.5 x - 1 in fp32, one rounding to bf16 (bit-exact)
        ms, (x, y) = timed(lambda: (rnd(rn, K), torch.empty((rn, K), dtype=torch.bfloat16, device=dev)),
                           lambda x, y: hc.axpy_scalar_affine(x, cfg["alpha"], cfg["beta"], y=y), 2 * rn * K * 2)
        ref = (x.float() * cfg["alpha"] + cfg["beta"]).to(torch.bfloat16)
        entry("axpy_scalar_affine", R, rn, 2 * K * 2, ms, exact(ref, y), "hbm")
    if "broadcast_binary" in want:  # x [16, 256, 128, 128] NCHW split over the batch; y [16, 256], bias [256]
        bc = specs.bench_config("broadcast_binary")
        B, Cc, H, W = bc["B"], bc["C"], bc["H"], bc["W"]
        b0, bn = shard_range(B, d.world, d.rank)
        y_ = rnd(bn, Cc)
        bias = rnd(Cc)
        ms, (x, z) = timed(lambda: (rnd(bn, Cc, H, W), torch.empty((bn, Cc, H, W), dtype=torch.bfloat16, device=dev)),
                           lambda x, z: hc.broadcast_binary(x, y_, bias, bn, z=z), 2 * bn * Cc * H * W * 2)
        ref = (x.float() * y_.float()[:, :, None, None] + bias.float()[None, :, None, None]).to(torch.bfloat16)
        entry("broadcast_binary", B, bn, Cc * H * W * 2 * 2, ms, exact(ref, z), "hbm")
    if "activation_gelu_silu" in want:  # tanh-GELU
        ms, (x, y) = timed(lambda: (rnd(rn, K), torch.empty((rn, K), dtype=torch.bfloat16, device=dev)),
                           lambda x, y: hc.activation_gelu_silu(x, "gelu", y=y), 2 * rn * K * 2)
        xd = x[:: max(1, rn // 64)].double()
        ref = 0.5 * xd * (1.0 + torch.tanh(0.7978845608028654 * (xd + 0.044715 * xd ** 3)))
        tol = specs.tolerance("activation_gelu_silu", "bfloat16")
        entry("activation_gelu_silu", R, rn, 2 * K * 2, ms, accuracy(ref, y[:: max(1, rn // 64)], tol["abs"], tol["rel"]),
              "hbm")
    if "reduce_sum_lastdim" in want:  # bf16 rows -> fp32 sums
        ms, (x, o) = timed(lambda: (rnd(rn, K), torch.empty((rn,), dtype=torch.float32, device=dev)),
                           lambda x, o: hc.reduce_sum_lastdim(x, out=o), rn * K * 2)
        tol = specs.tolerance("reduce_sum_lastdim", "bfloat16")
        entry("reduce_sum_lastdim", R, rn, K * 2 + 4, ms, accuracy(x.double().sum(-1), o, tol["abs"], tol["rel"]), "hbm")
    if "transpose_2d_4d" in want:  # [8192, 8192] bf16 -> [8192, 8192], row blocks split over the ranks
        tc = specs.bench_config("transpose_2d_4d")
        M, N = tc["M"], tc["N"]
        _, mn = shard_range(M, d.world, d.rank)
        ms, (x, o) = timed(lambda: (rnd(mn, N), torch.empty((N, mn), dtype=torch.bfloat16, device=dev)),
                           lambda x, o: hc.transpose_2d_4d(x, 0, out=o), 2 * mn * N * 2)
        entry("transpose_2d_4d", M, mn, N * 2 * 2, ms, exact(x.t().contiguous(), o), "hbm")


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
        print(json.dumps({"only": args.only, **sig(out[args.only])}), flush=True)
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
    ap.add_argument("--no-weak", action="store_true", help="with N > 1: skip the weak-scaling (full problem per GPU) figure")
    ap.add_argument("--gather-outputs", action="store_true",
                    help="with N > 1: all-gather every rank's attention output after the timed region and report it")
    ap.add_argument("--fa-batch", type=int, default=FA_B,
                    help="attention batch of the whole problem (default 16, the benchmarked size; smaller only for "
                         "profiling captures)")
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
