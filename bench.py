#!/usr/bin/env python
"""FlexAttention B200 benchmark: effective TFLOP/s of one forward+backward step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl flexattn|reference]

A step is one forward and one backward pass (``flash_attention`` + autograd
backward) of the chosen configuration (default cfg2: causal bf16
B4 H16 S4096 D128) on inputs already resident in HBM.  Effective FLOPs count
only unmasked (q, kv) pairs: forward 4*D*pairs*B*H, backward 2.5x that.

Multi-GPU (torchrun): the one problem of the config is split by heads over the
ranks (strong scaling; heads are independent, so no collective runs on the data
path); the time is the max over ranks and ``value`` counts the whole problem.
Each timed step is bracketed by its own CUDA events, after an L2 flush.

Extra keys: ``roofline`` for the dominant pass (algorithmic FLOPs per call over
its CUDA-event duration, against the measured bf16 peak), ``cpu_baseline`` (the
reference's tiled CPU path restated in torch, on one (b, h) slice), ``e2e`` (the
same step through the public API with pinned-host inputs copied in and dq, dk,
dv copied out every step), ``parity`` (four heads of the timed inputs, every
element of o/dq/dk/dv against fp32), ``per_config`` (forward and backward of
every other benchmark configuration at its full size, with parity), ``clocks``
(NVML sampled every 10 ms during the timed region) and ``gpu_launches``.

``--impl reference`` times the reference's CPU implementation of the path (the
restatement in oracle/cpu_reference.py; the reference itself needs jax, which
is not installed) on this box's host cores, on rank 0 only.

``--workload decode [--decode-config gqa_b64]`` prints a separate line for the
split-KV decode path (K/V cache bytes read per second against the measured HBM
bandwidth); the default workload is the forward+backward step above.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path
from typing import Optional

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "pallas-flexattn_b200"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

PEAK_FALLBACK = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


def load_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    d = dict(PEAK_FALLBACK)
    d["source"] = "fallback"
    return d


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled while the timed region runs.

    Reads NVML (nvidia_ml_py) every 10 ms from a thread, so even a sub-second timed region
    gets samples; falls back to `nvidia-smi -lms 100` when NVML cannot be opened.  Only
    reads state: it never changes a clock or any other GPU setting.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.sm: list[float] = []
        self.max_mhz = None
        self.reasons: set = set()
        self.lines: list[str] = []
        self.proc = None
        self.thread = None
        self.stop = threading.Event()
        self.nvml = None

    def _nvml_handle(self):
        import pynvml as N
        N.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        try:
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            return N, N.nvmlDeviceGetHandleByPciBusId_v2(bus)
        except Exception:
            return N, N.nvmlDeviceGetHandleByUUID("GPU-" + str(props.uuid))

    def _poll_nvml(self, N, h):
        bits = {"hw_slowdown": N.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": N.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": N.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": N.nvmlClocksEventReasonSwPowerCap}
        while not self.stop.is_set():
            try:
                self.sm.append(float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)))
                r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.reasons.update(n for n, b in bits.items() if r & b)
            except Exception:
                pass
            self.stop.wait(0.01)

    def __enter__(self):
        try:
            N, h = self._nvml_handle()
            self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM))
            self.nvml = N
            self.thread = threading.Thread(target=self._poll_nvml, args=(N, h), daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id=GPU-{torch.cuda.get_device_properties(self.device).uuid}",
                 f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read_smi, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read_smi(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        for ln in self.lines:  # nvidia-smi fallback
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                self.sm.append(float(parts[1]))
                self.max_mhz = float(parts[2])
            except ValueError:
                continue
            self.reasons.update(n for n, flag in zip(self.NAMES, parts[5:9]) if flag.lower() == "active")

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.sm),
                "source": "nvml" if self.nvml else "nvidia-smi"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        return dist, dist.get_rank(), world, local
    return None, 0, 1, 0


def barrier(dist):
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, x: float, device) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def score_value_grad(score_mod, raw, hi, qi, ki):
    """The registry score_mod on raw scaled logits, with d(score)/d(raw), from its spec."""
    from pallas_flexattn import _lib as L
    from pallas_flexattn.score_mod import spec_of

    spec = spec_of(score_mod)
    x, g = raw, torch.ones_like(raw)
    if spec is None or spec.flags == 0:
        return x, g
    if spec.flags & L.FA_SCORE_ALIBI:
        x = x + spec.alibi_slopes.to(raw.device)[hi] * (ki - qi)
    if spec.flags & L.FA_SCORE_REL_BIAS:
        t = spec.rel_bias.to(raw.device)
        x = x + t[hi if t.shape[0] > 1 else hi * 0, qi - ki + raw.shape[-1] - 1]
    if spec.flags & L.FA_SCORE_SOFTCAP:
        t = torch.tanh(x / spec.softcap)
        x, g = spec.softcap * t, g * (1 - t * t)
    return x, g


def reference_fwd_bwd(q, k, v, do, mask_mod, score_mod, chunk=512):
    """fp32 reference o, dq, dk, dv (the materialised formulas, in row chunks on the GPU)."""
    B, H, T, D = q.shape
    s = 1.0 / math.sqrt(D)
    qf, kf, vf, dof = (t.float() for t in (q, k, v, do))
    dev = q.device
    kvi = torch.arange(k.shape[2], device=dev)[None, :]
    hi = torch.arange(H, device=dev)[None, :, None, None]
    ninf = torch.tensor(-math.inf, device=dev)

    def scores(r0, r1):
        qi = torch.arange(r0, r1, device=dev)[:, None]
        x, g = score_value_grad(score_mod, torch.einsum("bhqd,bhkd->bhqk", qf[:, :, r0:r1], kf) * s, hi, qi, kvi)
        if mask_mod is not None:
            x = torch.where(mask_mod(qi, kvi), x, ninf)
        return x, g

    o = torch.empty_like(qf)
    lse = torch.empty(q.shape[:3], device=dev)
    for r0 in range(0, T, chunk):
        x, _ = scores(r0, min(r0 + chunk, T))
        lse[:, :, r0:r0 + chunk] = torch.logsumexp(x, -1)
        o[:, :, r0:r0 + chunk] = torch.exp(x - lse[:, :, r0:r0 + chunk, None]).nan_to_num(0.0) @ vf
    delta = (o * dof).sum(-1)
    dq, dk, dv = torch.zeros_like(qf), torch.zeros_like(kf), torch.zeros_like(vf)
    for r0 in range(0, T, chunk):
        r1 = min(r0 + chunk, T)
        x, g = scores(r0, r1)
        p = torch.exp(x - lse[:, :, r0:r1, None]).nan_to_num(0.0)
        ds = p * (dof[:, :, r0:r1] @ vf.transpose(-1, -2) - delta[:, :, r0:r1, None]) * g
        dv += p.transpose(-1, -2) @ dof[:, :, r0:r1]
        dk += ds.transpose(-1, -2) @ qf[:, :, r0:r1] * s
        dq[:, :, r0:r1] = ds @ kf * s
    return o, dq, dk, dv


PARITY_RULE = ("per element |err| <= 2e-2 + u, u = half an ulp of the output dtype at |ref| (the rounding of "
               "the result to bf16; 0 for fp32), and rel-L2 <= 5e-3, against fp32 on the same inputs")


def parity_stats(got: torch.Tensor, ref: torch.Tensor, bf16: bool) -> dict:
    got, ref = got.detach().float(), torch.nan_to_num(ref.detach().float())
    d = (got - ref).abs()
    if bf16:
        _, e = torch.frexp(ref.abs())
        u = torch.where(ref != 0, torch.ldexp(torch.ones_like(ref), e - 9), torch.zeros_like(ref))
    else:
        u = torch.zeros_like(ref)
    rel = float((got - ref).norm() / ref.norm().clamp_min(1e-30))
    max_abs = float(d.max())
    excess = float((d - 2e-2 - u).max())
    return {"max_abs": round(max_abs, 6), "max_err_beyond_output_rounding": round(max(float((d - u).max()), 0.0), 6),
            "rel_l2": round(rel, 7), "pass": excess <= 0 and rel <= 5e-3,
            "pass_max_abs_2e-2_alone": max_abs <= 2e-2 and rel <= 5e-3}


def parity_check(w, q, k, v, do, heads: int = 4) -> dict:
    """The first `heads` heads of batch 0 of the timed inputs through the public API (forward
    and autograd backward) against the fp32 reference, for o, dq, dk and dv."""
    import pallas_flexattn as pf
    from pallas_flexattn.score_mod import slice_heads

    n = min(heads, q.shape[1])
    sl = [t.detach()[:1, :n].contiguous() for t in (q, k, v, do)]
    sm = slice_heads(w.score_mod, 0, n)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in sl[:3])
    o = pf.flash_attention(qq, kk, vv, w.mask_mod, score_mod=sm)
    got = (o, *torch.autograd.grad(o, (qq, kk, vv), sl[3]))
    ref = reference_fwd_bwd(*sl, w.mask_mod, sm, chunk=512 if w.S > 8192 else 1024)
    bf16 = w.dtype == torch.bfloat16
    res = {name: parity_stats(g, r, bf16) for name, g, r in zip(("o", "dq", "dk", "dv"), got, ref)}
    h0 = w.extra.get("heads", (0, 0))[0]
    res["slice"] = f"b=0, heads {h0}..{h0 + n - 1} of the timed inputs, every element"
    res["rule"] = PARITY_RULE
    res["pass"] = all(res[n_]["pass"] for n_ in ("o", "dq", "dk", "dv"))
    return res


def sdpa_comparators(w, q, k, v, do, flops: float, steps: int = 20) -> Optional[dict]:
    """torch scaled_dot_product_attention (cuDNN and flash backends) on the same causal
    shapes, forward + backward, for context only (the reference benchmark's comparators);
    None for workloads that SDPA cannot express (score_mod, sparse masks)."""
    import pallas_flexattn as pf
    from torch.nn.attention import SDPBackend, sdpa_kernel

    if w.mask_mod is not pf.causal_mask or w.score_mod is not None or w.dtype != torch.bfloat16:
        return None
    res = {}
    for name, backend in (("torch_sdpa_cudnn", SDPBackend.CUDNN_ATTENTION),
                          ("torch_sdpa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))

            def step():
                with sdpa_kernel(backend):
                    o = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, is_causal=True)
                torch.autograd.grad(o, (qq, kk, vv), do)

            for _ in range(3):
                step()
            torch.cuda.synchronize()
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(steps):
                step()
            e_ev.record()
            torch.cuda.synchronize()
            ms = s_ev.elapsed_time(e_ev) / steps
            res[name] = {"ms_per_step": ms, "tflops": flops / (ms * 1e-3) / 1e12}
        except Exception as e:  # backend not built for this GPU / shape
            res[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:100]}"}
    return res


def block_mask_ms(w, device, reps: int = 5) -> float:
    """Wall time of create_block_mask for the workload's mask (GPU tables), after warm-up."""
    from pallas_flexattn.block_mask import create_block_mask

    for _ in range(2):
        create_block_mask(w.mask_mod, w.B, w.H, w.S, w.S, 128, device=device)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(reps):
        create_block_mask(w.mask_mod, w.B, w.H, w.S, w.S, 128, device=device)
    torch.cuda.synchronize(device)
    return (time.perf_counter() - t0) / reps * 1e3


def cpu_baseline(w, n_pairs: int, budget_s: float = 12.0) -> dict:
    """Time the reference's tiled CPU path (torch restatement) on one (b, h) slice."""
    from oracle import cpu_reference as ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v, do = (torch.randn(w.S, w.D, generator=g) * w.input_scale for _ in range(4))
    flops = 3.5 * 4.0 * w.D * n_pairs  # fwd + bwd effective FLOPs of one slice
    reps, t_tot = 0, 0.0
    while t_tot < budget_s and reps < 50:
        t0 = time.perf_counter()
        o, lse = ref.fwd(q, k, v, w.mask_mod, w.score_mod)
        ref.bwd(q, k, v, o, lse, do, w.mask_mod, w.score_mod)
        t_tot += time.perf_counter() - t0
        reps += 1
    per = t_tot / reps
    return {"value": flops / per / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x fwd+bwd of one (b,h) slice (S={w.S}, D={w.D}, fp32, all tiles as the reference); "
                      f"{per * 1e3:.0f} ms per slice, x{w.B * w.H} slices = {per * w.B * w.H:.1f} s per full step"}


def run_reference(args, w, n_pairs, rank):
    if rank != 0:
        return 0
    from oracle import cpu_reference as ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v, do = (torch.randn(w.S, w.D, generator=g) * w.input_scale for _ in range(4))
    flops = 3.5 * 4.0 * w.D * n_pairs

    def step():
        o, lse = ref.fwd(q, k, v, w.mask_mod, w.score_mod)
        ref.bwd(q, k, v, o, lse, do, w.mask_mod, w.score_mod)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = flops / dt / 1e12
    line = {
        "impl": "reference", "metric": "effective TFLOP/s fwd+bwd (unmasked FLOPs)", "value": value,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": w.name, "B": w.B, "H": w.H, "S": w.S, "D": w.D, "mask": w.desc,
                   "sample": "one (b,h) slice per step"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"one (b,h) slice of {w.name} fwd+bwd per step, fp32, all tiles visited as "
                                   "the reference's kernels do (oracle/cpu_reference.py)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference CPU path restated in torch (the reference needs jax, which is not installed)",
    }
    print(json.dumps(line), flush=True)
    return 0


class StepTimer:
    """Device time of single steps, each bracketed by CUDA events on the launching stream,
    with an L2 flush (a write of twice the 126 MB L2) before every step, outside its events."""

    def __init__(self, device, flush: bool = True):
        self.flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=device) if flush else None

    def run(self, dist, fn, n: int, stream=None) -> float:
        """Mean ms per step over n steps, max over ranks (barrier and synchronize around)."""
        stream = stream or torch.cuda.current_stream()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        barrier(dist)
        torch.cuda.synchronize()
        for s_ev, e_ev in evs:
            if self.flush_buf is not None:
                self.flush_buf.fill_(1)
            s_ev.record(stream)
            fn()
            e_ev.record(stream)
        torch.cuda.synchronize()
        barrier(dist)
        ms = sum(s_ev.elapsed_time(e_ev) for s_ev, e_ev in evs) / n
        return max_over_ranks(dist, ms, stream.device if hasattr(stream, "device") else None)


def measure_config(cfg: int, dist, rank: int, world: int, device, steps: int, peak: float, timer: StepTimer,
                   parity: bool = True) -> dict:
    """Forward-only and backward-only time of one benchmark configuration, heads split over the
    ranks, through the public API; effective TFLOP/s of the whole problem; parity on rank 0."""
    import pallas_flexattn as pf
    from pallas_flexattn import flash_attn as FA
    from pallas_flexattn import workloads as W

    wf = W.get(cfg)
    if wf.H % world:
        return {"workload": wf.name, "skipped": f"its {wf.H} heads do not split over {world} GPUs"}
    w = wf.head_shard(rank, world)
    n_pairs = W.count_pairs(w.mask_mod, w.S, w.S, device=device)
    fwd_flops = wf.fwd_flops(n_pairs)  # the whole problem, all ranks
    q, k, v, do = w.inputs(device, seed=100 * cfg + rank)

    def fwd():
        return pf.flash_attention_fwd(q, k, v, w.mask_mod, score_mod=w.score_mod)

    o, lse = fwd()

    def bwd():
        return FA.flash_attention_bwd(q, k, v, o, lse, do, w.mask_mod, score_mod=w.score_mod)

    for _ in range(3):
        fwd()
        bwd()
    torch.cuda.synchronize()
    FA.check_device_status(device)
    ms_f = timer.run(dist, fwd, steps)
    ms_b = timer.run(dist, bwd, steps)
    FA.check_device_status(device)
    f_tf = fwd_flops / (ms_f * 1e-3) / 1e12
    b_tf = 2.5 * fwd_flops / (ms_b * 1e-3) / 1e12
    plan = FA._Plan(q, k, v, w.mask_mod, w.score_mod, None, 64, 64, 3, None, True)
    res = {"workload": wf.name, "mask": wf.desc, "shape": f"B{wf.B} H{wf.H} S{wf.S} D{wf.D}",
           "dtype": "bf16" if wf.dtype == torch.bfloat16 else "f32",
           "kernel": "tcgen05" if plan.tc else "simt (CUDA cores)",
           "unmasked_pairs_per_bh": n_pairs, "density": n_pairs / (w.S * w.S),
           "fwd": {"ms": ms_f, "tflops": f_tf, "pct_of_peak": 100 * f_tf / peak},
           "bwd": {"ms": ms_b, "tflops": b_tf, "pct_of_peak": 100 * b_tf / peak},
           "per_rank": f"heads {w.extra['heads'][0]}..{w.extra['heads'][1] - 1} of {wf.H} on each of {world} GPUs"}
    if parity and rank == 0:
        res["parity"] = parity_check(w, q, k, v, do)
    del q, k, v, do, o, lse
    torch.cuda.empty_cache()
    return res


def measure_cp_ring(dist, rank: int, world: int, device, steps: int, peak: float, timer: StepTimer,
                    cfg: int = 5) -> dict:
    """The config (default cfg5) as context-parallel ring attention over the ranks: each rank
    holds its zig-zag share of the sequence for every head, K/V (and in the backward the
    fp32 dK/dV accumulators) travel the ring on NCCL send/recv.  Whole-problem effective
    TFLOP/s of the ring forward and backward, the exchange time of one step's K/V block
    against the compute per step, and parity of one head's full sequence against fp32."""
    from pallas_flexattn import ring
    from pallas_flexattn import workloads as W
    from pallas_flexattn.score_mod import slice_heads

    wf = W.get(cfg)
    n_pairs = W.count_pairs(wf.mask_mod, wf.S, wf.S, device=device)
    fwd_flops = wf.fwd_flops(n_pairs)
    T2 = wf.S // world
    g = torch.Generator(device=device).manual_seed(500 + rank)
    q, k, v, do = (torch.randn((wf.B, wf.H, T2, wf.D), generator=g, device=device).to(wf.dtype) for _ in range(4))
    grp = dist.group.WORLD if dist is not None else None
    if dist is None:  # one GPU: a single-rank process group keeps the ring code path
        import torch.distributed as tdist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29600 + os.getpid() % 1000))
        tdist.init_process_group("gloo", rank=0, world_size=1, timeout=timedelta(seconds=120))
        grp = tdist.group.WORLD
    o, lse = ring.ring_attention_fwd(q, k, v, wf.mask_mod, wf.score_mod, group=grp)

    def fwd():
        return ring.ring_attention_fwd(q, k, v, wf.mask_mod, wf.score_mod, group=grp)

    def bwd():
        return ring.ring_attention_bwd(q, k, v, o, lse, do, wf.mask_mod, wf.score_mod, group=grp)

    for _ in range(2):
        fwd()
        bwd()
    torch.cuda.synchronize()
    ms_f = timer.run(dist, fwd, steps)
    ms_b = timer.run(dist, bwd, steps)
    # one step's K/V exchange alone (the bytes the forward moves per step), for the limiter
    ms_x = None
    kv_bytes = 2 * q.numel() * q.element_size()
    if world > 1:
        import torch.distributed as tdist

        nk, nv = torch.empty_like(k), torch.empty_like(v)
        nxt, prv = (rank + 1) % world, (rank - 1) % world

        def exchange():
            ops = [tdist.P2POp(tdist.isend, k, nxt), tdist.P2POp(tdist.isend, v, nxt),
                   tdist.P2POp(tdist.irecv, nk, prv), tdist.P2POp(tdist.irecv, nv, prv)]
            for w_ in tdist.batch_isend_irecv(ops):
                w_.wait()

        exchange()
        ms_x = timer.run(dist, exchange, steps)
    res = {"workload": wf.name, "strategy": f"zig-zag K/V ring over {world} GPU(s), {2 * world} chunks of "
                                            f"{wf.S // (2 * world)} rows, all {wf.H} heads per GPU",
           "fwd": {"ms": ms_f, "tflops": fwd_flops / (ms_f * 1e-3) / 1e12,
                   "pct_of_peak": 100 * fwd_flops / (ms_f * 1e-3) / 1e12 / world / peak},
           "bwd": {"ms": ms_b, "tflops": 2.5 * fwd_flops / (ms_b * 1e-3) / 1e12,
                   "pct_of_peak": 100 * 2.5 * fwd_flops / (ms_b * 1e-3) / 1e12 / world / peak},
           "kv_bytes_per_step": kv_bytes, "exchange_ms_per_step": ms_x,
           "compute_ms_per_step": {"fwd": ms_f / world, "bwd": ms_b / world},
           "exchange_GBps": (kv_bytes / (ms_x * 1e-3) / 1e9) if ms_x else None}
    if ms_x is not None:
        res["limiter"] = ("K/V exchange (NCCL send/recv)" if ms_x > ms_f / world else "compute per step")
    del q, k, v, do, o, lse
    torch.cuda.empty_cache()
    # parity: one head, the full sequence generated identically on every rank and split zig-zag
    g1 = torch.Generator(device=device).manual_seed(77)
    full = [torch.randn((1, 1, wf.S, wf.D), generator=g1, device=device).to(wf.dtype) for _ in range(4)]
    sm = slice_heads(wf.score_mod, 0, 1)
    mine = [ring.split_zigzag(t, rank, world).contiguous() for t in full]
    qq, kk, vv = (t.clone().requires_grad_(True) for t in mine[:3])
    o1 = ring.ring_attention(qq, kk, vv, wf.mask_mod, sm, group=grp)
    got = (o1.detach(), *torch.autograd.grad(o1, (qq, kk, vv), mine[3]))
    gathered = []
    for t in got:
        if world > 1:
            import torch.distributed as tdist

            bufs = [torch.empty_like(t) for _ in range(world)]
            tdist.all_gather(bufs, t.contiguous())
            gathered.append(ring.gather_zigzag(bufs, world))
        else:
            gathered.append(ring.gather_zigzag([t], 1))
    if rank == 0:
        ref = reference_fwd_bwd(*full, wf.mask_mod, sm, chunk=512)
        par = {n: parity_stats(a, r_, True) for n, a, r_ in zip(("o", "dq", "dk", "dv"), gathered, ref)}
        par["slice"] = "head 0 of a separate seeded input, the whole sequence gathered from the ring"
        par["pass"] = all(par[n]["pass"] for n in ("o", "dq", "dk", "dv"))
        res["parity"] = par
    if dist is None:
        import torch.distributed as tdist

        tdist.destroy_process_group()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", default="flexattn", choices=["flexattn", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-per-config", action="store_true")
    ap.add_argument("--workload", default="train", choices=["train", "decode"],
                    help="train: forward+backward step (the headline); decode: split-KV decode")
    ap.add_argument("--decode-config", default="gqa_b64", choices=sorted(DECODE_CONFIGS))
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "decode":
        dist, rank, world, local = dist_setup()
        rc = run_decode(args, dist, rank, world, local)
        if dist is not None:
            dist.destroy_process_group()
        return rc

    from pallas_flexattn import workloads as W

    wf = W.get(args.config)
    dist, rank, world, local = dist_setup()

    if args.impl == "reference":
        rc = run_reference(args, wf, _pairs_cfg(wf), rank)
        if dist is not None:
            dist.destroy_process_group()
        return rc

    import pallas_flexattn as pf
    from pallas_flexattn import flash_attn as FA

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peaks = load_peaks()
    peak = float(peaks["bf16_tflops"])
    # Strong scaling: the one problem of the config, its heads split evenly over the ranks
    # (heads are independent, so no collective runs on the data path).
    w = wf.head_shard(rank, world)
    n_pairs = W.count_pairs(w.mask_mod, w.S, w.S, device=device)
    fwd_flops = wf.fwd_flops(n_pairs)  # whole problem
    bwd_flops = 2.5 * fwd_flops
    q, k, v, do = w.inputs(device, seed=1000 + rank)
    for t in (q, k, v):
        t.requires_grad_(True)

    def step():
        o = pf.flash_attention(q, k, v, w.mask_mod, score_mod=w.score_mod)
        return torch.autograd.grad(o, (q, k, v), do)

    def fwd_only():
        return pf.flash_attention_fwd(q.detach(), k.detach(), v.detach(), w.mask_mod, score_mod=w.score_mod)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    FA.check_device_status(device)
    plan = FA._Plan(q.detach(), k.detach(), v.detach(), w.mask_mod, w.score_mod, None, 64, 64, 3, None, True)
    fwd_launches = 1
    # tcgen05 backward: preprocess (delta, lse2, zeroing of the dQ accumulator) + fused kernel
    # + dQ convert; generic backward: memset + preprocess + dQ kernel + dK/dV kernel + convert
    bwd_launches = 3 if plan.tc else 4
    timer = StepTimer(device)

    with ClockSampler(device) as clk:
        ms_step = timer.run(dist, step, args.steps)
    ms_fwd = timer.run(dist, fwd_only, args.steps)
    o0, lse0 = fwd_only()
    o0 = o0.detach()

    def bwd_only():
        return FA.flash_attention_bwd(q.detach(), k.detach(), v.detach(), o0, lse0, do, w.mask_mod,
                                      score_mod=w.score_mod)

    ms_bwd = timer.run(dist, bwd_only, args.steps)
    FA.check_device_status(device)

    value = (fwd_flops + bwd_flops) / (ms_step * 1e-3) / 1e12
    fwd_tf = fwd_flops / (ms_fwd * 1e-3) / 1e12
    bwd_tf = bwd_flops / (ms_bwd * 1e-3) / 1e12
    dominant = "bwd" if ms_bwd >= ms_fwd else "fwd"
    ach = (bwd_tf if dominant == "bwd" else fwd_tf) / world  # per GPU, against one GPU's peak
    traffic = None
    prof = REPO / "profiles" / "traffic.json"
    if prof.exists() and world == 1:
        entry = json.loads(prof.read_text()).get(f"{w.name}:{dominant}")
        traffic = entry["bytes"] if isinstance(entry, dict) else entry  # DRAM bytes per launch (ncu)

    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(dist, device, w, q, k, v, do, fwd_flops + bwd_flops, max(3, args.steps // 2))

    parity = parity_check(w, q, k, v, do) if rank == 0 else None
    bm_ms = block_mask_ms(w, device)
    comparators = sdpa_comparators(w, q, k, v, do, (fwd_flops + bwd_flops) / world) if rank == 0 else None
    del q, k, v, do, o0, lse0
    torch.cuda.empty_cache()

    per_config = None
    if not args.no_per_config:
        per_config = {}
        head = {"fwd": {"ms": ms_fwd, "tflops": fwd_tf}, "bwd": {"ms": ms_bwd, "tflops": bwd_tf}}
        for c in (1, 2, 3, 4, 5):
            if c == args.config:
                continue
            per_config[f"cfg{c}"] = measure_config(c, dist, rank, world, device, max(5, args.steps // 2), peak,
                                                   timer)
        ref2 = head if args.config == 2 else per_config.get("cfg2")
        for key, r in per_config.items():
            if ref2 is not None and key != "cfg1" and "skipped" not in r:
                r["rate_vs_cfg2_per_unmasked_flop"] = {
                    "fwd": r["fwd"]["tflops"] / ref2["fwd"]["tflops"], "bwd": r["bwd"]["tflops"] / ref2["bwd"]["tflops"]}

    cp_ring = None
    if not args.no_per_config:
        cp_ring = measure_cp_ring(dist, rank, world, device, max(3, args.steps // 4), peak, timer)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, n_pairs)

    if rank == 0:
        line = {
            "metric": "effective TFLOP/s fwd+bwd (unmasked FLOPs)", "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if w.dtype == torch.bfloat16 else "f32", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": wf.name, "B": wf.B, "H": wf.H, "S": wf.S, "D": wf.D, "mask": wf.desc,
                       "parallelism": f"heads split over {world} GPU(s): {w.H} heads x B{w.B} per GPU, "
                                      "no collective on the data path",
                       "l2": "L2 flushed before every timed step (256 MB write, outside the step's events)"},
            "pct_of_peak": 100.0 * value / world / peak,
            "fwd": {"ms": ms_fwd, "tflops": fwd_tf, "pct_of_peak": 100 * fwd_tf / world / peak,
                    "pct_of_2250": 100 * fwd_tf / world / 2250.0, "kernel": "tcgen05" if plan.tc else "simt"},
            "bwd": {"ms": ms_bwd, "tflops": bwd_tf, "pct_of_peak": 100 * bwd_tf / world / peak,
                    "pct_of_2250": 100 * bwd_tf / world / 2250.0},
            "roofline": {"bound": "tensor",
                         "kernel": ("bwd: one fa_bwd call = preprocess + bwd_tc + dq_convert launches"
                                    if dominant == "bwd" else "fwd: fwd_tc (one launch)"),
                         "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                         "frac": ach / peak, "peak_source": f"bf16_tflops ({peaks['source']})",
                         "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clk.summary(),
            "gpu_launches": args.steps * (fwd_launches + bwd_launches),
            "parity": parity,
            "per_config": per_config,
            "cp_ring": cp_ring,
            "block_mask_ms": bm_ms,
            "comparators": comparators,
            "unmasked_pairs_per_bh": n_pairs,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def measure_e2e(dist, device, w, q, k, v, do, flops: float, n: int) -> dict:
    """The step through the public API from pinned host memory: every step copies its q, k, v
    and dO in and its dq, dk and dv out.  Step i+1's inputs load on a copy stream while step i
    computes (two device input sets, ordered with events) and step i's gradients drain on a
    second copy stream; the timed region ends when the last gradient byte is on the host."""
    import pallas_flexattn as pf

    hq, hk, hv, hdo = (t.detach().to("cpu").pin_memory() for t in (q, k, v, do))
    sets = [tuple(torch.empty_like(t.detach()) for t in (q, k, v, do)) for _ in range(2)]
    g_host = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q, k, v)]
    comp, h2d, d2h = torch.cuda.current_stream(device), torch.cuda.Stream(device), torch.cuda.Stream(device)
    loaded = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    for ev in freed:
        ev.record(comp)
    state = {"i": 0}

    def load(slot):
        with torch.cuda.stream(h2d):
            h2d.wait_event(freed[slot])
            for dst, src in zip(sets[slot], (hq, hk, hv, hdo)):
                dst.copy_(src, non_blocking=True)
            loaded[slot].record(h2d)

    def e2e_step():
        i = state["i"]
        slot = i % 2
        load(1 - slot)  # next step's inputs, overlapping this step's compute
        comp.wait_event(loaded[slot])
        bq, bk, bv, bdo = sets[slot]
        qq, kk, vv = (t.requires_grad_(True) for t in (bq, bk, bv))
        o = pf.flash_attention(qq, kk, vv, w.mask_mod, score_mod=w.score_mod)
        grads = torch.autograd.grad(o, (qq, kk, vv), bdo)
        for t in (bq, bk, bv):
            t.requires_grad_(False)
        freed[slot].record(comp)
        d2h.wait_stream(comp)
        with torch.cuda.stream(d2h):
            for dst, g in zip(g_host, grads):
                g.record_stream(d2h)
                dst.copy_(g, non_blocking=True)
        state["i"] = i + 1

    load(0)
    for _ in range(2):
        e2e_step()
    barrier(dist)
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record(comp)
    for _ in range(n):
        e2e_step()
    comp.wait_stream(d2h)
    e_ev.record(comp)
    torch.cuda.synchronize()
    barrier(dist)
    ms = max_over_ranks(dist, s_ev.elapsed_time(e_ev) / n, device)
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (q, k, v, do)),
            "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in g_host), "ms_per_step": ms,
            "pipeline": "H2D of step i+1 and D2H of step i's dq/dk/dv on two copy streams overlap compute"}


DECODE_CONFIGS = {
    # name: (B, H, H_kv, Tq, Tkv, D) -- grouped-query decode of one new token per sequence
    "gqa_b64": (64, 32, 8, 1, 4096, 128),  # Llama-3-8B-like heads, 4k context, batch 64
    "gqa_b8": (8, 32, 8, 1, 8192, 128),    # smaller case (ncu captures)
    "mha_b32_d64": (32, 16, 16, 1, 8192, 64),
}


def run_decode(args, dist, rank, world, local) -> int:
    """Split-KV decode (flash_attention_decode) against a resident bf16 K/V cache: the
    metric is cache bytes read per second (K and V, every valid row once per call), the
    roofline the measured HBM copy bandwidth.  One step = one call for all B sequences."""
    import numpy as np

    import pallas_flexattn as pf
    from pallas_flexattn import flash_attn as FA

    B, H, Hkv, Tq, Tkv, D = DECODE_CONFIGS[args.decode_config]
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "workload": f"decode_{args.decode_config}",
                              "unavailable": "the reference has no decode (K/V cache) path"}), flush=True)
        return 0
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    peaks = load_peaks()
    g = torch.Generator(device="cpu").manual_seed(2000 + rank)
    kc, vc = (torch.randn(B, Hkv, Tkv, D, generator=g).to(device, torch.bfloat16) for _ in range(2))
    q = torch.randn(B, H, Tq, D, generator=g).to(device, torch.bfloat16)
    lens = torch.full((B,), Tkv, dtype=torch.int32, device=device)
    cache_bytes = 2 * B * Hkv * Tkv * D * 2

    def step():
        return pf.flash_attention_decode(q, kc, vc, lens, pf.causal_mask)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    FA.check_device_status(device)

    def timed(fn, n):
        barrier(dist)
        torch.cuda.synchronize()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(n):
            fn()
        e_ev.record()
        torch.cuda.synchronize()
        barrier(dist)
        return s_ev.elapsed_time(e_ev) / n

    with ClockSampler(device) as clk:
        ms = max_over_ranks(dist, timed(step, args.steps), device)
    FA.check_device_status(device)
    value = cache_bytes * world / (ms * 1e-3) / 1e9
    peak = float(peaks["hbm_gbs"])

    e2e = None
    if not args.no_e2e:
        # A serving step: the new tokens' q and their K/V rows come from pinned host memory
        # (appended to the cache on the device), the output rows go back to the host.
        hq = q.detach().cpu().pin_memory()
        hk, hv = (torch.randn(B, Hkv, Tq, D).to(torch.bfloat16).pin_memory() for _ in range(2))
        dq = torch.empty_like(q)
        out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()

        def e2e_step():
            dq.copy_(hq, non_blocking=True)
            kc[:, :, Tkv - Tq:].copy_(hk, non_blocking=True)
            vc[:, :, Tkv - Tq:].copy_(hv, non_blocking=True)
            o, _ = pf.flash_attention_decode(dq, kc, vc, lens, pf.causal_mask)
            out_host.copy_(o, non_blocking=True)

        for _ in range(3):
            e2e_step()
        ms_e2e = max_over_ranks(dist, timed(e2e_step, args.steps), device)
        e2e = {"value": cache_bytes * world / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": (hq.numel() + hk.numel() + hv.numel()) * 2,
               "d2h_bytes_per_step": out_host.numel() * 2, "ms_per_step": ms_e2e}

    # parity: two sequences of the timed inputs against the oracle
    parity = None
    if rank == 0:
        from oracle import flexattn_oracle as O

        o, lse = step()
        torch.cuda.synchronize()
        sl = slice(0, 2)
        qn, kn, vn = (t[sl].float().cpu().numpy().astype(np.float64) for t in (q, kc, vc))
        ro, rl = O.decode_reference(qn, kn, vn, [Tkv] * 2, O.causal)
        got = o[sl].float().cpu().numpy()
        diff = np.abs(got - ro)
        rel = float(np.linalg.norm(got - ro) / max(np.linalg.norm(ro), 1e-30))
        ok = bool((diff - (2e-2 + 2.0 ** -8 * np.abs(ro))).max() <= 0 and rel <= 5e-3)
        parity = {"o": {"max_abs": round(float(diff.max()), 6), "rel_l2": round(rel, 7)},
                  "lse_max_abs": round(float(np.abs(lse[sl].cpu().numpy() - rl).max()), 6),
                  "slice": "b = 0, 1 of the timed inputs", "pass": ok}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import flexattn_oracle as O

        qn, kn, vn = (t[:1].float().cpu().numpy().astype(np.float64) for t in (q, kc, vc))
        reps, t_tot = 0, 0.0
        while t_tot < 8.0 and reps < 200:
            t0 = time.perf_counter()
            O.decode_reference(qn, kn, vn, [Tkv], O.causal)
            t_tot += time.perf_counter() - t0
            reps += 1
        per = t_tot / reps
        cpu = {"value": cache_bytes / B / per / 1e9, "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{reps} x oracle decode_reference of one sequence (numpy fp64, Tkv={Tkv}); "
                         f"{per * 1e3:.1f} ms per sequence"}

    if rank == 0:
        line = {
            "metric": "decode K/V cache read GB/s", "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": f"decode_{args.decode_config}", "B": B, "H": H, "H_kv": Hkv, "Tq": Tq,
                       "Tkv": Tkv, "D": D, "mask": "causal",
                       "l2": f"cache {cache_bytes / 1e6:.0f} MB per rank, larger than L2"},
            "roofline": {"bound": "hbm", "kernel": "decode_tc_kernel + decode_merge_kernel (one fa_decode call)",
                         "achieved": value / world, "peak": peak, "unit": "GB/s", "frac": value / world / peak,
                         "peak_source": f"hbm_gbs ({peaks['source']})", "traffic": None},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(), "gpu_launches": 2 * args.steps,
            "parity": parity,
        }
        print(json.dumps(line), flush=True)
    return 0


def _pairs_cfg(w) -> int:
    from pallas_flexattn import workloads as W

    if "tile_table" in w.extra:
        import numpy as np

        t = w.extra["tile_table"]
        n = t.shape[0]
        return int(np.tril(t, -1).sum()) * 128 * 128 + n * (128 * 129 // 2)
    return W.count_pairs(w.mask_mod, w.S, w.S)


if __name__ == "__main__":
    sys.exit(main())
