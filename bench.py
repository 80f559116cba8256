#!/usr/bin/env python
"""Throughput of the LinOSS-IMEX oscillatory scan (forward + backward) on B200.

Workload (one "step"): the LinOSS-IMEX scan of a 4-utterance batch with P = 256
oscillators and H = 64 input channels, along time (B*F = 404 sequences x 321 steps) and
along frequency (B*T = 1284 sequences x 101 steps), forward and backward, at the scan
boundary: Bu (complex) in, y2 (complex) out; backward dY2 in, dBu and the parameter
gradients out. Synthetic seeded inputs with the workload's distributions: A = relu(N(0,1)),
dt = sigmoid(N(0,1)), complex B entries N(0, 1/sqrt(H)) per part, u ~ N(0,1), Bu = B u,
upstream gradient ~ N(0,1).

Metric: scan GB/s of algorithmic bytes (fwd 16 P B per (sequence, step): Bu in + y2 out;
bwd 24 P B: Bu + dY2 in, dBu out). Every operand is 265 MB (> the 126 MB L2), so no L2
flush is needed between steps.

Arms:
  default           — libsemx kernels through the C ABI, inputs resident in HBM (`value`);
                      plus `e2e` (host buffers, copies inside the timed region), the
                      roofline of the dominant kernel, clocks, and the CPU baseline.
  --impl reference  — the reference's CPU implementation of the path (the oracle port of
                      models/linoss/linoss.py) on the host cores, on a bounded sample.

Multi-GPU (torchrun, one process per GPU): weak scaling, each rank scans its own batch;
no collective is on the data path; time = max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
P, H = 256, 64
PASSES = (("time", 404, 321), ("freq", 1284, 101))
FWD_BYTES_PER_STEP = 16 * P  # Bu in, y2 out (complex64)
BWD_BYTES_PER_STEP = 24 * P  # Bu, dY2 in; dBu out
METRIC = "LinOSS-IMEX scan fwd+bwd, algorithmic HBM GB/s (config 1: time 404x321 + freq 1284x101, P=256)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["semx", "reference"], default="semx")
    ap.add_argument("--workload", choices=["linoss", "generator", "inference"], default="linoss",
                    help="linoss: config 1 (default); generator: config-3 training step; "
                         "inference: config-4 long-utterance inference")
    ap.add_argument("--batch", type=int, default=16, help="generator: utterances per GPU")
    ap.add_argument("--micro-batch", type=int, default=4, help="inference: utterances per forward")
    ap.add_argument("--chunk", type=int, default=64)
    ap.add_argument("--cpu-sample-frac", type=float, default=0.125)
    ap.add_argument("--ref-sample-frac", type=float, default=1.0 / 16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--clocks-log", default=None)
    ap.add_argument("--no-soak", action="store_true",
                    help="skip the 1.5 s busy period before timing (for profiler runs)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- helpers
def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` recorded by an ncu capture in profiles/*.md
    (a line `traffic_bytes_per_launch[<kernel>]: <int>`), or None."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        m = re.search(rf"traffic_bytes_per_launch\[{re.escape(kernel)}\]:\s*([0-9.e+]+)", f.read_text())
        if m:
            return float(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples (200 ms) of one GPU while it runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_uuid: str | None, log_path: str | None):
        self.samples = []
        self.proc = None
        self.log = open(log_path, "w") if log_path else None
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "200"]
        if device_uuid:
            cmd += ["-i", device_uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            t = time.time()
            if self.log:
                self.log.write(f"{t:.3f},{line}")
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                self.samples.append((t, float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.log:
            self.log.close()

    def summary(self, t0: float, t1: float):
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted({name for s in win for name, flag in zip(self.REASONS, s[3])
                          if flag.lower().startswith("active")})
        return {"sm_mhz": statistics.median(s[1] for s in win), "sm_max_mhz": max(s[2] for s in win),
                "reasons": reasons, "samples": len(win)}


# ----------------------------------------------------------------------------- workload
class LinossPass:
    """One scan pass (S sequences x L steps x P oscillators) with resident device buffers
    and prebuilt C-ABI argument structs for semx_linoss_fwd / semx_linoss_bwd."""

    def __init__(self, S, L, seed, device, chunk):
        from semambaxlinoss_b200 import _lib

        self.lib = _lib.load()
        self._lib = _lib
        self.S, self.L = S, L
        g = torch.Generator(device=device).manual_seed(seed)
        self.steps = torch.randn(P, generator=g, device=device)
        self.A = torch.randn(P, generator=g, device=device)  # relu applied in-kernel
        Bw = torch.randn(P, H, 2, generator=g, device=device) / H**0.5
        W = Bw.permute(0, 2, 1).reshape(2 * P, H)
        self.Bu = torch.empty(S, L, P, dtype=torch.complex64, device=device)
        Bu_r = torch.view_as_real(self.Bu).view(S * L, 2 * P)
        for i in range(0, S * L, 65536):
            u = torch.randn(min(65536, S * L - i), H, generator=g, device=device)
            torch.matmul(u, W.t(), out=Bu_r[i:i + u.shape[0]])
        self.dY2 = torch.randn(S, L, P, dtype=torch.complex64, generator=g, device=device)
        self.Y2 = torch.empty_like(self.Bu)
        self.dBu = torch.empty_like(self.Bu)
        self.dparams = torch.zeros(3, P, device=device)
        ck = self.lib.semx_linoss_ckpt_bytes(S, L, P, chunk)
        self.ckpt = torch.empty(ck // 4, device=device)
        a = _lib.new_args(_lib.SemxLinossArgs)
        a.variant, a.a_from_g, a.chunk, a.S, a.L, a.P = _lib.LINOSS_IMEX, 1, chunk, S, L, P
        a.steps, a.A_diag, a.Bu = self.steps.data_ptr(), self.A.data_ptr(), self.Bu.data_ptr()
        a.Y2, a.ckpt, a.dY2 = self.Y2.data_ptr(), self.ckpt.data_ptr(), self.dY2.data_ptr()
        a.dBu, a.dparams = self.dBu.data_ptr(), self.dparams.data_ptr()
        self.ws = torch.empty(self.lib.semx_linoss_workspace_bytes(ctypes.byref(a)) // 4,
                              device=device)
        a.workspace = self.ws.data_ptr()
        self.args = a
        self.units = S * L

    def fwd(self, stream):
        self._lib.check("semx_linoss_fwd", self.lib.semx_linoss_fwd(ctypes.byref(self.args), stream))

    def bwd(self, stream):
        self._lib.check("semx_linoss_bwd", self.lib.semx_linoss_bwd(ctypes.byref(self.args), stream))


def run_semx(args, rank, local_rank, world):
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    passes = [LinossPass(S, L, seed=1000 * rank + i, device=device, chunk=args.chunk)
              for i, (_, S, L) in enumerate(PASSES)]
    stream = torch.cuda.current_stream(device)
    sh = stream.cuda_stream
    step_bytes = sum(p.units * (FWD_BYTES_PER_STEP + BWD_BYTES_PER_STEP) for p in passes)
    launches_per_step = 3 * len(passes)  # fwd, bwd, finalize per pass

    def step(ev=None):
        for i, p in enumerate(passes):
            if ev is not None:
                ev[i][0].record(stream)
            p.fwd(sh)
            if ev is not None:
                ev[i][1].record(stream)
            p.bwd(sh)
            if ev is not None:
                ev[i][2].record(stream)

    def barrier():
        torch.cuda.synchronize(device)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(device)

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    clocks = ClockSampler(uuid, args.clocks_log if rank == 0 else None)

    for _ in range(max(args.warmup, 3)):
        step()
    # Keep the GPU busy ~1.5 s before timing so the clock samples see it under load.
    soak_t0 = time.time()
    torch.cuda.synchronize(device)
    while not args.no_soak and time.time() - soak_t0 < 1.5:
        for _ in range(20):
            step()
        torch.cuda.synchronize(device)

    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in passes]
          for _ in range(args.steps)]
    barrier()
    t_wall0 = time.time()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for k in range(args.steps):
        step(ev[k])
    end.record(stream)
    barrier()
    t_wall1 = time.time()
    elapsed = start.elapsed_time(end)
    clocks.stop()
    fwd_ms = [ev[k][i][0].elapsed_time(ev[k][i][1]) for k in range(args.steps) for i in range(len(passes))]
    bwd_ms = [ev[k][i][1].elapsed_time(ev[k][i][2]) for k in range(args.steps) for i in range(len(passes))]

    t = torch.tensor([elapsed], device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed = t.item()
    ms_per_step = elapsed / args.steps
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9

    e2e = None if args.no_e2e else run_e2e(passes, args, device, stream, step_bytes, world)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peak, peak_kind = load_peaks()
    units = passes[0].units  # both passes process S*L = 129,684 (sequence, step) units
    fwd_avg, bwd_avg = statistics.mean(fwd_ms), statistics.mean(bwd_ms)
    fwd_gbs = units * FWD_BYTES_PER_STEP / (fwd_avg * 1e-3) / 1e9
    bwd_gbs = units * BWD_BYTES_PER_STEP / (bwd_avg * 1e-3) / 1e9
    dom = "linoss_bwd_kernel" if bwd_avg >= fwd_avg else "linoss_fwd_kernel"
    dom_gbs = bwd_gbs if dom == "linoss_bwd_kernel" else fwd_gbs
    traffic = profiled_traffic(dom)
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; distributions of config 1)",
        "config": {
            "workload": "LinOSS-IMEX scan fwd+bwd, time 404x321 + freq 1284x101, P=256, H=64",
            "passes": [{"axis": n, "sequences": S, "steps": L} for n, S, L in PASSES],
            "oscillators": P, "chunk": args.chunk,
            "bytes_per_step": step_bytes,
            "l2": "no flush: every operand is 265 MB, larger than the 126 MB L2",
            "parallelism": f"weak dp{world}: each rank scans its own batch, no collective",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": dom,
            "achieved": round(dom_gbs, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(dom_gbs / peak, 4),
            "peak_kind": peak_kind,
            "traffic": traffic,
            "note": "event pair around semx_linoss_bwd also covers its finalize launch (a few us)",
        },
        "kernels": {
            "linoss_fwd_kernel": {"ms": round(fwd_avg, 4), "GB/s": round(fwd_gbs, 1),
                                  "bytes_per_launch": units * FWD_BYTES_PER_STEP},
            "linoss_bwd_kernel+finalize": {"ms": round(bwd_avg, 4), "GB/s": round(bwd_gbs, 1),
                                           "bytes_per_launch": units * BWD_BYTES_PER_STEP},
        },
        "hbm_frac_of_8tbs": round(value / world / 8000.0, 4),
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(soak_t0, t_wall1),
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.cpu_sample_frac, repeats=3)
    print(json.dumps(out), flush=True)


def run_e2e(passes, args, device, stream, step_bytes, world):
    """Same metric through the C ABI with host buffers: every step copies Bu and dY2 from
    pinned host memory, runs forward and backward, and copies y2, dBu and the parameter
    gradients back to pinned host memory, all inside the timed region."""
    sh = stream.cuda_stream
    host = []
    for p in passes:
        host.append({
            "Bu": p.Bu.cpu().pin_memory(), "dY2": p.dY2.cpu().pin_memory(),
            "Y2": torch.empty(p.Y2.shape, dtype=p.Y2.dtype).pin_memory(),
            "dBu": torch.empty(p.dBu.shape, dtype=p.dBu.dtype).pin_memory(),
            "dparams": torch.empty(3, P).pin_memory(),
        })
    h2d = sum(h["Bu"].numel() * 8 + h["dY2"].numel() * 8 for h in host)
    d2h = sum(h["Y2"].numel() * 8 + h["dBu"].numel() * 8 + 3 * P * 4 for h in host)

    def e2e_step():
        for p, h in zip(passes, host):
            p.Bu.copy_(h["Bu"], non_blocking=True)
            p.dY2.copy_(h["dY2"], non_blocking=True)
            p.fwd(sh)
            p.bwd(sh)
            h["Y2"].copy_(p.Y2, non_blocking=True)
            h["dBu"].copy_(p.dBu, non_blocking=True)
            h["dparams"].copy_(p.dparams, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e.record(stream)
    torch.cuda.synchronize(device)
    t = torch.tensor([s.elapsed_time(e)], device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item() / args.e2e_steps
    return {"value": round(world * step_bytes / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "ms_per_step": round(ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "C ABI (semx_linoss_fwd/bwd) with pinned host buffers, one stream"}


# ----------------------------------------------------------------------------- CPU legs
def _cpu_sample(frac, seed=0):
    g = torch.Generator().manual_seed(seed)
    steps = torch.randn(P, generator=g)
    A = torch.randn(P, generator=g)
    sample = []
    for _, S, L in PASSES:
        s = max(1, int(round(S * frac)))
        Bw = torch.randn(P, H, 2, generator=g) / H**0.5
        u = torch.randn(s, L, H, generator=g)
        Bu = torch.complex(u @ Bw[..., 0].t(), u @ Bw[..., 1].t())
        gy = torch.complex(torch.randn(s, L, P, generator=g), torch.randn(s, L, P, generator=g))
        sample.append((s, L, Bu, gy))
    return steps, A, sample


def _cpu_step(steps, A, sample):
    """The reference's CPU path for this scan (oracle port of models/linoss/linoss.py:
    constraints, IMEX discretisation and the sequential _linoss_recurrence), fwd + bwd."""
    from oracle import linoss as olin

    for s, L, Bu, gy in sample:
        st = steps.clone().requires_grad_(True)
        a = A.clone().requires_grad_(True)
        b = Bu.clone().requires_grad_(True)
        y2 = olin.linoss_scan_fused("IMEX", st, a, None, b)
        (y2.real * gy.real + y2.imag * gy.imag).sum().backward()


def _sample_bytes(sample):
    return sum(s * L * (FWD_BYTES_PER_STEP + BWD_BYTES_PER_STEP) for s, L, _, _ in sample)


def cpu_baseline(frac, repeats=3):
    torch.set_num_threads(os.cpu_count())
    steps, A, sample = _cpu_sample(frac)
    _cpu_step(steps, A, sample)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        _cpu_step(steps, A, sample)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    desc = " + ".join(f"{s}x{L}" for s, L, _, _ in sample)
    return {"value": round(_sample_bytes(sample) / t / 1e9, 4), "unit": "GB/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{frac:.4g} of each pass's sequences ({desc}), fwd+bwd float32, median of {repeats}",
            "seconds": round(t, 3)}


def run_reference(args, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count())
    steps, A, sample = _cpu_sample(args.ref_sample_frac)
    for _ in range(args.warmup):
        _cpu_step(steps, A, sample)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _cpu_step(steps, A, sample)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = _sample_bytes(sample) / (ms * 1e-3) / 1e9
    desc = " + ".join(f"{s}x{L}" for s, L, _, _ in sample)
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": 0,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; distributions of config 1)",
        "config": {"workload": "LinOSS-IMEX scan fwd+bwd, time 404x321 + freq 1284x101, P=256, H=64",
                   "sample": desc},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{args.ref_sample_frac:.4g} of each pass's sequences ({desc}) per step"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------- generator workloads
def _barrier(world, device):
    torch.cuda.synchronize(device)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize(device)


def _max_over_ranks(ms, world, device):
    t = torch.tensor([ms], device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def _init_dist(world, device):
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)


def run_generator(args, rank, local_rank, world):
    """Config 3: SEMamba generator training step (forward + generator losses + backward +
    DDP gradient all-reduce + AdamW), bf16 autocast around fp32 scans, `--batch`
    two-second utterances per GPU. Metric: frames/s over all GPUs."""
    from semambaxlinoss_b200.generator import SEMamba, config3_cfg, generator_loss, mag_phase_stft

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _init_dist(world, device)
    cfg = config3_cfg()
    sc, cf = cfg["stft_cfg"], cfg["model_cfg"]["compress_factor"]
    torch.manual_seed(1234)
    model = SEMamba(cfg).to(device)
    n_params = sum(p.numel() for p in model.parameters())
    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP

        model = DDP(model, device_ids=[local_rank], broadcast_buffers=False, gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=5e-4, betas=(0.8, 0.99))
    B, seg = args.batch, 32000
    g = torch.Generator().manual_seed(100 + rank)
    clean_h = (torch.randn(B, seg, generator=g) * 0.1).pin_memory()
    noisy_h = (clean_h + torch.randn(B, seg, generator=g) * 0.05).pin_memory()
    clean_d, noisy_d = clean_h.to(device), noisy_h.to(device)
    loss_h = torch.empty(1).pin_memory()
    frames = (seg // sc["hop_size"]) + 1

    def step(clean, noisy, copy_in=False):
        if copy_in:
            clean.copy_(clean_h, non_blocking=True)
            noisy.copy_(noisy_h, non_blocking=True)
        clean_mag, clean_pha, clean_com = mag_phase_stft(clean, sc["n_fft"], sc["hop_size"], sc["win_size"], cf)
        noisy_mag, noisy_pha, _ = mag_phase_stft(noisy, sc["n_fft"], sc["hop_size"], sc["win_size"], cf)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            mag_g, pha_g, com_g = model(noisy_mag, noisy_pha)
        loss = generator_loss(cfg, clean, clean_mag, clean_pha, clean_com, mag_g.float(), pha_g.float(),
                              com_g.float())
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss

    stream = torch.cuda.current_stream(device)
    for _ in range(max(args.warmup, 3)):
        step(clean_d, noisy_d)
    uuid = _device_uuid(device)
    clocks = ClockSampler(uuid, args.clocks_log if rank == 0 else None)
    soak_t0 = time.time()
    _barrier(world, device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(args.steps):
        loss = step(clean_d, noisy_d)
    e.record(stream)
    _barrier(world, device)
    t_end = time.time()
    ms = _max_over_ranks(s.elapsed_time(e), world, device) / args.steps
    # End to end: audio copied in from pinned host memory and the loss read back, every step.
    _barrier(world, device)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    for _ in range(args.e2e_steps):
        loss = step(clean_d, noisy_d, copy_in=True)
        loss_h.copy_(loss.detach().reshape(1), non_blocking=True)
    e2.record(stream)
    _barrier(world, device)
    ms_e2e = _max_over_ranks(s2.elapsed_time(e2), world, device) / args.e2e_steps
    clocks.stop()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return
    fps = world * B * frames / (ms * 1e-3)
    print(json.dumps({
        "metric": "SEMamba generator training step, frames/s (config 3: 2 s utterances, batch 16 per GPU)",
        "value": round(fps, 1), "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 autocast, fp32 scans",
        "data": "synthetic (clean ~ N(0, 0.1), noise ~ N(0, 0.05), seeded per rank)",
        "config": {"workload": "config 3: generator fwd + losses + bwd + AdamW, 4 TF-blocks (time: selective-LRU "
                               "d_inner 256 N 16; freq: damped-IMEX LinOSS P 16), hid 64",
                   "global_batch": world * B, "seq_len": frames, "parallelism": f"ddp{world}",
                   "parameters": n_params,
                   "l2": "no flush: activations per step are tens of GB, far beyond the 126 MB L2"},
        "e2e": {"value": round(world * B * frames / (ms_e2e * 1e-3), 1), "unit": "frames/s",
                "ms_per_step": round(ms_e2e, 3), "h2d_bytes_per_step": 2 * B * seg * 4,
                "d2h_bytes_per_step": 4},
        "clocks": clocks.summary(soak_t0, t_end),
    }), flush=True)


def run_inference(args, rank, local_rank, world):
    """Config 4: 64 sixty-second utterances (T = 9601 frames) enhanced end to end (STFT ->
    generator -> iSTFT) under no_grad with bf16 autocast, sharded over the GPUs,
    `--micro-batch` utterances per forward. Metric: frames/s over all GPUs."""
    from semambaxlinoss_b200.generator import SEMamba, config3_cfg, mag_phase_istft, mag_phase_stft

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _init_dist(world, device)
    cfg = config3_cfg()
    sc, cf = cfg["stft_cfg"], cfg["model_cfg"]["compress_factor"]
    torch.manual_seed(1234)
    model = SEMamba(cfg).to(device).eval()
    total, seg = 64, 960000
    per_rank = [len(range(r, total, world)) for r in range(world)][rank]
    mb = args.micro_batch
    g = torch.Generator().manual_seed(200 + rank)
    audio = (torch.randn(per_rank, seg, generator=g) * 0.1).pin_memory()
    out_h = torch.empty(per_rank, seg).pin_memory()
    frames = seg // sc["hop_size"] + 1
    buf = torch.empty(mb, seg, device=device)

    def run_all():
        for i in range(0, per_rank, mb):
            n = min(mb, per_rank - i)
            x = buf[:n]
            x.copy_(audio[i:i + n], non_blocking=True)
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                mag, pha, _ = mag_phase_stft(x, sc["n_fft"], sc["hop_size"], sc["win_size"], cf)
                mag_g, pha_g, _ = model(mag, pha)
                wav = mag_phase_istft(mag_g.float(), pha_g.float(), sc["n_fft"], sc["hop_size"], sc["win_size"], cf)
            out_h[i:i + n, :wav.shape[-1]].copy_(wav[:, :seg], non_blocking=True)

    stream = torch.cuda.current_stream(device)
    run_all()  # warm-up pass over the shard
    uuid = _device_uuid(device)
    clocks = ClockSampler(uuid, args.clocks_log if rank == 0 else None)
    t0 = time.time()
    _barrier(world, device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(args.steps):
        run_all()
    e.record(stream)
    _barrier(world, device)
    t1 = time.time()
    clocks.stop()
    ms = _max_over_ranks(s.elapsed_time(e), world, device) / args.steps
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return
    fps = total * frames / (ms * 1e-3)
    print(json.dumps({
        "metric": "SEMamba long-utterance inference, frames/s (config 4: 64 x 60 s, sharded)",
        "value": round(fps, 1), "unit": "frames/s", "n_gpus": world, "steps": args.steps, "warmup": 1,
        "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 autocast, fp32 scans", "data": "synthetic (audio ~ N(0, 0.1), seeded per rank)",
        "config": {"workload": "config 4: STFT -> generator -> iSTFT, no_grad", "global_batch": total,
                   "seq_len": frames, "micro_batch": mb, "parallelism": f"sharded over {world} GPUs"},
        "e2e": {"value": round(fps, 1), "unit": "frames/s", "h2d_bytes_per_step": total * seg * 4 // world,
                "d2h_bytes_per_step": total * seg * 4 // world,
                "note": "every step copies its audio in from pinned host memory and the enhanced audio out"},
        "clocks": clocks.summary(t0, t1),
    }), flush=True)


def _device_uuid(device):
    try:
        u = str(torch.cuda.get_device_properties(device).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


def main():
    args = parse_args()
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        if args.workload != "linoss":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference generator needs the "
                                  "third-party mamba_ssm package, which the reference does not ship"}))
            return
        run_reference(args, rank)
        return
    if args.workload == "generator":
        run_generator(args, rank, local_rank, world)
    elif args.workload == "inference":
        run_inference(args, rank, local_rank, world)
    else:
        run_semx(args, rank, local_rank, world)


if __name__ == "__main__":
    main()
