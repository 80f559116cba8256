#!/usr/bin/env python
"""Throughput of the SEMamba TF-block scans on B200.

Workloads (`--workload`; one "step" = one forward + backward of every pass listed):

  scans (default)   configs 0, 1 and 2 below in one step (slru, then linoss, then mimo);
                    `value` = their algorithmic bytes / the step's time, with a per-config
                    table and a per-kernel roofline table. Also measures the generator
                    training step (config 3) as the `generator` sub-line, and at N > 1 the
                    named shapes split over the ranks (`sharded`, strong scaling).
  slru              Config 0. Real selective-LRU diagonal scan (fused discretisation + readout
                    + D skip), 404 sequences x 321 steps, C = 256 channels, N = 16 modes, Mamba
                    gain: x ~ N(0,1), dt = softplus(N(-2, 0.5)), a = exp(A_log) with A_log ~
                    log U(1,16), B_t, C_t ~ N(0, 1/16), D ~ N(0,1). Algorithmic bytes per
                    (sequence, step): fwd 4 (3C + 2N) = 3200 (x, dt, B, C in; y out), bwd
                    4 (5C + 4N) = 5376 (x, dt, dy, B, C in; d_dt, dx, dB, dC out).
  linoss            Config 1. LinOSS-IMEX oscillatory scan, P = 256 oscillators, H = 64 inputs,
                    at the scan boundary (Bu in, y2 out; dY2 in, dBu + parameter gradients
                    out): time pass 404 sequences x 321 steps, frequency pass 1284 x 101.
                    A = relu(N(0,1)), dt = sigmoid(N(0,1)), complex B entries N(0, 1/sqrt(H)),
                    u ~ N(0,1), Bu = B u, upstream gradient N(0,1).
                    Algorithmic bytes per (sequence, step): fwd 16 P, bwd 24 P.
  mimo              Config 2. SelectiveLRUMIMO layer, 256 features = 8 heads x 32, 128 state
                    (16 per head), rank 4, bf16 input, fp32 state: time pass 404 x 321,
                    frequency pass 1284 x 101. Algorithmic bytes per (sequence, step) of the
                    layer's token-level operands: fwd 4768, bwd 8512.
  generator         Config 3. SEMamba generator training step (STFT, forward, losses, backward,
                    AdamW), 2 s utterances, batch 16 per GPU, DDP over NCCL; frames/s.
  inference         Config 4. 64 sixty-second utterances enhanced end to end, sharded; frames/s.

Scan workloads report algorithmic GB/s (`value`, inputs resident in HBM), `e2e` (the same
metric with host buffers and the copies inside the timed region), the roofline of the
dominant kernel (and the table of every kernel), clocks sampled during the timed region,
the kernel launch count and a CPU baseline (the reference algorithm on the host cores, on a
fixed sample per config). Every scan operand is larger than the 126 MB L2 except where
`config.l2` says otherwise.

`--impl reference` times the reference's CPU implementation of the path (the oracle port)
on the host cores, on the same fixed sample of the same workload.

Multi-GPU (torchrun, one process per GPU): weak scaling for the scans (the global batch is
N times the named shapes; rank r scans its contiguous slice r, no collective on the data
path) plus the strong-scaling `sharded` run, and the training step (DDP); time = max over
ranks, measured with CUDA events.
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
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default per workload)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["semx", "reference"], default="semx")
    ap.add_argument("--workload", choices=["scans", "linoss", "slru", "mimo", "ops", "surround", "generator",
                                           "inference"],
                    default="scans")
    ap.add_argument("--batch", type=int, default=16, help="generator: utterances per GPU")
    ap.add_argument("--micro-batch", type=int, default=8, help="inference: utterances per forward")
    ap.add_argument("--stream-chunk", type=int, default=0,
                    help="inference: time-scan pieces of this many frames carrying the scan state "
                         "(SelectiveLRU.stream_chunk; 0 = one piece)")
    ap.add_argument("--chunk", type=int, default=None, help="checkpoint interval of the scan")
    ap.add_argument("--slru-complex", action="store_true",
                    help="slru: the complex scan with the gamma gain (the generator's time scans)")
    ap.add_argument("--sequences", type=int, default=None, help="slru: sequences (default 404)")
    ap.add_argument("--ref-sample-frac", type=float, default=None,
                    help="reference arm: fraction of each pass's sequences per step (default: the "
                         "workload's fixed sample)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="N > 1: skip the strong-scaling run over the named shapes")
    ap.add_argument("--no-generator", action="store_true",
                    help="scans: skip the generator training-step sub-measurement")
    ap.add_argument("--gen-steps", type=int, default=10, help="timed generator steps (scans workload)")
    ap.add_argument("--no-inference", action="store_true",
                    help="scans: skip the long-utterance inference sub-measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--clocks-log", default=None)
    ap.add_argument("--no-soak", action="store_true",
                    help="skip the 1.5 s busy period before timing (for profiler runs)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"scans": 20, "linoss": 200, "slru": 20, "mimo": 20, "ops": 20, "surround": 20,
                      "generator": 10, "inference": 1}[args.workload]
    return args


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


def profiled_traffic(kernel: str, workload: str, units: int):
    """DRAM bytes of one launch of `kernel` over `units` (sequence, step) units, from an
    ncu capture recorded in profiles/*.md as `traffic_bytes_per_launch[<kernel>|<workload>|
    <units>]: <bytes>`; a capture of a different size is scaled by the units processed
    (the traffic of these scans grows in proportion). Returns (bytes, source) with source
    naming the profile file and the capture's size, or (None, None) if none is recorded."""
    pat = re.compile(rf"traffic_bytes_per_launch\[{re.escape(kernel)}\|{re.escape(workload)}\|(\d+)\]:\s*(\d+)")
    for f in sorted((ROOT / "profiles").glob("*.md")):
        m = pat.search(f.read_text())
        if m:
            return (float(m.group(2)) * units / int(m.group(1)),
                    f"profiles/{f.name} (ncu capture of {m.group(1)} units"
                    + (", scaled by units)" if int(m.group(1)) != units else ")"))
    return None, None


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


def _device_uuid(device):
    try:
        u = str(torch.cuda.get_device_properties(device).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


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


def _finish_dist(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ LinOSS scan workload
LIN_P, LIN_H = 256, 64
LIN_PASSES = (("time", 404, 321), ("freq", 1284, 101))


class LinossPass:
    """One LinOSS-IMEX pass (S sequences x L steps x P oscillators) with resident device
    buffers and prebuilt C-ABI argument structs for semx_linoss_fwd / semx_linoss_bwd."""

    fwd_bytes_per_unit = 16 * LIN_P  # Bu in, y2 out (complex64)
    bwd_bytes_per_unit = 24 * LIN_P  # Bu, dY2 in; dBu out
    kernels = ("linoss_fwd_kernel", "linoss_bwd_kernel")

    def __init__(self, S, L, seed, device, chunk):
        from semambaxlinoss_b200 import _lib

        P, H = LIN_P, LIN_H
        self.lib, self._lib = _lib.load(), _lib
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
        self.inputs = [self.Bu, self.dY2]
        self.outputs = [self.Y2, self.dBu, self.dparams]

    def fwd(self, sh):
        self._lib.check("semx_linoss_fwd", self.lib.semx_linoss_fwd(ctypes.byref(self.args), sh))

    def bwd(self, sh):
        self._lib.check("semx_linoss_bwd", self.lib.semx_linoss_bwd(ctypes.byref(self.args), sh))


def _linoss_cpu_sample(frac, seed=0):
    P, H = LIN_P, LIN_H
    g = torch.Generator().manual_seed(seed)
    steps = torch.randn(P, generator=g)
    A = torch.randn(P, generator=g)
    sample = []
    for _, S, L in LIN_PASSES:
        s = max(1, int(round(S * frac)))
        Bw = torch.randn(P, H, 2, generator=g) / H**0.5
        u = torch.randn(s, L, H, generator=g)
        Bu = torch.complex(u @ Bw[..., 0].t(), u @ Bw[..., 1].t())
        gy = torch.complex(torch.randn(s, L, P, generator=g), torch.randn(s, L, P, generator=g))
        sample.append((s, L, Bu, gy))
    return {"params": (steps, A), "passes": sample, "frac": sample[0][0] / LIN_PASSES[0][1],
            "bytes": sum(s * L * (16 + 24) * P for s, L, _, _ in sample),
            "desc": " + ".join(f"{s}x{L}" for s, L, _, _ in sample)}


def _linoss_cpu_step(sample):
    """The reference's CPU path for this scan (oracle port of models/linoss/linoss.py:
    constraints, IMEX discretisation and the sequential _linoss_recurrence), fwd + bwd."""
    from oracle import linoss as olin

    steps, A = sample["params"]
    for _, _, Bu, gy in sample["passes"]:
        st = steps.clone().requires_grad_(True)
        a = A.clone().requires_grad_(True)
        b = Bu.clone().requires_grad_(True)
        y2 = olin.linoss_scan_fused("IMEX", st, a, None, b)
        (y2.real * gy.real + y2.imag * gy.imag).sum().backward()


# ------------------------------------------------------------- selective-LRU SISO workload
SLRU_S, SLRU_L, SLRU_C, SLRU_N = 404, 321, 256, 16


class SlruPass:
    """The selective-LRU scan over S x L x C channels x N modes with resident buffers and
    prebuilt argument structs for semx_selective_lru_fwd / _bwd: the real scan with the
    Mamba gain, or (`complex_`) the generator's complex scan with the gamma gain
    (delta_theta ~ N(0, 0.1^2), omega ~ N(0, 1), B_im, C_im ~ N(0, 1/16))."""

    kernels = ("slru_fwd_kernel", "slru_bwd_kernel")

    def __init__(self, S, L, seed, device, chunk, complex_=False):
        from semambaxlinoss_b200 import _lib

        C, N = SLRU_C, SLRU_N
        self.lib, self._lib = _lib.load(), _lib
        self.complex_ = complex_
        # The real forward with N <= 16 modes runs slru_fwd_real16_kernel.
        self.kernels = ("slru_fwd_kernel" if complex_ else "slru_fwd_real16_kernel", "slru_bwd_kernel")
        if complex_:  # x, dt, dth, B, C (re, im) in, y out / + dy in, 3 channel + 4 mode grads out
            self.fwd_bytes_per_unit = 4 * (4 * C + 4 * N)
            self.bwd_bytes_per_unit = 4 * (7 * C + 8 * N)
        else:
            self.fwd_bytes_per_unit = 4 * (3 * C + 2 * N)
            self.bwd_bytes_per_unit = 4 * (5 * C + 4 * N)
        g = torch.Generator(device=device).manual_seed(seed)
        f = torch.float32
        self.x = torch.randn(S, L, C, generator=g, device=device)
        self.dnu = torch.nn.functional.softplus(torch.randn(S, L, C, generator=g, device=device) * 0.5 - 2.0)
        self.a = torch.rand(C, N, generator=g, device=device) * 15.0 + 1.0
        self.B = torch.randn(S, L, N, generator=g, device=device) * 0.25
        self.Cr = torch.randn(S, L, N, generator=g, device=device) * 0.25
        self.D = torch.randn(C, generator=g, device=device)
        self.dy = torch.randn(S, L, C, generator=g, device=device)
        self.y = torch.empty(S, L, C, dtype=f, device=device)
        self.d_dnu, self.dx = torch.empty_like(self.y), torch.empty_like(self.y)
        self.dB, self.dC = torch.empty_like(self.B), torch.empty_like(self.B)
        self.da, self.dD = torch.empty(C, N, device=device), torch.empty(C, device=device)
        a = _lib.new_args(_lib.SemxSelectiveLruArgs)
        a.real, a.input_gain, a.chunk = int(not complex_), _lib.GAIN_CODES["gamma" if complex_ else "mamba"], chunk
        a.S, a.L, a.C, a.N = S, L, C, N
        named = [("delta_nu", self.dnu), ("a", self.a), ("B_re", self.B), ("C_re", self.Cr),
                 ("x", self.x), ("D", self.D), ("y", self.y), ("dy", self.dy),
                 ("d_delta_nu", self.d_dnu), ("dx", self.dx), ("dB_re", self.dB),
                 ("dC_re", self.dC), ("da", self.da), ("dD", self.dD)]
        extra_in, extra_out = [], []
        if complex_:
            self.dth = torch.randn(S, L, C, generator=g, device=device) * 0.1
            self.om = torch.randn(C, N, generator=g, device=device)
            self.Bi = torch.randn(S, L, N, generator=g, device=device) * 0.25
            self.Ci = torch.randn(S, L, N, generator=g, device=device) * 0.25
            self.d_dth = torch.empty_like(self.y)
            self.dBi, self.dCi = torch.empty_like(self.B), torch.empty_like(self.B)
            self.dom = torch.empty(C, N, device=device)
            named += [("delta_theta", self.dth), ("omega", self.om), ("B_im", self.Bi), ("C_im", self.Ci),
                      ("d_delta_theta", self.d_dth), ("dB_im", self.dBi), ("dC_im", self.dCi),
                      ("domega", self.dom)]
            extra_in = [self.dth, self.Bi, self.Ci]
            extra_out = [self.d_dth, self.dBi, self.dCi, self.dom]
        for name, t in named:
            setattr(a, name, t.data_ptr())
        self.ckpt = _lib.empty_f32(self.lib.semx_selective_lru_ckpt_bytes(ctypes.byref(a)), device)
        a.ckpt = self.ckpt.data_ptr()
        self.ws = _lib.empty_f32(self.lib.semx_selective_lru_workspace_bytes(ctypes.byref(a)), device)
        a.workspace = self.ws.data_ptr()
        self.args = a
        self.units = S * L
        self.S, self.L = S, L
        self.inputs = [self.x, self.dnu, self.B, self.Cr, self.dy] + extra_in
        self.outputs = [self.y, self.d_dnu, self.dx, self.dB, self.dC, self.da, self.dD] + extra_out

    def fwd(self, sh):
        self._lib.check("semx_selective_lru_fwd", self.lib.semx_selective_lru_fwd(ctypes.byref(self.args), sh))

    def bwd(self, sh):
        self._lib.check("semx_selective_lru_bwd", self.lib.semx_selective_lru_bwd(ctypes.byref(self.args), sh))


def _slru_cpu_sample(frac, seed=0, complex_=False, S=None):
    C, N = SLRU_C, SLRU_N
    S = S or SLRU_S
    g = torch.Generator().manual_seed(seed)
    s = max(1, int(round(S * frac)))
    L = SLRU_L
    t = {"dnu": torch.nn.functional.softplus(torch.randn(s, L, C, generator=g) * 0.5 - 2.0),
         "a": torch.rand(C, N, generator=g) * 15.0 + 1.0,
         "B": torch.randn(s, L, N, generator=g) * 0.25, "C": torch.randn(s, L, N, generator=g) * 0.25,
         "x": torch.randn(s, L, C, generator=g), "D": torch.randn(C, generator=g)}
    per_unit = 4 * (8 * C + 6 * N)
    if complex_:
        t.update(dth=torch.randn(s, L, C, generator=g) * 0.1, om=torch.randn(C, N, generator=g),
                 Bi=torch.randn(s, L, N, generator=g) * 0.25, Ci=torch.randn(s, L, N, generator=g) * 0.25)
        per_unit = 4 * (11 * C + 12 * N)
    gy = torch.randn(s, L, C, generator=g)
    return {"t": t, "gy": gy, "bytes": s * L * per_unit, "desc": f"{s}x{L}", "frac": s / S,
            "complex": complex_}


def _slru_cpu_step(sample):
    """The reference's CPU path (oracle port of the materialised SelectiveLRU path,
    models/selective_lru/selective_lru.py:242-276 with _selective_recurrence), fwd + bwd."""
    from oracle import selective_lru as oslru

    t = {k: v.clone().requires_grad_(True) for k, v in sample["t"].items()}
    if sample["complex"]:
        y = oslru.selective_lru_op(t["dnu"], t["dth"], t["a"], t["om"], t["B"], t["Bi"], t["C"],
                                   t["Ci"], t["x"], t["D"], input_gain="gamma")
    else:
        y = oslru.selective_lru_real_op(t["dnu"], t["a"], t["B"], t["C"], t["x"], t["D"], "mamba")
    (y * sample["gy"]).sum().backward()


# -------------------------------------------------------------------- MIMO layer workload
MIMO_F, MIMO_STATE, MIMO_HEADS, MIMO_RANK = 256, 128, 8, 4
MIMO_PASSES = (("time", 404, 321), ("freq", 1284, 101))


def _mimo_layer(device, seed):
    from semambaxlinoss_b200.selective_lru import SelectiveLRUMIMO

    torch.manual_seed(seed)
    m = SelectiveLRUMIMO(MIMO_F, MIMO_STATE, n_heads=MIMO_HEADS, rank=MIMO_RANK)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        # Token-level operands of the workload: dt = softplus(N(-2, 0.5)) per (token, head)
        # and b_t, c_t ~ N(0, 1/4) for x ~ N(0, 1/4); static B, C, D ~ N(0, 1/4).
        for lin in (m.dt_nu_proj, m.dt_theta_proj, m.b_dir, m.c_read, m.b_coef, m.c_coef):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) / 16.0)
        m.dt_nu_proj.bias.fill_(-2.0)
        for p in (m.B, m.C, m.D):
            p.copy_(torch.randn(p.shape, generator=g) * 0.5)
    return m.to(device)


class MimoPass:
    """One SelectiveLRUMIMO layer pass (bf16 input, fp32 state): forward builds the graph,
    backward runs it against a fixed upstream gradient. Algorithmic bytes per token are
    the layer's token I/O with the reference's 1616 projection columns (8 heads, rank 4):
    fwd x + projections (bf16) in, y (fp32) out = 4768; bwd x, projections (bf16), dy
    (fp32) in, dx, d projections (bf16) out = 8512. The static drive columns this
    package adds to the projection GEMM are an implementation choice and not counted."""

    fwd_bytes_per_unit = 4768
    bwd_bytes_per_unit = 8512
    kernels = ("mimo_layer_fwd_tc_kernel", "mimo_layer_bwd_tc_kernel")

    def __init__(self, layer, S, L, seed, device):
        g = torch.Generator(device=device).manual_seed(seed)
        self.layer = layer
        self.x = (torch.randn(S, L, MIMO_F, generator=g, device=device) * 0.5).to(torch.bfloat16)
        self.gy = torch.randn(S, L, MIMO_F, generator=g, device=device)
        self.units = S * L
        self.S, self.L = S, L
        self.inputs = [self.x, self.gy]
        self.xg = None
        self.y = None
        self.outputs = []

    def fwd(self, sh):
        self.xg = self.x.detach().requires_grad_(True)
        self.y = self.layer(self.xg)

    def bwd(self, sh):
        self.y.backward(self.gy)
        self.outputs = [self.y.detach(), self.xg.grad]


class MimoKernelPass:
    """The fused MIMO layer kernels alone (semx_mimo_layer_fwd / _bwd) on resident bf16
    token operands (x and the projection rows, 1872 columns including the static drive),
    for the kernel roofline of the MIMO workload. Bytes per token: fwd x + proj (bf16) in,
    y (fp32) out = 5280; bwd x, proj (bf16), dy (fp32) in, dx, dproj (bf16) out = 9536."""

    kernels = ("mimo_layer_fwd_tc_kernel", "mimo_layer_bwd_tc_kernel")

    def __init__(self, layer, S, L, seed, device):
        from semambaxlinoss_b200 import _lib

        H, Nh, Fh, R = MIMO_HEADS, MIMO_STATE // MIMO_HEADS, MIMO_F // MIMO_HEADS, MIMO_RANK
        self.lib, self._lib = _lib.load(), _lib
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        self.x = (torch.randn(S, L, MIMO_F, generator=g, device=device) * 0.5).to(bf)
        with torch.no_grad():
            W, b = layer._projection()
            self.proj = torch.nn.functional.linear(self.x, W.to(bf))
        self.dt_bias = b.detach().float().contiguous()
        self.d_dt_bias = torch.empty_like(self.dt_bias)
        P = self.proj.shape[-1]
        self.fwd_bytes_per_unit = 2 * MIMO_F + 2 * P + 4 * MIMO_F
        self.bwd_bytes_per_unit = (2 * MIMO_F + 2 * P + 4 * MIMO_F) + (2 * MIMO_F + 2 * P)
        self.y = torch.empty(S, L, MIMO_F, device=device)
        self.dy = torch.randn(S, L, MIMO_F, generator=g, device=device)
        self.dx = torch.empty_like(self.x)
        self.dproj = torch.empty_like(self.proj)
        self.params = [t.detach().float().contiguous() for t in (
            layer.A_log, layer.omega, layer.C, layer.D, layer.c_out)]
        self.grads = [torch.empty_like(t) for t in self.params]
        a = _lib.new_args(_lib.SemxMimoLayerArgs)
        a.input_gain, a.rank, a.rate_scale, a.bf16 = _lib.GAIN_CODES["gamma"], R, 1.0, 1
        a.S, a.L, a.H, a.Nh, a.Fh = S, L, H, Nh, Fh
        a.x, a.proj, a.y, a.dy, a.dx, a.dproj = [t.data_ptr() for t in (
            self.x, self.proj, self.y, self.dy, self.dx, self.dproj)]
        a.A_log, a.omega, a.C, a.D, a.c_out = [t.data_ptr() for t in self.params]
        a.dA_log, a.domega, a.dC, a.dD, a.dc_out = [t.data_ptr() for t in self.grads]
        a.dt_bias, a.d_dt_bias = self.dt_bias.data_ptr(), self.d_dt_bias.data_ptr()
        self.ckpt = _lib.empty_f32(self.lib.semx_mimo_layer_ckpt_bytes(ctypes.byref(a)), device)
        a.ckpt = self.ckpt.data_ptr()
        self.ws = _lib.empty_f32(self.lib.semx_mimo_layer_workspace_bytes(ctypes.byref(a)), device)
        a.workspace = self.ws.data_ptr()
        self.args = a
        self.units = S * L
        self.S, self.L = S, L

    def fwd(self, sh):
        self._lib.check("semx_mimo_layer_fwd", self.lib.semx_mimo_layer_fwd(ctypes.byref(self.args), sh))

    def bwd(self, sh):
        self._lib.check("semx_mimo_layer_bwd", self.lib.semx_mimo_layer_bwd(ctypes.byref(self.args), sh))


def _mimo_cpu_sample(frac, seed=0):
    from oracle import selective_lru as oslru  # noqa: F401  (import check before timing)

    layer = _mimo_layer("cpu", seed)
    params = {k: v.detach().clone() for k, v in layer.state_dict().items()}
    cfg = {"in_features": MIMO_F, "state_dim": MIMO_STATE, "n_heads": MIMO_HEADS, "rank": MIMO_RANK,
           "input_gain": "gamma"}
    g = torch.Generator().manual_seed(seed + 1)
    passes = []
    for _, S, L in MIMO_PASSES:
        s = max(1, int(round(S * frac)))
        x = (torch.randn(s, L, MIMO_F, generator=g) * 0.5).to(torch.bfloat16).float()
        passes.append((s, L, x, torch.randn(s, L, MIMO_F, generator=g)))
    return {"params": params, "cfg": cfg, "passes": passes, "frac": passes[0][0] / MIMO_PASSES[0][1],
            "bytes": sum(s * L * (4768 + 8512) for s, L, _, _ in passes),
            "desc": " + ".join(f"{s}x{L}" for s, L, _, _ in passes)}


def _mimo_cpu_step(sample):
    """The reference's CPU path for the layer (oracle port of SelectiveLRUMIMO's PyTorch
    path, models/selective_lru/selective_lru.py:488-587 with _selective_recurrence)."""
    from oracle import selective_lru as oslru

    for _, _, x, gy in sample["passes"]:
        p = {k: v.clone().requires_grad_(v.is_floating_point()) for k, v in sample["params"].items()}
        xx = x.clone().requires_grad_(True)
        y = oslru.selective_lru_mimo_forward(p, xx, sample["cfg"])
        (y * gy).sum().backward()


# ------------------------------------------------------------- operator-level workloads
OPS_S, OPS_L, OPS_H, OPS_NH, OPS_FH = 404, 321, 8, 16, 32


class CscanPass:
    """The plain complex diagonal scan (selective_scan_triton_real's replacement) over the
    MIMO workload's state, 404 sequences x 321 steps x 128 modes, fwd + bwd with an
    upstream gradient on h. Bytes per (sequence, step): fwd lam, Bu in + h out (complex
    fp32) = 24 N; bwd lam, h, dh in + dlam, dBu out = 40 N."""

    kernels = ("cscan_fwd_kernel", "cscan_bwd_kernel")

    def __init__(self, S, L, seed, device):
        N = OPS_H * OPS_NH
        g = torch.Generator(device=device).manual_seed(seed)
        mag = torch.rand(S, L, N, generator=g, device=device) * 0.98
        ph = torch.randn(S, L, N, generator=g, device=device)
        self.ins = [(mag * torch.cos(ph)).contiguous(), (mag * torch.sin(ph)).contiguous(),
                    torch.randn(S, L, N, generator=g, device=device),
                    torch.randn(S, L, N, generator=g, device=device)]
        self.gh = [torch.randn(S, L, N, generator=g, device=device) for _ in range(2)]
        self.fwd_bytes_per_unit = 24 * N
        self.bwd_bytes_per_unit = 40 * N
        self.units, self.S, self.L = S * L, S, L
        self.inputs = self.ins + self.gh
        self.outputs = []

    def fwd(self, sh):
        from semambaxlinoss_b200.selective_lru import selective_scan_triton_real

        self.leaf = [t.detach().requires_grad_(True) for t in self.ins]
        self.h = selective_scan_triton_real(*self.leaf)

    def bwd(self, sh):
        torch.autograd.backward(self.h, self.gh)
        self.outputs = [self.h[0].detach(), self.h[1].detach()] + [t.grad for t in self.leaf]


class MimoOpPass:
    """The fused MIMO scan + block-diagonal readout operator (fused_selective_lru_mimo's
    replacement) on given poles and drive, 8 heads x 16 modes, 32 channels per head,
    404 sequences x 321 steps, fwd + bwd with upstream gradients on y and h. Bytes per
    (sequence, step): fwd lam, Bu (complex fp32), x in + y, h out = 24 N + 8 Fd; bwd lam,
    h, dh, dy, x in + dlam, dBu, dx out = 40 N + 12 Fd."""

    kernels = ("mimo_fwd_kernel", "mimo_bwd_kernel")

    def __init__(self, S, L, seed, device):
        H, Nh, Fh = OPS_H, OPS_NH, OPS_FH
        N, Fd = H * Nh, H * Fh
        g = torch.Generator(device=device).manual_seed(seed)
        mag = torch.rand(S, L, N, generator=g, device=device) * 0.98
        ph = torch.randn(S, L, N, generator=g, device=device)
        self.ins = [(mag * torch.cos(ph)).contiguous(), (mag * torch.sin(ph)).contiguous(),
                    torch.randn(S, L, N, generator=g, device=device),
                    torch.randn(S, L, N, generator=g, device=device),
                    torch.randn(H, Fh, Nh, generator=g, device=device) * 0.3,
                    torch.randn(H, Fh, Nh, generator=g, device=device) * 0.3,
                    torch.randn(S, L, Fd, generator=g, device=device),
                    torch.randn(Fd, generator=g, device=device)]
        self.gy = torch.randn(S, L, Fd, generator=g, device=device)
        self.gh = [torch.randn(S, L, N, generator=g, device=device) for _ in range(2)]
        self.fwd_bytes_per_unit = 24 * N + 8 * Fd
        self.bwd_bytes_per_unit = 40 * N + 12 * Fd
        self.units, self.S, self.L = S * L, S, L
        self.inputs = self.ins[:4] + self.ins[6:7] + [self.gy] + self.gh
        self.outputs = []

    def fwd(self, sh):
        from semambaxlinoss_b200.selective_lru import fused_selective_lru_mimo

        self.leaf = [t.detach().requires_grad_(True) for t in self.ins]
        self.out = fused_selective_lru_mimo(*self.leaf, OPS_H, OPS_NH, OPS_FH)

    def bwd(self, sh):
        torch.autograd.backward(self.out, [self.gy] + self.gh)
        self.outputs = [self.out[0].detach()] + [self.leaf[i].grad for i in (0, 1, 2, 3, 6)]


def _ops_cpu_sample(frac, seed=0):
    N, Fd = OPS_H * OPS_NH, OPS_H * OPS_FH
    g = torch.Generator().manual_seed(seed)
    s = max(1, int(round(OPS_S * frac)))
    L = OPS_L
    mag = torch.rand(s, L, N, generator=g) * 0.98
    ph = torch.randn(s, L, N, generator=g)
    t = {"lr": mag * torch.cos(ph), "li": mag * torch.sin(ph), "br": torch.randn(s, L, N, generator=g),
         "bi": torch.randn(s, L, N, generator=g), "cr": torch.randn(OPS_H, OPS_FH, OPS_NH, generator=g) * 0.3,
         "ci": torch.randn(OPS_H, OPS_FH, OPS_NH, generator=g) * 0.3, "x": torch.randn(s, L, Fd, generator=g),
         "D": torch.randn(Fd, generator=g)}
    gy = torch.randn(s, L, Fd, generator=g)
    gh = (torch.randn(s, L, N, generator=g), torch.randn(s, L, N, generator=g))
    return {"t": t, "gy": gy, "gh": gh, "desc": f"{s}x{L} (both operators)",
            "bytes": s * L * ((24 + 40) * N + (24 * N + 8 * Fd) + (40 * N + 12 * Fd))}


def _ops_cpu_step(sample):
    """The reference's PyTorch equivalents (oracle port of the sequential complex scan and
    the MIMO scan + readout, models/selective_lru/selective_lru.py:550-574, 590-599), fwd + bwd."""
    from oracle import selective_lru as oslru

    t = {k: v.clone().requires_grad_(True) for k, v in sample["t"].items()}
    h = oslru.selective_recurrence(torch.complex(t["lr"], t["li"]), torch.complex(t["br"], t["bi"]))
    gh = sample["gh"]
    (h.real * gh[0] + h.imag * gh[1]).sum().backward()
    t = {k: v.clone().requires_grad_(True) for k, v in sample["t"].items()}
    y, hr, hi = oslru.mimo_scan_readout(t["lr"], t["li"], t["br"], t["bi"], t["cr"], t["ci"], t["x"], t["D"],
                                        OPS_H, OPS_NH, OPS_FH)
    ((y * sample["gy"]).sum() + (hr * gh[0] + hi * gh[1]).sum()).backward()


# ---------------------------------------------------- layer surround kernels (generator)
# One generator time-axis layer's token rows (16 utterances x 321 frames x 100 bins), its
# d_inner, dt_rank and the frequency-axis LinOSS state.
SUR_ROWS, SUR_C, SUR_R, SUR_P = 16 * 321 * 100, 256, 4, 16


class StepProjPass:
    """The SelectiveLRU step projections (semx_step_proj: delta_nu = softplus(dt_nu_up(dnu_r)),
    delta_theta = dt_theta_up(dth_r)) on bf16 projection rows of 2r + 64 columns, fwd + bwd
    with upstream gradients on both. Bytes per row: fwd z in (2r bf16) + 2 C fp32 out =
    8 C + 4 r; bwd 2 C fp32 in + z in + dz out = 8 C + 8 r."""

    kernels = ("step_proj_fwd_kernel", "step_proj_bwd_kernel")

    def __init__(self, rows, seed, device):
        C, r = SUR_C, SUR_R
        g = torch.Generator(device=device).manual_seed(seed)
        self.proj = torch.randn(rows, 2 * r + 64, generator=g, device=device).to(torch.bfloat16)
        self.w = [torch.randn(C, r, generator=g, device=device) * 0.5, torch.randn(C, generator=g, device=device) - 1.0,
                  torch.randn(C, r, generator=g, device=device) * 0.5, torch.randn(C, generator=g, device=device)]
        self.g = [torch.randn(rows, C, generator=g, device=device) for _ in range(2)]
        self.fwd_bytes_per_unit = 8 * C + 4 * r
        self.bwd_bytes_per_unit = 8 * C + 8 * r
        self.units, self.S, self.L = rows, rows, 1
        self.inputs = [self.proj] + self.g
        self.outputs = []

    def fwd(self, sh):
        from semambaxlinoss_b200.selective_lru.selective_lru import _StepProjections

        r = SUR_R
        self.leaf = [self.proj.detach().requires_grad_(True)] + [t.detach().requires_grad_(True) for t in self.w]
        self.out = _StepProjections.apply(self.leaf[0][:, :r], self.leaf[0][:, r:2 * r], *self.leaf[1:], 1.0)

    def bwd(self, sh):
        torch.autograd.backward(self.out, self.g)
        self.outputs = [self.out[0].detach(), self.out[1].detach(), self.leaf[0].grad]


class ReadoutPass:
    """The LinOSS readout and D skip (semx_linoss_readout: y = Re(C y2) + D x), fwd + bwd.
    Bytes per row: fwd x in, y out (fp32) + y2 in = 8 H + 8 P; bwd dy, x in, dx out + y2
    in = 12 H + 8 P (the fused kernel's own; the bwd time also holds the dy2 = dy conj(C)
    GEMM, which reads dy once more)."""

    kernels = ("linoss_readout_fwd_kernel", "linoss_readout_bwd_kernel")

    def __init__(self, rows, seed, device):
        H, P = SUR_C, SUR_P
        g = torch.Generator(device=device).manual_seed(seed)
        self.y2 = torch.randn(rows, P, dtype=torch.complex64, generator=g, device=device)
        self.x = torch.randn(rows, H, generator=g, device=device)
        self.C = torch.randn(H, P, 2, generator=g, device=device) * 0.3
        self.D = torch.randn(H, generator=g, device=device)
        self.gy = torch.randn(rows, H, generator=g, device=device)
        self.fwd_bytes_per_unit = 8 * H + 8 * P
        self.bwd_bytes_per_unit = 12 * H + 8 * P
        self.units, self.S, self.L = rows, rows, 1
        self.inputs = [self.y2, self.x, self.gy]
        self.outputs = []

    def fwd(self, sh):
        from semambaxlinoss_b200.linoss.linoss import _Readout

        self.leaf = [t.detach().requires_grad_(True) for t in (self.y2, self.x, self.C, self.D)]
        self.out = _Readout.apply(*self.leaf)

    def bwd(self, sh):
        self.out.backward(self.gy)
        self.outputs = [self.out.detach(), self.leaf[0].grad, self.leaf[1].grad]


def _surround_cpu_sample(frac, seed=0):
    g = torch.Generator().manual_seed(seed)
    rows = max(1, int(round(SUR_ROWS * frac)))
    C, r, P = SUR_C, SUR_R, SUR_P
    t = {"z": torch.randn(rows, 2 * r, generator=g), "wn": torch.randn(C, r, generator=g) * 0.5,
         "bn": torch.randn(C, generator=g) - 1.0, "wt": torch.randn(C, r, generator=g) * 0.5,
         "bt": torch.randn(C, generator=g), "y2": torch.randn(rows, P, dtype=torch.complex64, generator=g),
         "x": torch.randn(rows, C, generator=g), "C": torch.randn(C, P, 2, generator=g) * 0.3,
         "D": torch.randn(C, generator=g)}
    gs = [torch.randn(rows, C, generator=g) for _ in range(3)]
    return {"t": t, "g": gs, "desc": f"{rows} rows (both operations)",
            "bytes": rows * (8 * C + 4 * r + 8 * C + 8 * r + 8 * C + 8 * P + 12 * C + 8 * P)}


def _surround_cpu_step(sample):
    """The reference's PyTorch expressions (models/selective_lru/selective_lru.py:216-220,
    models/linoss/linoss.py:118-120), fwd + bwd."""
    import torch.nn.functional as F

    t = {k: v.clone().requires_grad_(True) for k, v in sample["t"].items()}
    r = SUR_R
    dnu = F.softplus(F.linear(t["z"][:, :r], t["wn"], t["bn"]))
    dth = F.linear(t["z"][:, r:], t["wt"], t["bt"])
    Cc = torch.complex(t["C"][..., 0], t["C"][..., 1])
    y = torch.einsum("fn,bn->bf", Cc, t["y2"]).real + t["x"] * t["D"]
    g = sample["g"]
    ((dnu * g[0]).sum() + (dth * g[1]).sum() + (y * g[2]).sum()).backward()


# ------------------------------------------------------------------------ scan workloads
WORKLOADS = {
    "linoss": {
        "config": "1",
        "metric": "LinOSS-IMEX scan fwd+bwd, algorithmic HBM GB/s (time 404x321 + freq 1284x101, P=256)",
        "describe": "LinOSS-IMEX scan fwd+bwd at the scan boundary, time 404x321 + freq 1284x101, "
                    "P=256 oscillators, H=64",
        "data": "synthetic, seeded: A = relu(N(0,1)), dt = sigmoid(N(0,1)), B ~ N(0, 1/sqrt(64)), u ~ N(0,1)",
        "dtype": "f32",
        "chunk": 64, "sample_frac": 1.0 / 32,
        "l2": "no flush: every operand is 265 MB, larger than the 126 MB L2",
        "cpu_sample": _linoss_cpu_sample, "cpu_step": _linoss_cpu_step,
    },
    "slru": {
        "config": "0",
        "metric": "Selective-LRU real diagonal scan fwd+bwd, algorithmic HBM GB/s (404x321, C=256, N=16)",
        "describe": "real selective-LRU scan (Mamba gain) fwd+bwd, 404 sequences x 321 steps, "
                    "C=256 channels, N=16 modes",
        "data": "synthetic, seeded: x ~ N(0,1), dt = softplus(N(-2,0.5)), a ~ U(1,16), B, C ~ N(0,1/16)",
        "dtype": "f32",
        "chunk": 16, "sample_frac": 1.0 / 404,
        "l2": "no flush: x, dt, dy, y and each gradient are 133 MB, larger than the 126 MB L2",
        "cpu_sample": _slru_cpu_sample, "cpu_step": _slru_cpu_step,
    },
    "mimo": {
        "config": "2",
        "metric": "Selective-LRU MIMO layer fwd+bwd, algorithmic HBM GB/s (time 404x321 + freq 1284x101, "
                  "8 heads x 32, state 128, rank 4)",
        "describe": "SelectiveLRUMIMO layer fwd+bwd (bf16 input, fp32 state), 256 features = 8 heads x 32, "
                    "state 128, rank 4, time 404x321 + freq 1284x101",
        "data": "synthetic, seeded: x ~ N(0,1/4) bf16, dt = softplus(N(-2,0.5)), b_t, c_t, B, C, D ~ N(0,1/4)",
        "dtype": "bf16 in / f32 state",
        "chunk": 0, "sample_frac": 0.01,
        "l2": "no flush: the layer's activations per pass are GBs, far beyond the 126 MB L2",
        "cpu_sample": _mimo_cpu_sample, "cpu_step": _mimo_cpu_step,
    },
}
WORKLOADS["ops"] = {
    "config": "ops",
    "metric": "Selective-LRU MIMO operator + plain complex scan fwd+bwd, algorithmic HBM GB/s "
              "(404x321, 8 heads x 16 modes, 32 channels per head)",
    "describe": "fused_selective_lru_mimo (scan + block-diagonal readout + D skip on given poles and drive) "
                "and selective_scan_triton_real (plain complex diagonal scan), 404 sequences x 321 steps, "
                "128 modes, 256 channels",
    "data": "synthetic, seeded: |lam| ~ U(0, 0.98), phase ~ N(0,1), Bu, x, D ~ N(0,1), C ~ N(0, 0.09)",
    "dtype": "f32",
    "chunk": 0, "sample_frac": 2.0 / 404,
    "l2": "no flush: every (404, 321, 128) operand is 66 MB and (404, 321, 256) 133 MB; a step moves "
          "6.7 GB, far beyond the 126 MB L2",
    "cpu_sample": _ops_cpu_sample, "cpu_step": _ops_cpu_step,
}
WORKLOADS["surround"] = {
    "config": "surround",
    "metric": "SelectiveLRU step projections + LinOSS readout fwd+bwd, algorithmic HBM GB/s "
              "(generator layer shape: 513600 token rows, C=256, rank 4, P=16)",
    "describe": "the fused step projections (bf16 z, rank 4) and the fused LinOSS readout + D skip (P=16) "
                "of one generator layer, 513600 token rows x 256 channels, fwd + bwd",
    "data": "synthetic, seeded: z, x, W ~ N(0, 1/4 .. 1), y2 ~ CN(0, 1), C ~ N(0, 0.09)",
    "dtype": "bf16 z / f32",
    "chunk": 0, "sample_frac": 2048.0 / SUR_ROWS,
    "l2": "no flush: every (513600, 256) fp32 operand is 526 MB, far beyond the 126 MB L2",
    "cpu_sample": _surround_cpu_sample, "cpu_step": _surround_cpu_step,
}
# The default workload: configs 0, 1 and 2 in one step, in this order.
SCAN_SET = ("slru", "linoss", "mimo")


def _scans_cpu_sample(frac=None):
    """One fixed sample per config (each workload's own `sample_frac`)."""
    parts = {k: WORKLOADS[k]["cpu_sample"](WORKLOADS[k]["sample_frac"]) for k in SCAN_SET}
    return {"parts": parts, "bytes": sum(p["bytes"] for p in parts.values()),
            "desc": "; ".join(f"config {WORKLOADS[k]['config']}: {p['desc']}" for k, p in parts.items())}


def _scans_cpu_step(sample):
    for k, part in sample["parts"].items():
        WORKLOADS[k]["cpu_step"](part)


WORKLOADS["scans"] = {
    "config": "0+1+2",
    "metric": "scan fwd+bwd, algorithmic HBM GB/s over BASELINE configs 0-2 (selective-LRU SISO real 404x321 "
              "C=256 N=16; LinOSS-IMEX P=256 time 404x321 + freq 1284x101; SelectiveLRUMIMO 8x32 heads, "
              "state 128, rank 4, bf16, time 404x321 + freq 1284x101)",
    "describe": "configs 0, 1 and 2 fwd+bwd in one step: " + "; ".join(
        f"config {WORKLOADS[k]['config']}: {WORKLOADS[k]['describe']}" for k in SCAN_SET),
    "data": "synthetic, seeded: " + "; ".join(
        f"config {WORKLOADS[k]['config']}: {WORKLOADS[k]['data'].split(': ', 1)[1]}" for k in SCAN_SET),
    "dtype": "f32 (configs 0, 1); bf16 in / f32 state (config 2)",
    "chunk": None, "sample_frac": None,
    "l2": "no flush: every operand of every pass is larger than the 126 MB L2 (133 MB - GBs)",
    "cpu_sample": _scans_cpu_sample, "cpu_step": _scans_cpu_step,
}


def workload_spec(args):
    """The workload table entry, adapted to the SISO variant options."""
    import functools

    spec = dict(WORKLOADS[args.workload])
    if args.workload == "slru" and (args.slru_complex or args.sequences):
        S = args.sequences or SLRU_S
        kind = "complex selective-LRU scan (gamma gain)" if args.slru_complex else spec["describe"].split(" fwd")[0]
        spec["metric"] = (f"Selective-LRU {'complex' if args.slru_complex else 'real'} diagonal scan fwd+bwd, "
                          f"algorithmic HBM GB/s ({S}x321, C=256, N=16)")
        spec["describe"] = f"{kind} fwd+bwd, {S} sequences x 321 steps, C=256 channels, N=16 modes"
        if args.slru_complex:
            spec["data"] += ", dth ~ N(0, 0.01), omega ~ N(0,1)"
        spec["cpu_sample"] = functools.partial(_slru_cpu_sample, complex_=args.slru_complex, S=S)
        spec["sample_frac"] = 1.0 / S
    return spec


def _shard(S, rank, world):
    """Rank `rank`'s contiguous slice [floor(r S / W), floor((r + 1) S / W)) of S sequences."""
    return (rank + 1) * S // world - rank * S // world


def _make_passes(name, rank, device, chunk, args, world=1, sharded=False):
    """The passes of one step. `sharded`: each pass holds this rank's contiguous slice of the
    named shape's sequences (strong scaling); otherwise the full named shape (every rank
    its own batch: weak scaling)."""
    if name == "scans":
        return [p for sub in SCAN_SET for p in _make_passes(sub, rank, device, None, args, world, sharded)]
    chunk = chunk or WORKLOADS[name]["chunk"]
    size = (lambda S: _shard(S, rank, world)) if sharded else (lambda S: S)
    if name == "ops":
        ps = [MimoOpPass(size(OPS_S), OPS_L, seed=1000 * rank, device=device),
              CscanPass(size(OPS_S), OPS_L, seed=1000 * rank + 1, device=device)]
        ps[0].workload, ps[1].workload = "ops", "ops_cscan"
        for p in ps:
            p.chunk = chunk
        return ps
    if name == "surround":
        ps = [StepProjPass(size(SUR_ROWS), seed=1000 * rank, device=device),
              ReadoutPass(size(SUR_ROWS), seed=1000 * rank + 1, device=device)]
        ps[0].workload, ps[1].workload = "surround_step", "surround_readout"
        for p in ps:
            p.chunk = chunk
        return ps
    if name == "linoss":
        ps = [LinossPass(size(S), L, seed=1000 * rank + i, device=device, chunk=chunk)
              for i, (_, S, L) in enumerate(LIN_PASSES)]
    elif name == "slru":
        ps = [SlruPass(size(args.sequences or SLRU_S), SLRU_L, seed=1000 * rank, device=device, chunk=chunk,
                       complex_=args.slru_complex)]
    else:
        layer = _mimo_layer(device, seed=7)
        ps = [MimoPass(layer, size(S), L, seed=1000 * rank + i, device=device)
              for i, (_, S, L) in enumerate(MIMO_PASSES)]
    for p in ps:
        p.workload = name
        p.chunk = chunk
    return ps


def _kernel_passes(passes, device):
    """The passes whose kernels carry the roofline: the scan passes themselves, and for the
    MIMO layer the fused layer kernels alone on resident bf16 operands (MimoKernelPass)."""
    out = []
    for i, p in enumerate(passes):
        if isinstance(p, MimoPass):
            k = MimoKernelPass(p.layer, p.S, p.L, seed=5000 + i, device=device)
            k.workload = p.workload
            out.append(k)
        else:
            out.append(p)
    return out


def _time_passes(passes, steps, stream):
    """Runs `steps` fwd+bwd sweeps over `passes`; returns (start, end, per-pass events)."""
    sh = stream.cuda_stream
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in passes] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for k in range(steps):
        for i, p in enumerate(passes):
            ev[k][i][0].record(stream)
            p.fwd(sh)
            ev[k][i][1].record(stream)
            p.bwd(sh)
            ev[k][i][2].record(stream)
    end.record(stream)
    return start, end, ev


def _per_pass_ms(passes, ev, steps):
    return [(p, statistics.mean(ev[k][i][0].elapsed_time(ev[k][i][1]) for k in range(steps)),
             statistics.mean(ev[k][i][1].elapsed_time(ev[k][i][2]) for k in range(steps)))
            for i, p in enumerate(passes)]


def _cfg_of(workload):
    """The BASELINE config a pass group belongs to (its workload name where it has none)."""
    return WORKLOADS[workload]["config"] if workload in WORKLOADS else workload


def _traffic_tag(p):
    if p.workload == "slru":
        return "slru complex" if getattr(p, "complex_", False) else "slru real"
    return p.workload


def _kernel_table(kpasses, peak):
    """Per workload and direction: kernel, ms per step (all its passes), algorithmic bytes,
    achieved GB/s, fraction of the peak, ncu traffic of one launch of its first pass."""
    rows = []
    for w in dict.fromkeys(p.workload for p, _, _ in kpasses):
        group = [(p, f, b) for p, f, b in kpasses if p.workload == w]
        for d, name in ((1, "fwd"), (2, "bwd")):
            p0 = group[0][0]
            kernel = p0.kernels[d - 1]
            ms = sum(x[d] for x in group)
            by = sum(p.units * (p.fwd_bytes_per_unit if d == 1 else p.bwd_bytes_per_unit) for p, _, _ in group)
            gbs = by / (ms * 1e-3) / 1e9
            traffic, source = profiled_traffic(kernel, _traffic_tag(p0), p0.units)
            rows.append({"config": _cfg_of(w), "workload": w, "dir": name, "kernel": kernel,
                         "ms": round(ms, 4), "bytes": by, "achieved": round(gbs, 1),
                         "frac": round(gbs / peak, 4), "traffic": traffic, "traffic_source": source,
                         "algorithmic_bytes_first_launch": p0.units * (
                             p0.fwd_bytes_per_unit if d == 1 else p0.bwd_bytes_per_unit)})
    return rows


def _timed_scan(passes, args, device, stream, world, steps):
    """Warm-up, then `steps` timed steps between barriers; returns (ms per step as the max
    over ranks, per-pass (pass, fwd ms, bwd ms), kernel launches)."""
    from semambaxlinoss_b200 import _lib

    sh = stream.cuda_stream
    for _ in range(max(args.warmup, 3)):
        for p in passes:
            p.fwd(sh)
            p.bwd(sh)
    _barrier(world, device)
    n0 = _lib.launch_count()
    start, end, ev = _time_passes(passes, steps, stream)
    _barrier(world, device)
    launches = _lib.launch_count() - n0
    ms = _max_over_ranks(start.elapsed_time(end), world, device) / steps
    return ms, _per_pass_ms(passes, ev, steps), launches


def run_scan(args, rank, local_rank, world):
    spec = workload_spec(args)
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _init_dist(world, device)
    passes = _make_passes(args.workload, rank, device, args.chunk, args)
    stream = torch.cuda.current_stream(device)
    sh = stream.cuda_stream
    step_bytes = sum(p.units * (p.fwd_bytes_per_unit + p.bwd_bytes_per_unit) for p in passes)

    for _ in range(max(args.warmup, 3)):
        for p in passes:
            p.fwd(sh)
            p.bwd(sh)
    clocks = ClockSampler(_device_uuid(device), args.clocks_log if rank == 0 else None)
    # Keep the GPU busy ~1.5 s before timing so the clock samples see it under load.
    soak_t0 = time.time()
    torch.cuda.synchronize(device)
    while not args.no_soak and time.time() - soak_t0 < 1.5:
        for _ in range(5):
            for p in passes:
                p.fwd(sh)
                p.bwd(sh)
        torch.cuda.synchronize(device)

    ms_per_step, per_pass, launches = _timed_scan(passes, args, device, stream, world, args.steps)
    t_wall1 = time.time()
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9

    # Kernel rooflines (the MIMO layer's fused kernels timed alone).
    kp = _kernel_passes(passes, device)
    if any(k is not p for k, p in zip(kp, passes)):
        kn = max(3, args.steps // 2)
        _, kpasses, _ = _timed_scan(kp, args, device, stream, 1, kn)
    else:
        kpasses = per_pass
    del kp

    e2e = None if args.no_e2e else run_scan_e2e(
        passes, args, device, stream, step_bytes, world,
        lambda: _make_passes(args.workload, rank, device, args.chunk, args))

    # Strong scaling over the named shapes: rank r scans its contiguous slice of every pass.
    sharded = None
    if world > 1 and not args.no_sharded:
        sp = _make_passes(args.workload, rank, device, args.chunk, args, world, sharded=True)
        full_bytes = step_bytes  # the named shapes' bytes (every rank's full batch is one named set)
        ms_sh, _, _ = _timed_scan(sp, args, device, stream, world, args.steps)
        sharded = {"value": round(full_bytes / (ms_sh * 1e-3) / 1e9, 2), "unit": "GB/s",
                   "ms_per_step": round(ms_sh, 4), "scaling": "strong",
                   "sequences_rank0": [p.S for p in sp] if rank == 0 else None,
                   "note": "the named shapes split into contiguous per-rank sequence slices "
                           "[floor(r S / W), floor((r+1) S / W)); time = max over ranks"}
        del sp
    gen = inf = None
    if args.workload == "scans" and not args.no_generator:
        gen = measure_generator(args, rank, local_rank, world, device, args.gen_steps, clocks=False)
        torch.cuda.empty_cache()
    if args.workload == "scans" and not args.no_inference:
        inf = measure_inference(args, rank, local_rank, world, device, 1, clocks=False)
    clocks.stop()
    _finish_dist(world)
    if rank != 0:
        return

    peak, peak_kind = load_peaks()
    table = _kernel_table(kpasses, peak)
    dom = max(table, key=lambda r: r["ms"])
    slow = min(table, key=lambda r: r["frac"])
    configs = {}
    for w in dict.fromkeys(p.workload for p in passes):
        group = [(p, f, b) for p, f, b in per_pass if p.workload == w]
        by = sum(p.units * (p.fwd_bytes_per_unit + p.bwd_bytes_per_unit) for p, _, _ in group)
        ms = sum(f + b for _, f, b in group)
        configs[_cfg_of(w)] = {
            "workload": w, "fwd_ms": round(sum(f for _, f, _ in group), 4),
            "bwd_ms": round(sum(b for _, _, b in group), 4), "bytes": by,
            "GB/s": round(by / (ms * 1e-3) / 1e9, 1), "frac": round(by / (ms * 1e-3) / 1e9 / peak, 4),
            "passes": [{"sequences": p.S, "steps": p.L} for p, _, _ in group],
            "chunk": group[0][0].chunk or None}
    out = {
        "metric": spec["metric"],
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": spec["dtype"],
        "data": spec["data"],
        "config": {
            "workload": spec["describe"],
            "bytes_per_step": step_bytes,
            "l2": spec["l2"],
            "parallelism": f"weak dp{world}: the global batch is {world}x the named shapes, rank r scans "
                           "its contiguous slice r (one named set), no collective",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": dom["kernel"],
            "config": dom["config"],
            "achieved": dom["achieved"],
            "peak": peak,
            "unit": "GB/s",
            "frac": dom["frac"],
            "peak_kind": peak_kind,
            "traffic": dom["traffic"],
            "traffic_source": dom["traffic_source"],
            "algorithmic_bytes_first_launch": dom["algorithmic_bytes_first_launch"],
            "slowest_frac_kernel": {k: slow[k] for k in ("config", "kernel", "dir", "achieved", "frac")},
            "note": "the dominant kernel = the largest share of the step's kernel time; achieved = "
                    "algorithmic bytes / CUDA-event time of the entry point (includes its small reduction "
                    "launches); traffic = ncu DRAM bytes of one launch of the first pass, recorded in the "
                    "named profile (not measured in this run)",
        },
        "kernels": table,
        "configs": configs,
        "hbm_frac_of_8tbs": round(value / world / 8000.0, 4),
        "gpu_launches": launches,
        "clocks": clocks.summary(soak_t0, t_wall1),
        "e2e": e2e,
    }
    if sharded is not None:
        out["sharded"] = sharded
    if gen is not None:
        out["generator"] = gen
    if inf is not None:
        out["inference"] = inf
    if any(p.workload == "mimo" for p in passes):
        out["gpu_launches_note"] = ("libsemx kernels only; the MIMO layer's token projections (one GEMM "
                                    "forward, two backward) run as cuBLAS kernels")
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(spec, repeats=3)
    print(json.dumps(out), flush=True)


def run_scan_e2e(passes, args, device, stream, step_bytes, world, make_set):
    """The same metric through the public entry points with host buffers: every step copies
    the pass inputs from pinned host memory, runs forward and backward, and copies the
    outputs and gradients back to pinned host memory, all inside the timed region. Steps
    alternate between two device buffer sets, with the host-to-device copies on one
    stream and the device-to-host copies on another, ordered by events, so the two copy
    directions and the kernels of neighbouring steps overlap."""
    sh = stream.cuda_stream
    sets = [passes, make_set()]
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)
    host_in = [[t.detach().cpu().pin_memory() for t in p.inputs] for p in passes]
    for ps in sets:  # outputs exist after one step
        for p in ps:
            p.fwd(sh)
            p.bwd(sh)
    torch.cuda.synchronize(device)
    host_out = [[[torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in p.outputs] for p in ps]
                for ps in sets]
    h2d = sum(t.numel() * t.element_size() for hs in host_in for t in hs)
    d2h = sum(t.numel() * t.element_size() for hs in host_out[0] for t in hs)
    ev = [{k: torch.cuda.Event() for k in ("in", "comp", "out")} for _ in sets]

    def e2e_step(k):
        X = k % 2
        ps, e = sets[X], ev[X]
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(e["comp"])  # the set's previous kernels have read their inputs
            for p, hi in zip(ps, host_in):
                for d, h in zip(p.inputs, hi):
                    d.copy_(h, non_blocking=True)
            e["in"].record(h2d_s)
        stream.wait_event(e["in"])
        stream.wait_event(e["out"])  # the set's previous outputs have been copied out
        for p in ps:
            p.fwd(sh)
            p.bwd(sh)
        e["comp"].record(stream)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(e["comp"])
            for p, ho in zip(ps, host_out[X]):
                for d, h in zip(p.outputs, ho):
                    d.record_stream(d2h_s)
                    h.copy_(d, non_blocking=True)
            e["out"].record(d2h_s)

    for k in range(2):
        e2e_step(k)
    _barrier(world, device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    h2d_s.wait_event(start)
    for k in range(args.e2e_steps):
        e2e_step(k)
    for e in ev:
        stream.wait_event(e["out"])
    end.record(stream)
    torch.cuda.synchronize(device)
    ms = _max_over_ranks(start.elapsed_time(end), world, device) / args.e2e_steps
    del sets[1]
    return {"value": round(world * step_bytes / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "ms_per_step": round(ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "public entry points with pinned host buffers; copies in and out on two "
                    "streams overlapping the kernels (two device buffer sets)"}


# ----------------------------------------------------------------------------- CPU legs
def cpu_baseline(spec, repeats=3, frac=None):
    torch.set_num_threads(os.cpu_count())
    sample = spec["cpu_sample"](frac if frac is not None else spec["sample_frac"])
    spec["cpu_step"](sample)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        spec["cpu_step"](sample)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(sample["bytes"] / t / 1e9, 5), "unit": "GB/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"fixed sample ({sample['desc']}), fwd+bwd float32, median of {repeats}",
            "seconds": round(t, 3)}


def run_reference(args, rank):
    if rank != 0:
        return
    if args.workload not in WORKLOADS:
        print(json.dumps({"impl": "reference", "unavailable": "the reference generator needs the "
                          "third-party mamba_ssm package, which the reference does not ship"}))
        return
    spec = workload_spec(args)
    torch.set_num_threads(os.cpu_count())
    # A fixed, stated sample per config (the same one the GPU arm's cpu_baseline times), so
    # the ratio to the GPU arm does not depend on this host's speed.
    sample = spec["cpu_sample"](args.ref_sample_frac if args.ref_sample_frac is not None else spec["sample_frac"])
    for _ in range(args.warmup):
        spec["cpu_step"](sample)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        spec["cpu_step"](sample)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = sample["bytes"] / (ms * 1e-3) / 1e9
    print(json.dumps({
        "impl": "reference",
        "metric": spec["metric"],
        "value": round(value, 5),
        "unit": "GB/s",
        "n_gpus": 0,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": spec["dtype"],
        "data": spec["data"],
        "config": {"workload": spec["describe"], "sample": sample["desc"]},
        "cpu_baseline": {"value": round(value, 5), "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"fixed sample per step ({sample['desc']}), fwd+bwd float32"},
        "e2e": {"value": round(value, 5), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------- generator workloads
def measure_generator(args, rank, local_rank, world, device, steps, clocks=True):
    """SEMamba generator training step (forward + generator losses + backward + DDP
    gradient all-reduce + AdamW), bf16 autocast around fp32 scans, `--batch` two-second
    utterances per GPU, on an initialised process group when world > 1. Returns, on rank 0,
    the measurement as a dict (frames/s over all GPUs, device time = max over ranks, an
    end-to-end figure with the audio copied in from pinned host memory and the loss read
    back every step); None on other ranks."""
    from semambaxlinoss_b200 import _lib
    from semambaxlinoss_b200.generator import SEMamba, config3_cfg, generator_loss, mag_phase_stft

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
    sampler = ClockSampler(_device_uuid(device), args.clocks_log if rank == 0 else None) if clocks else None
    soak_t0 = time.time()
    _barrier(world, device)
    n0 = _lib.launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    # cudaProfilerStart / Stop bracket the timed steps, so that a profiler run with
    # --profile-from-start off captures exactly their launches, from every host thread
    # (autograd runs the backward on its own thread).
    torch.cuda.profiler.start()
    for _ in range(steps):
        loss = step(clean_d, noisy_d)
    torch.cuda.profiler.stop()
    e.record(stream)
    _barrier(world, device)
    launches = _lib.launch_count() - n0
    t_end = time.time()
    ms = _max_over_ranks(s.elapsed_time(e), world, device) / steps
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
    if sampler is not None:
        sampler.stop()
    del model, opt
    if rank != 0:
        return None
    out = {
        "metric": "SEMamba generator training step, frames/s (2 s utterances, batch 16 per GPU)",
        "value": round(world * B * frames / (ms * 1e-3), 1), "unit": "frames/s", "n_gpus": world,
        "steps": steps, "ms_per_step": round(ms, 3), "scaling": "weak",
        "dtype": "bf16 autocast, fp32 scans",
        "data": "synthetic (clean ~ N(0, 0.1), noise ~ N(0, 0.05), seeded per rank), random-init weights",
        "config": {"workload": "generator fwd + losses + bwd + AdamW, 4 TF-blocks (time: selective-LRU "
                               "d_inner 256 N 16; freq: damped-IMEX LinOSS P 16), hid 64",
                   "global_batch": world * B, "seq_len": frames, "parallelism": f"ddp{world}",
                   "parameters": n_params,
                   "l2": "no flush: activations per step are tens of GB, far beyond the 126 MB L2"},
        "e2e": {"value": round(world * B * frames / (ms_e2e * 1e-3), 1), "unit": "frames/s",
                "ms_per_step": round(ms_e2e, 3), "h2d_bytes_per_step": 2 * B * seg * 4,
                "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "gpu_launches_note": "libsemx kernels only (scans, their reductions, mixer and norm kernels); "
                             "convolutions, GEMMs and the optimizer run as torch/cuDNN/cuBLAS kernels",
    }
    if sampler is not None:
        out["clocks"] = sampler.summary(soak_t0, t_end)
    return out


def run_generator(args, rank, local_rank, world):
    """The generator training step as the bench line (`--workload generator`)."""
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _init_dist(world, device)
    out = measure_generator(args, rank, local_rank, world, device, args.steps)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if out is None:
        return
    out.update(warmup=args.warmup, higher_is_better=True, vs_baseline=None)
    print(json.dumps(out), flush=True)


def measure_inference(args, rank, local_rank, world, device, steps, clocks=True):
    """64 sixty-second utterances (T = 9601 frames) enhanced end to end (STFT -> generator
    -> iSTFT) under no_grad with bf16 autocast, sharded over the GPUs (rank r takes
    utterances r, r + W, ...), `--micro-batch` utterances per forward, the time scans
    streamed in `--stream-chunk`-frame pieces. Every step copies its audio in from pinned
    host memory and the enhanced audio out. Returns, on rank 0, the measurement (frames/s
    over all GPUs, device time = max over ranks); None on other ranks."""
    from semambaxlinoss_b200 import _lib
    from semambaxlinoss_b200.generator import SEMamba, config3_cfg, mag_phase_istft, mag_phase_stft

    cfg = config3_cfg()
    sc, cf = cfg["stft_cfg"], cfg["model_cfg"]["compress_factor"]
    torch.manual_seed(1234)
    model = SEMamba(cfg).to(device).eval()
    if args.stream_chunk > 0:
        from semambaxlinoss_b200.selective_lru import SelectiveLRU

        for m in model.modules():
            if isinstance(m, SelectiveLRU):
                m.stream_chunk = args.stream_chunk
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
    sampler = ClockSampler(_device_uuid(device), args.clocks_log if rank == 0 else None) if clocks else None
    t0 = time.time()
    _barrier(world, device)
    n0 = _lib.launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        run_all()
    e.record(stream)
    _barrier(world, device)
    launches = _lib.launch_count() - n0
    t1 = time.time()
    if sampler is not None:
        sampler.stop()
    ms = _max_over_ranks(s.elapsed_time(e), world, device) / steps
    del model, buf
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    fps = total * frames / (ms * 1e-3)
    out = {
        "metric": "SEMamba long-utterance inference, frames/s (64 x 60 s utterances, sharded)",
        "value": round(fps, 1), "unit": "frames/s", "n_gpus": world, "steps": steps, "warmup": 1,
        "ms_per_step": round(ms, 2), "scaling": "strong",
        "dtype": "bf16 autocast, fp32 scans", "data": "synthetic (audio ~ N(0, 0.1), seeded per rank), "
                                                     "random-init weights",
        "config": {"workload": "STFT -> generator -> iSTFT, no_grad, 64 utterances of 60 s",
                   "global_batch": total, "seq_len": frames, "micro_batch": mb,
                   "stream_chunk": args.stream_chunk or None,
                   "parallelism": f"sharded over {world} GPUs"},
        "e2e": {"value": round(fps, 1), "unit": "frames/s", "h2d_bytes_per_step": total * seg * 4 // world,
                "d2h_bytes_per_step": total * seg * 4 // world,
                "note": "every step copies its audio in from pinned host memory and the enhanced audio out"},
        "gpu_launches": launches,
    }
    if sampler is not None:
        out["clocks"] = sampler.summary(t0, t1)
    return out


def run_inference(args, rank, local_rank, world):
    """The long-utterance inference as the bench line (`--workload inference`)."""
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    _init_dist(world, device)
    out = measure_inference(args, rank, local_rank, world, device, args.steps)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if out is None:
        return
    out.update(higher_is_better=True, vs_baseline=None)
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "generator":
        run_generator(args, rank, local_rank, world)
    elif args.workload == "inference":
        run_inference(args, rank, local_rank, world)
    else:
        run_scan(args, rank, local_rank, world)


if __name__ == "__main__":
    main()
