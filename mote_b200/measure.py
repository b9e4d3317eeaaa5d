"""Measurement helpers shared by bench.py's one-GPU leg and its N-GPU leg (mote_b200/dist_bench.py): the measured
peaks, the step roofline the target is stated against, nvidia-smi clock sampling during a timed region, the
host-fed end-to-end loop, and the benchmark line's `config` (the same dict in the library's arm and the reference
arm, so the two lines describe one workload). Reading the GPU's clocks is all this module does with nvidia-smi.
"""

from __future__ import annotations

import json
import statistics
import subprocess
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
METRIC = "ms/optimizer step (96M set)"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
NVLINK_GBS = 770.0   # the pool's measured peer copy, GB/s per direction per GPU


def load_peaks():
    """(peaks, "measured" | "fallback"): the driver-measured MEASURED_PEAKS.json at the repository root when present."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def bench_config(w, world: int) -> dict:
    """The benchmark line's `config`: the workload and how it is split, nothing measured, so that the library's line
    and the reference arm's line carry the same dict for the same workload and GPU count."""
    m, a = w.numel()
    return {"workload": w.name, "muon_matrices": len(w.muon_shapes), "muon_elems": m, "adamw_elems": a,
            "ns_steps": w.ns_steps, "clip": w.clip,
            "parallelism": f"muon-owner+zero1 x{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (126 MB); no flush"}


def step_roofline(flops: float, state_bytes: float, exchange_bytes: float, peaks: dict, ms: float,
                  link_gbs: float = NVLINK_GBS) -> dict:
    """The step-level roofline the target is stated against: the slower of the reference algorithm's GEMM FLOPs at
    the bf16 peak and the optimizer-state bytes at HBM bandwidth, plus the bytes a GPU receives in the exchange at
    the NVLink rate (the pool's measured peer copy, 770 GB/s per direction), per GPU. Given for the measured
    sustained and burst bf16 peaks; `frac` = roofline time / measured step time."""
    out = {"unit": "ms", "gemm_tflop": round(flops / 1e12, 4), "state_gb": round(state_bytes / 1e9, 4),
           "exchange_gb": round(exchange_bytes / 1e9, 4)}
    link_ms = exchange_bytes / (link_gbs * 1e9) * 1e3
    hbm_ms = state_bytes / (peaks["hbm_gbs"] * 1e9) * 1e3
    for key, tf in (("sustained", peaks["bf16_tflops_sustained"]), ("burst", peaks["bf16_tflops"])):
        roof = max(flops / (tf * 1e12) * 1e3, hbm_ms) + link_ms
        out[key] = {"roofline_ms": round(roof, 4), "frac": round(roof / ms, 4)}
    return out


def streamed_e2e(step_fn, pairs, host_norm, steps: int, stream) -> float:
    """ms per step of a host-fed training loop: every step's grads are copied from pinned host memory (each (device
    buffer, host tensor) pair) and the step's grad norm is read back to pinned host memory, all inside the timed
    region. The upload of step k+1 runs on a copy stream into a staging buffer while step k computes (the way a
    host-fed loop would stream its inputs); the step then moves its grads staging -> device buffer on the compute
    stream before it starts. CUDA events on the compute stream bracket the loop."""
    import torch
    copy = torch.cuda.Stream(device=pairs[0][0].device)
    staging = [torch.empty_like(d) for d, _ in pairs]
    copied, free = torch.cuda.Event(), torch.cuda.Event()

    def upload():
        with torch.cuda.stream(copy):
            copy.wait_event(free)   # the previous staging -> device copy has read the staging buffers
            for st, (_, h) in zip(staging, pairs):
                st.copy_(h, non_blocking=True)
            copied.record(copy)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    copy.wait_stream(stream)   # the first upload starts inside the timed region
    upload()
    for k in range(steps):
        stream.wait_event(copied)
        for st, (d, _) in zip(staging, pairs):
            d.copy_(st, non_blocking=True)
        free.record(stream)
        if k + 1 < steps:
            upload()
        host_norm.copy_(step_fn(), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


class ClockSampler:
    """nvidia-smi clocks and throttle reasons while the timed region runs (read only). Sampling every 20 ms, it waits
    for nvidia-smi's first sample before the region starts, and keeps the samples taken from the start of the region
    until 150 ms after its end (the sample in flight when a region of a few tens of milliseconds ends)."""
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_id: str, interval_ms: int = 20):
        self.gpu_id = gpu_id
        self.interval_ms = interval_ms
        self.proc = None
        self.samples = []   # (monotonic time, line)
        self.lines = []
        self._thread = None
        self.t0 = self.t1 = 0.0

    def _read(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.samples.append((time.monotonic(), ln))

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}",
                                          "--format=csv,noheader,nounits", "-i", self.gpu_id, "-lms",
                                          str(self.interval_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
            deadline = time.monotonic() + 5.0
            while not self.samples and time.monotonic() < deadline and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        self.t0 = time.monotonic()
        return self

    def restart(self):
        """Keep only the samples taken from now on (the timed region starts here)."""
        self.t0 = time.monotonic()

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            if self._thread is not None:
                self._thread.join(timeout=5)
        self.lines = [ln for t, ln in self.samples if self.t0 <= t <= self.t1 + 0.15]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}
