"""Benchmark of the B200 optimizer step (Muon + AdamW + global grad-norm clip) on the Mote-96M-shaped workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1]

One step = train.py:944-947 of the reference: grads /= 1 (no divisor), clip_grad_norm_(all grads, 1.0), AdamW on
the embedding and vectors, Muon (momentum + 5 Newton-Schulz iterations + apply) on every hidden matrix. Inputs
(fp32 params, bf16 grads, fp32 optimizer state; 1.1 GB) stay resident in HBM and are larger than L2, so nothing is
flushed between steps. Prints one JSON line (rank 0).

--impl reference times the reference's step on the host CPU: oracle/torch_port.py performs the reference's own torch
operations (the reference is Python and is not installed on the GPU host; the port equals it bit for bit on the
golden fixtures), one Newton-Schulz stack per step, extrapolated to the full step by stack counts.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "ms/optimizer step (96M set)"


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-adamw-sweep", action="store_true", help="skip the c4 AdamW sweep (1e6..2e9 elements)")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------------------
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
    """nvidia-smi clocks and throttle reasons every 100 ms while the timed region runs."""
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}",
                                          "--format=csv,noheader,nounits", "-i", self.gpu_id, "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
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


# ---------------------------------------------------------------------------------------------------------------
class TorchReference:
    """The reference's step on the host CPU (oracle/torch_port.py: the reference's own torch operations, equal to it
    bit for bit on the golden fixtures), sampled one Newton-Schulz stack at a time. `counts` maps each distinct
    stack of the workload's Muon step (the member params' shapes; muon.py:81-90 caps a stack at 32 MiB) to how often
    it occurs; `time_stack(key)` runs the whole Muon update of one such stack (momentum, stacked Newton-Schulz,
    decay, apply); `time_rest()` the grad division, the clip over every grad and the AdamW step."""

    def __init__(self, w):
        import torch
        from oracle import torch_port as TP
        self.torch, self.TP, self.w = torch, TP, w
        torch.set_num_threads(len(os.sched_getaffinity(0)))
        self.cores = torch.get_num_threads()
        gen = torch.Generator().manual_seed(0)

        def randn(shape, std):
            return torch.randn(shape, generator=gen) * std

        self.counts, self.stack = {}, {}
        for _, idx in TP.stacks([tuple(s) for s in w.muon_shapes]):
            key = tuple(tuple(w.muon_shapes[i]) for i in idx)
            self.counts[key] = self.counts.get(key, 0) + 1
            if key not in self.stack:
                ps = [torch.nn.Parameter(randn(s, 0.02)) for s in key]
                for q in ps:
                    q.grad = randn(q.shape, 1e-3).to(torch.bfloat16).float()
                self.stack[key] = (ps, [None] * len(ps))
        n_muon = w.numel()[0]
        self.flat = torch.nn.Parameter(torch.zeros(n_muon))   # every Muon grad, for the division and the clip
        self.adam_p = [torch.nn.Parameter(randn(s, 0.02)) for s in w.adam_shapes]
        nd = len(w.adam_decay_shapes)
        self.adam = torch.optim.AdamW([{"params": self.adam_p[:nd], "weight_decay": w.adam_wd},
                                       {"params": self.adam_p[nd:], "weight_decay": 0.0}], lr=w.adam_lr,
                                      betas=w.betas, eps=w.eps, fused=torch.cuda.is_available())   # train.py:98
        for key in self.stack:   # momentum buffers created, first-touch costs paid
            self.time_stack(key)
        self.time_rest()

    def time_stack(self, key) -> float:
        ps, bufs = self.stack[key]
        w = self.w
        t0 = time.perf_counter()
        self.TP.muon_update(ps, bufs, lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True,
                            weight_decay=w.muon_wd, ns_steps=w.ns_steps)
        return time.perf_counter() - t0

    def time_rest(self) -> float:
        torch = self.torch
        self.flat.grad = torch.full_like(self.flat, 1e-3)
        for q in self.adam_p:
            q.grad = torch.full_like(q, 1e-3)
        params = [self.flat] + self.adam_p
        t0 = time.perf_counter()
        torch._foreach_div_([q.grad for q in params], 1.0)
        torch.nn.utils.clip_grad_norm_(params, self.w.clip)
        self.adam.step()
        return time.perf_counter() - t0

    def describe(self, how: str) -> str:
        kinds = ", ".join(f"{len(k)} x {k[0]} ({c}x)" for k, c in self.counts.items())
        return (f"oracle/torch_port.py (the reference's torch CPU operations; bit-equal to the reference on the golden "
                f"fixtures) on {self.cores} host threads: {how} Muon stacks of the step [{kinds}]; plus grads /= n, "
                "clip_grad_norm_ and the AdamW step on the whole workload; summed by stack counts to the full step")


def cpu_baseline_sample(w) -> dict:
    """The reference's step on this host's cores (TorchReference): every stack kind timed twice after a warm-up,
    the medians summed by stack counts, plus the clip and AdamW."""
    ref = TorchReference(w)
    total = sum(c * statistics.median([ref.time_stack(k) for _ in range(2)]) for k, c in ref.counts.items())
    total += ref.time_rest()
    return {"value": round(total * 1e3, 3), "unit": "ms/step", "cores": int(ref.cores), "kind": "port",
            "sample": ref.describe("each of the")}


# ---------------------------------------------------------------------------------------------------------------
def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    from mote_b200 import _lib as L
    from mote_b200 import configs
    from mote_b200.functional import AdamWItem, CapturedStep, MuonItem, optimizer_step

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = configs.CONFIGS[args.config]()
    nd = len(w.adam_decay_shapes)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)

    def randn(shape, std, dtype=torch.float32):
        return (torch.randn(shape, generator=gen, device=dev) * std).to(dtype)

    mp = [randn(s, 0.02) for s in w.muon_shapes]
    ap = [randn(s, 0.02) for s in w.adam_shapes]
    # grads live in one flat bf16 buffer so the end-to-end run can refresh them with one host->device copy
    shapes = list(w.adam_shapes) + list(w.muon_shapes)
    sizes = [int(torch.Size(s).numel()) for s in shapes]
    flat = randn((sum(sizes),), 1e-3, torch.bfloat16)
    views = list(torch.split(flat, sizes))
    grads = [v.view(s) for v, s in zip(views, shapes)]
    ag, mg = grads[: len(ap)], grads[len(ap):]
    mb = [torch.zeros_like(p) for p in mp]
    am = [torch.zeros_like(p) for p in ap]
    av = [torch.zeros_like(p) for p in ap]
    norm = torch.empty((), dtype=torch.float32, device=dev)
    muon_items = [MuonItem(p, g, b, w.muon_lr, w.muon_lr * w.muon_wd, w.muon_momentum, True) for p, g, b in zip(mp, mg, mb)]
    counter = {"step": 0}

    def step():
        counter["step"] += 1
        adam_items = [AdamWItem(p, g, m, v, w.adam_lr, w.adam_wd if i < nd else 0.0, counter["step"])
                      for i, (p, g, m, v) in enumerate(zip(ap, ag, am, av))]
        optimizer_step(muon_items, adam_items, ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip,
                       out_norm=norm)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # eager steps (one library call per step), with the Newton-Schulz span recorded by the library's event hook
    n_eager = max(5, min(50, args.steps))
    ns_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_eager)]
    for a, b in ns_ev:
        a.record(stream)
        b.record(stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for k in range(n_eager):
        L.check(L.lib.moteopt_profile_ns_events(ns_ev[k][0].cuda_event, ns_ev[k][1].cuda_event), "events")
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    L.check(L.lib.moteopt_profile_ns_events(None, None), "events")
    eager_ms = e0.elapsed_time(e1) / n_eager
    ns_ms = statistics.mean(a.elapsed_time(b) for a, b in ns_ev)

    # the same step captured once in a CUDA graph and replayed (mote_b200.CapturedStep): the timed value
    adam_fixed = [AdamWItem(p, g, m, v, w.adam_lr, w.adam_wd if i < nd else 0.0, 1)
                  for i, (p, g, m, v) in enumerate(zip(ap, ag, am, av))]
    cs = CapturedStep(muon_items, adam_fixed, ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip,
                      start_step=counter["step"])
    cs()
    cs()   # captures
    for _ in range(args.warmup):
        cs()
    torch.cuda.synchronize(dev)
    gpu_id = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
    with ClockSampler(gpu_id) as clk:
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(args.steps):
            cs()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    launches = cs.launches_per_step * args.steps
    ms = e0.elapsed_time(e1) / args.steps
    st, _ = __import__("mote_b200.ops", fromlist=["read_status"]).read_status(dev)
    if st & 3:
        raise RuntimeError(f"kernel status {st}")

    # AdamW bandwidth on a flat 1e8-element tensor (the metric's "AdamW % HBM BW")
    n_flat = 100_000_000
    fp = randn((n_flat,), 0.02)
    fg = randn((n_flat,), 1e-3, torch.bfloat16)
    fm, fv = torch.zeros_like(fp), torch.zeros_like(fp)
    for k in range(3):
        optimizer_step((), [AdamWItem(fp, fg, fm, fv, 3e-4, 0.1, k + 1)], betas=w.betas)
    torch.cuda.synchronize(dev)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for k in range(10):
        optimizer_step((), [AdamWItem(fp, fg, fm, fv, 3e-4, 0.1, k + 4)], betas=w.betas)
    a1.record(stream)
    torch.cuda.synchronize(dev)
    adam_ms = a0.elapsed_time(a1) / 10
    del fp, fg, fm, fv

    sweep = None if args.no_adamw_sweep else _adamw_sweep(dev, gen, w.betas, load_peaks()[0]["hbm_gbs"], stream)

    # the fused extras (EMA of the weights, Muon param norms) against the separate torch passes the reference runs
    # after its step (train.py:950-953 _foreach_lerp_, elr.py:85-87 stacked norms), on the same c1 tensors
    extras = _time_extras(step, muon_items, adam_fixed, w, stream, counter)

    # end to end through the public API with host buffers: grads copied in from pinned memory, norm read back
    host_grads = flat.cpu().pin_memory()
    host_norm = torch.empty((), dtype=torch.float32).pin_memory()
    e2e_steps = max(5, min(50, args.steps // 6))
    streamed_e2e(cs, [(flat, host_grads)], host_norm, 3, stream)
    e2e_ms = streamed_e2e(cs, [(flat, host_grads)], host_norm, e2e_steps, stream)

    peaks, src = load_peaks()
    ns_flops = w.ns_flops_issued()          # what the tensor cores perform (upper-triangle Gram / A A blocks)
    # the library's default launch mode: one persistent launch up to 48 waves of tiles per iteration (74 CTA pairs)
    ns_launches = 1 if w.ns_tiles_per_iter() <= 48 * 74 else 3 * w.ns_steps
    ref_flops = w.ns_flops()                # the reference algorithm's full products
    achieved = ns_flops / (ns_ms * 1e-3) / 1e12
    traffic = None
    prof = ROOT / "profiles" / "ns_gemm_kernel_c1_traffic.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
    adam_gbs = 28.0 * n_flat / (adam_ms * 1e-3) / 1e9
    step_roof = step_roofline(ref_flops, w.state_bytes(), 0.0, peaks, ms)
    line = {
        "metric": METRIC, "value": round(ms, 4), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded params N(0,0.02^2) fp32, grads N(0,1e-3^2) bf16 (no dataset: an optimizer step)",
        "config": {"workload": w.name, "muon_matrices": len(w.muon_shapes), "muon_elems": w.numel()[0],
                   "adamw_elems": w.numel()[1], "ns_steps": w.ns_steps, "clip": w.clip,
                   "parallelism": f"dp{world}" if world > 1 else "single",
                   "l2": "inputs (1.1 GB) larger than L2; no flush",
                   "launch": "CUDA graph of the whole step (mote_b200.CapturedStep)", "eager_ms_per_step": round(eager_ms, 4)},
        "roofline": {"bound": "tensor", "kernel": "ns_gemm_kernel", "achieved": round(achieved, 1),
                     "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": round(achieved / peaks["bf16_tflops_sustained"], 4), "traffic": traffic,
                     "peak_source": f"{src} (sustained bf16: the kernel is timed inside back-to-back steps under the "
                                    f"power cap)", "frac_of_burst": round(achieved / peaks["bf16_tflops"], 4),
                     "ns_ms_per_step": round(ns_ms, 4), "ns_launches_per_step": ns_launches,
                     "ns_tflop_per_step": round(ns_flops / 1e12, 5), "ref_tflop_per_step": round(ref_flops / 1e12, 5),
                     "ref_equivalent_tflops": round(ref_flops / (ns_ms * 1e-3) / 1e12, 1),
                     "timed": "library events around the Newton-Schulz launch(es) of each eager step (one persistent "
                              "cooperative launch for all iterations, or one launch per phase for large problems)"},
        "step_roofline": step_roof,
        "adamw_hbm": {"achieved": round(adam_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                      "frac": round(adam_gbs / peaks["hbm_gbs"], 4), "elems": n_flat, "ms": round(adam_ms, 4)},
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms/step", "h2d_bytes_per_step": int(flat.numel() * 2),
                "d2h_bytes_per_step": 4, "how": "host-fed loop: each step's grads uploaded from pinned memory on a "
                "copy stream while the previous step computes, then moved to the grad buffer; norm read back"},
        "clocks": clk.summary(),
        "gpu_launches": int(launches),
        "extras": extras,
        "adamw_sweep": sweep,
    }
    return line


# ---------------------------------------------------------------------------------------------------------------
def step_roofline(flops: float, state_bytes: float, exchange_bytes: float, peaks: dict, ms: float,
                  link_gbs: float = 770.0) -> dict:
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


# ---------------------------------------------------------------------------------------------------------------
def _adamw_sweep(dev, gen, betas, hbm_gbs, stream) -> dict:
    """The AdamW-only bandwidth sweep (config c4): flat fp32 params of 1e6 to 2e9 elements, bf16 grads
    N(0, 1e-3^2), m/v from a 5-step warm-up, each step the global clip (norm pass) plus AdamW, captured as a CUDA
    graph. Reported per size: ms per step and GB/s at 28 B/elem (grad read by the norm and by the update, p, m, v
    read and written)."""
    import torch

    from mote_b200.functional import AdamWItem, CapturedStep
    sizes = [1_000_000, 10_000_000, 100_000_000, 1_000_000_000, 2_000_000_000]
    free = torch.cuda.mem_get_info(dev)[0]
    sizes = [n for n in sizes if 16 * n < free * 0.8]   # p, m, v fp32 + g bf16 = 14 B/elem, with headroom
    nmax = sizes[-1]
    p = torch.empty(nmax, device=dev).normal_(0.0, 0.02, generator=gen)
    g = torch.empty(nmax, device=dev).normal_(0.0, 1e-3, generator=gen).to(torch.bfloat16)
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    rows = []
    for n in sizes:
        cs = CapturedStep((), [AdamWItem(p[:n], g[:n], m[:n], v[:n], 3e-4, 0.1, 1)], betas=betas, max_norm=1.0)
        for _ in range(5):   # the m/v warm-up; the first call runs eagerly, the second captures
            cs()
        reps = 20 if n <= 100_000_000 else 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(reps):
            cs()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        gbs = 28.0 * n / (ms * 1e-3) / 1e9
        rows.append({"elems": n, "ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / hbm_gbs, 4)})
        del cs
    del p, g, m, v
    torch.cuda.empty_cache()
    return {"unit": "ms/step, GB/s", "bytes_per_elem": 28, "step": "clip_grad_norm_ + AdamW (CUDA graph)",
            "l2": "sizes above 4.5e6 elements exceed L2; smaller ones are L2-resident between steps", "rows": rows}


# ---------------------------------------------------------------------------------------------------------------
def _time_extras(step, muon_items, adam_items, w, stream, counter, reps: int = 10) -> dict:
    """ms per step of: the plain eager step; the step with the fused EMA; the step with the fused norms; and the
    reference's separate passes on the GPU (torch._foreach_lerp_ over every param; stacked per-matrix norms)."""
    import torch

    from mote_b200.functional import optimizer_step
    params = [it.param for it in adam_items] + [it.param for it in muon_items]
    ema = [p.clone() for p in params]
    norms = torch.empty(len(muon_items), dtype=torch.float32, device=params[0].device)

    def fused(**kw):
        counter["step"] += 1
        for it in adam_items:
            it.step = counter["step"]
        optimizer_step(muon_items, adam_items, ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip, **kw)

    def timed(fn):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    base = timed(step)
    with_ema = timed(lambda: fused(ema=ema, ema_weight=1e-3))
    with_norms = timed(lambda: fused(muon_norms=norms))
    sep_ema = timed(lambda: torch._foreach_lerp_(ema, params, 1e-3))
    mp = [it.param for it in muon_items]
    sep_norms = timed(lambda: torch.stack([p.float().norm() for p in mp]))
    return {"unit": "ms/step", "step": round(base, 4),
            "ema_fused_extra": round(with_ema - base, 4), "ema_separate_torch": round(sep_ema, 4),
            "norms_fused_extra": round(with_norms - base, 4), "norms_separate_torch": round(sep_norms, 4),
            "note": "fused: added time of the step with the extra; separate: torch pass on the same device tensors"}


def run_reference(args, rank: int, world: int):
    """The reference's step on the host CPU (TorchReference), one bounded sample per step: step k runs the Muon
    update of one Newton-Schulz stack, cycling through the workload's stack kinds; the per-kind medians summed by
    stack counts, plus the clip and AdamW, give the full step."""
    from mote_b200 import configs
    w = configs.CONFIGS[args.config]()
    ref = TorchReference(w)
    keys = list(ref.counts)
    t = {k: [] for k in keys}
    rest_t = []
    for k in range(args.warmup + args.steps):
        if not keys:   # a workload without Muon matrices (c4): every step samples the clip + AdamW step
            dt = ref.time_rest()
            if k >= args.warmup:
                rest_t.append(dt)
            continue
        key = keys[k % len(keys)]
        dt = ref.time_stack(key)
        if k >= args.warmup:
            t[key].append(dt)
    for key in keys:   # a kind not reached by a short run gets one measurement here
        if not t[key]:
            t[key].append(ref.time_stack(key))
    rest = statistics.median(rest_t or [ref.time_rest() for _ in range(3)])
    ms = (sum(ref.counts[k] * statistics.median(t[k]) for k in keys) + rest) * 1e3
    return {"metric": METRIC, "value": round(ms, 3), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "impl": "reference",
            "data": "synthetic: seeded params N(0,0.02^2) fp32, grads N(0,1e-3^2) bf16-valued fp32",
            "config": {"workload": w.name, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(ms, 3), "unit": "ms/step", "cores": int(ref.cores), "kind": "port",
                             "sample": ref.describe("per step one of the")},
            "e2e": {"value": round(ms, 3), "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args, rank, world)), flush=True)
        return 0
    if world > 1:
        from mote_b200 import dist_bench
        line = dist_bench.run(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
        return 0
    line = run_ours(args, rank, world, local_rank)
    if not args.no_cpu_baseline:
        from mote_b200 import configs
        line["cpu_baseline"] = cpu_baseline_sample(configs.CONFIGS[args.config]())
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
