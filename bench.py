"""Benchmark of the B200 optimizer step (Muon + AdamW + global grad-norm clip) on the Mote-96M-shaped workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1]

One step = train.py:944-947 of the reference: grads /= 1 (no divisor), clip_grad_norm_(all grads, 1.0), AdamW on
the embedding and vectors, Muon (momentum + 5 Newton-Schulz iterations + apply) on every hidden matrix. Inputs
(fp32 params, bf16 grads, fp32 optimizer state; 1.1 GB) stay resident in HBM and are larger than L2, so nothing is
flushed between steps. Prints one JSON line (rank 0). With N > 1 (under torch.distributed.run) the sharded step of
mote_b200/distributed.py runs instead (mote_b200/dist_bench.py).

--impl reference times the reference's own step on the host CPU, whole steps: oracle/torch_port.py performs the
reference's torch operations (the reference is Python and is not installed on the GPU host; the port equals it bit
for bit on the golden fixtures) over the whole workload, each timed step one complete optimizer step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from mote_b200.measure import (METRIC, ClockSampler, bench_config, load_peaks, step_roofline,  # noqa: E402
                               streamed_e2e)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-adamw-sweep", action="store_true", help="skip the c4 AdamW sweep (1e6..2e9 elements)")
    ap.add_argument("--no-other-configs", action="store_true", help="skip the c2 / c3 step lines and the c4 ZeRO-1 sweep")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------------------
class TorchReference:
    """The reference's whole optimizer step on the host CPU over workload `w`: oracle/torch_port.py performs the
    reference's own torch operations (train.py:944-947: grads /= n, clip_grad_norm_, torch.optim.AdamW built as
    train.py:98 builds it, then the reference's Muon step, muon.py:52-99) on seeded params and bf16-valued grads."""

    def __init__(self, w):
        import torch
        from oracle import torch_port as TP
        self.torch, self.TP, self.w = torch, TP, w
        torch.set_num_threads(len(os.sched_getaffinity(0)))
        self.cores = torch.get_num_threads()
        gen = torch.Generator().manual_seed(0)

        def param(shape):
            p = torch.nn.Parameter(torch.randn(shape, generator=gen) * 0.02)
            p.grad = (torch.randn(shape, generator=gen) * 1e-3).to(torch.bfloat16).float()
            return p

        self.adam_p = [param(s) for s in w.adam_shapes]
        self.muon_p = [param(s) for s in w.muon_shapes]
        self.bufs = [None] * len(self.muon_p)
        nd = len(w.adam_decay_shapes)
        groups = [g for g in ({"params": self.adam_p[:nd], "weight_decay": w.adam_wd},
                              {"params": self.adam_p[nd:], "weight_decay": 0.0}) if g["params"]]
        self.adam = (torch.optim.AdamW(groups, lr=w.adam_lr, betas=w.betas, eps=w.eps,
                                       fused=torch.cuda.is_available()) if groups else None)   # train.py:98

    def time_step(self) -> float:
        """Seconds of one whole reference step (the grads are left as the step scales them: with the clip active
        they settle at norm max_norm, so every step does the same work)."""
        w = self.w
        t0 = time.perf_counter()
        self.TP.optimizer_step(self.adam, self.muon_p, self.bufs, self.adam_p + self.muon_p, divisor=1.0,
                               max_norm=w.clip, muon_kw=dict(lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True,
                                                             weight_decay=w.muon_wd, ns_steps=w.ns_steps))
        return time.perf_counter() - t0

    def describe(self, n: int) -> str:
        return (f"oracle/torch_port.py (the reference's torch CPU operations; bit-equal to the reference on the golden "
                f"fixtures) on {self.cores} host threads: {n} whole steps of the workload (grads /= n, clip_grad_norm_, "
                f"AdamW, Muon with Newton-Schulz stacked under the 32 MiB cap), median")


def cpu_baseline_sample(w, steps: int = 5) -> dict:
    """The reference's step on this host's cores (TorchReference): one warm-up step, then the median of `steps`
    whole steps (fewer when a step takes more than 6 s, so the sample stays near 30 s of CPU work)."""
    ref = TorchReference(w)
    first = ref.time_step()
    n = max(1, min(steps, int(30.0 / max(first, 1e-3))))
    t = [ref.time_step() for _ in range(n)]
    return {"value": round(statistics.median(t) * 1e3, 3), "unit": "ms/step", "cores": int(ref.cores), "kind": "port",
            "sample": ref.describe(n)}


# ---------------------------------------------------------------------------------------------------------------
def _ns_roofline(w, ns_ms: float, peaks: dict, src: str) -> dict:
    """The Newton-Schulz kernel against the tensor roofline: achieved = the reference algorithm's FLOPs (the
    north star's per-matrix 5 (4 m^2 n + 2 m^3)) / the kernel's time, against the measured burst bf16 peak (the
    kernel is timed inside steps of a few milliseconds); the sustained figure and the FLOPs the tensor cores issue
    (upper-triangle blocks of the symmetric products only) are given beside it."""
    ref = w.ns_flops()
    issued = w.ns_flops_issued()
    achieved = ref / (ns_ms * 1e-3) / 1e12
    return {"bound": "tensor", "kernel": "ns_gemm_kernel", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
            "peak_source": f"{src} (burst bf16, of measured)" if src == "measured" else f"{src} (burst bf16)",
            "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4),
            "ns_ms_per_step": round(ns_ms, 4), "ref_tflop_per_step": round(ref / 1e12, 5),
            "issued_tflop_per_step": round(issued / 1e12, 5),
            "issued_tflops": round(issued / (ns_ms * 1e-3) / 1e12, 1)}


def _make_workload(w, dev, seed: int):
    """Seeded device tensors of workload w: fp32 params ~ N(0, 0.02^2); bf16 grads ~ N(0, 1e-3^2) (each expert of a
    3-D stack scaled by its grad_scale factor) in one flat buffer; zero optimizer state. Returns (muon items,
    adam items factory, flat grads, params)."""
    import torch
    from mote_b200.functional import AdamWItem, MuonItem
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)

    def randn(shape, std):
        return torch.randn(shape, generator=gen, device=dev) * std

    mp = [randn(s, 0.02) for s in w.muon_shapes]
    ap = [randn(s, 0.02) for s in w.adam_shapes]
    shapes = list(w.adam_shapes) + list(w.muon_shapes)
    sizes = [int(torch.Size(s).numel()) for s in shapes]
    flat = torch.empty(sum(sizes), dtype=torch.bfloat16, device=dev)
    for v, s in zip(torch.split(flat, sizes), shapes):
        g = randn(s, 1e-3)
        if w.grad_scale is not None and len(s) == 3:
            g *= torch.tensor(w.grad_scale[: s[0]], device=dev)[:, None, None]
        v.copy_(g.reshape(-1))
    grads = [v.view(s) for v, s in zip(torch.split(flat, sizes), shapes)]
    ag, mg = grads[: len(ap)], grads[len(ap):]
    mb = [torch.zeros_like(p) for p in mp]
    am = [torch.zeros_like(p) for p in ap]
    av = [torch.zeros_like(p) for p in ap]
    nd = len(w.adam_decay_shapes)
    muon = [MuonItem(p, g, b, w.muon_lr, w.muon_lr * w.muon_wd, w.muon_momentum, True) for p, g, b in zip(mp, mg, mb)]

    def adam(step):
        return [AdamWItem(p, g, m, v, w.adam_lr, w.adam_wd if i < nd else 0.0, step)
                for i, (p, g, m, v) in enumerate(zip(ap, ag, am, av))]
    return muon, adam, flat, (mp, ap)


def _eager_ns_ms(step, n: int, stream) -> float:
    """Mean Newton-Schulz time of `n` eager steps, from the library's events around its Newton-Schulz launch(es)."""
    import torch
    from mote_b200 import _lib as L
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for a, b in ev:
        a.record(stream)
        b.record(stream)
    torch.cuda.synchronize()
    for k in range(n):
        L.check(L.lib.moteopt_profile_ns_events(ev[k][0].cuda_event, ev[k][1].cuda_event), "events")
        step()
    torch.cuda.synchronize()
    L.check(L.lib.moteopt_profile_ns_events(None, None), "events")
    return statistics.mean(a.elapsed_time(b) for a, b in ev)


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    from mote_b200 import configs
    from mote_b200.functional import AdamWItem, CapturedStep, optimizer_step

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = configs.CONFIGS[args.config]()
    muon_items, adam_items, flat, (mp, ap) = _make_workload(w, dev, seed=0)
    norm = torch.empty((), dtype=torch.float32, device=dev)
    counter = {"step": 0}

    def step():
        counter["step"] += 1
        optimizer_step(muon_items, adam_items(counter["step"]), ns_steps=w.ns_steps, betas=w.betas, eps=w.eps,
                       max_norm=w.clip, out_norm=norm)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # eager steps (one library call per step), with the Newton-Schulz span recorded by the library's event hook
    n_eager = max(5, min(50, args.steps))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    ns_ms = _eager_ns_ms(step, n_eager, stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    eager_ms = e0.elapsed_time(e1) / n_eager

    # the same step captured once in a CUDA graph and replayed (mote_b200.CapturedStep): the timed value
    cs = CapturedStep(muon_items, adam_items(1), ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip,
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

    # end to end through the public API with host buffers: grads copied in from pinned memory, norm read back
    host_grads = flat.cpu().pin_memory()
    host_norm = torch.empty((), dtype=torch.float32).pin_memory()
    e2e_steps = max(5, min(50, args.steps // 6))
    streamed_e2e(cs, [(flat, host_grads)], host_norm, 3, stream)
    e2e_ms = streamed_e2e(cs, [(flat, host_grads)], host_norm, e2e_steps, stream)

    # AdamW bandwidth on a flat 1e8-element tensor (the metric's "AdamW % HBM BW")
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    n_flat = 100_000_000
    fp = torch.randn(n_flat, generator=gen, device=dev) * 0.02
    fg = (torch.randn(n_flat, generator=gen, device=dev) * 1e-3).to(torch.bfloat16)
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

    peaks, src = load_peaks()
    sweep = None if args.no_adamw_sweep else _adamw_sweep(dev, gen, w.betas, peaks["hbm_gbs"], stream)

    # the fused extras (EMA of the weights, Muon param norms) against the separate torch passes the reference runs
    # after its step (train.py:950-953 _foreach_lerp_, elr.py:85-87 stacked norms), on the same c1 tensors
    extras = _time_extras(step, muon_items, adam_items(1), w, stream, counter)
    extras["class_swap"] = _class_swap(w, dev, stream)
    del cs, muon_items, adam_items, flat, mp, ap
    torch.cuda.empty_cache()
    other = None
    if not args.no_other_configs and args.config == "c1":
        other = {name: _config_line(name, dev, stream, peaks) for name in ("c2", "c3")}
        other["c1_gram_ns"] = _config_line("c1", dev, stream, peaks, ns_variant=1)

    roof = _ns_roofline(w, ns_ms, peaks, src)
    prof = ROOT / "profiles" / "ns_gemm_kernel_c1_traffic.json"
    roof["traffic"] = json.loads(prof.read_text()).get("dram_bytes_per_launch") if prof.exists() and \
        args.config == "c1" else None
    roof["timed"] = ("library events around the Newton-Schulz launch(es) of each eager step (one persistent "
                     "cooperative launch for all iterations, or one launch per phase for large problems)")
    adam_gbs = 28.0 * n_flat / (adam_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(ms, 4), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded params N(0,0.02^2) fp32, grads N(0,1e-3^2) bf16 (no dataset: an optimizer step)",
        "config": bench_config(w, world),
        "launch": {"timed": "CUDA graph of the whole step (mote_b200.CapturedStep)",
                   "eager_ms_per_step": round(eager_ms, 4)},
        "roofline": roof,
        "step_roofline": step_roofline(w.ns_flops(), w.state_bytes(), 0.0, peaks, ms),
        "adamw_hbm": {"achieved": round(adam_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                      "frac": round(adam_gbs / peaks["hbm_gbs"], 4), "elems": n_flat, "ms": round(adam_ms, 4)},
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms/step", "h2d_bytes_per_step": int(flat_bytes(w)),
                "d2h_bytes_per_step": 4, "how": "host-fed loop: each step's grads uploaded from pinned memory on a "
                "copy stream while the previous step computes, then moved to the grad buffer; norm read back"},
        "clocks": clk.summary(),
        "gpu_launches": int(launches),
        "extras": extras,
        "adamw_sweep": sweep,
        "other_configs": other,
    }
    return line


def flat_bytes(w) -> int:
    m, a = w.numel()
    return 2 * (m + a)


# ---------------------------------------------------------------------------------------------------------------
def _config_line(name: str, dev, stream, peaks, steps: int = 10, warmup: int = 3, ns_variant: int = 0) -> dict:
    """One other benchmark configuration on this GPU (c2: batched Muon stress; c3: MoE expert stacks with Zipf-scaled
    expert grads; or c1 with the opt-in Gram Newton-Schulz variant, ns_variant 1): the step as a CUDA graph, its
    Newton-Schulz time from eager steps, and both rooflines (the variant's against its own algorithmic FLOPs)."""
    import torch
    from mote_b200 import configs
    from mote_b200.functional import CapturedStep, optimizer_step
    w = configs.CONFIGS[name]()
    muon, adam, flat, _ = _make_workload(w, dev, seed=1)
    k = {"n": 0}

    def step():
        k["n"] += 1
        optimizer_step(muon, adam(k["n"]), ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip,
                       ns_variant=ns_variant)
    for _ in range(warmup):
        step()
    ns_ms = _eager_ns_ms(step, 3, stream)
    cs = CapturedStep(muon, adam(1), ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip,
                      start_step=k["n"], ns_variant=ns_variant)
    for _ in range(warmup):
        cs()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(steps):
        cs()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    flops = w.ns_flops_gram() if ns_variant else w.ns_flops()
    roof = _ns_roofline(w, ns_ms, peaks, "measured")
    if ns_variant:   # achieved on the variant's own algorithmic FLOPs
        roof["achieved"] = round(flops / (ns_ms * 1e-3) / 1e12, 1)
        roof["frac"] = round(roof["achieved"] / peaks["bf16_tflops"], 4)
        roof["frac_of_sustained"] = round(roof["achieved"] / peaks["bf16_tflops_sustained"], 4)
        roof["variant_tflop_per_step"] = round(flops / 1e12, 5)
    out = {"workload": w.name, "config": bench_config(w, 1), "ms_per_step": round(ms, 4), "steps": steps,
           "ns_variant": "gram (opt-in, not the reference's iteration)" if ns_variant else "reference", "ns": roof,
           "step_roofline": step_roofline(flops, w.state_bytes(), 0.0, peaks, ms)}
    del cs, muon, adam, flat
    torch.cuda.empty_cache()
    return out


def _class_swap(w, dev, stream, reps: int = 10) -> dict:
    """What the trainer pays when only its optimizer classes are swapped for this package's: train.py:945-946
    (torch._foreach_div_ and clip_grad_norm_) stay on ATen and MultiOpt.step runs the library's step, against
    fused_step (the division and the clip folded into the library's step). The trainer's grads are fp32."""
    import torch
    from mote_b200.optim import AdamW, Muon, MultiOpt, fused_step
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    nd = len(w.adam_decay_shapes)

    def param(s):
        p = torch.nn.Parameter(torch.randn(s, generator=gen, device=dev) * 0.02)
        p.grad = (torch.randn(s, generator=gen, device=dev) * 1e-3).to(torch.bfloat16).float()
        return p
    ap = [param(s) for s in w.adam_shapes]
    mp = [param(s) for s in w.muon_shapes]
    opt = MultiOpt([AdamW([{"params": ap[:nd], "weight_decay": w.adam_wd}, {"params": ap[nd:], "weight_decay": 0.0}],
                          lr=w.adam_lr, betas=w.betas, eps=w.eps),
                    Muon(mp, lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True, weight_decay=w.muon_wd)])
    params = ap + mp
    total_n = torch.tensor(1.0, device=dev)

    def aten_div_clip():
        torch._foreach_div_([p.grad for p in params], total_n)
        torch.nn.utils.clip_grad_norm_(params, w.clip)

    def swapped():
        aten_div_clip()
        opt.step()

    def timed(fn):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps
    out = {"unit": "ms/step", "grads": "fp32 (the trainer's)",
           "aten_div_clip": round(timed(aten_div_clip), 4),
           "multiopt_step": round(timed(opt.step), 4),
           "classes_swapped_total": round(timed(swapped), 4),
           "fused_step": round(timed(lambda: fused_step(opt, max_norm=w.clip, grad_divisor=total_n)), 4)}
    del opt, ap, mp, params
    torch.cuda.empty_cache()
    return out


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
    """The reference's step on the host CPU (TorchReference): W warm-up steps, then K timed whole steps; the value is
    their median."""
    from mote_b200 import configs
    w = configs.CONFIGS[args.config]()
    ref = TorchReference(w)
    for _ in range(args.warmup):
        ref.time_step()
    t = [ref.time_step() for _ in range(max(1, args.steps))]
    ms = statistics.median(t) * 1e3
    return {"metric": METRIC, "value": round(ms, 3), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "impl": "reference",
            "data": "synthetic: seeded params N(0,0.02^2) fp32, grads N(0,1e-3^2) bf16-valued fp32",
            "config": bench_config(w, world),
            "cpu_baseline": {"value": round(ms, 3), "unit": "ms/step", "cores": int(ref.cores), "kind": "port",
                             "sample": ref.describe(len(t))},
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
