"""bench.py's N > 1 leg: the sharded optimizer step of mote_b200.distributed on N GPUs of one node, one process per
GPU (launched by torch.distributed.run), NCCL over NVLink.

Each rank holds the whole c1 model in its flat param regions and its own local bf16 grads; one step is the
reduce-scatter of the grads, the global clip from per-rank sums, the owned updates, and the exchange and apply of
the Muon updates (read from their owners over NVLink) with the AdamW slices all-gathered. Time is measured with CUDA
events on each rank and the maximum over ranks is reported, with a per-phase breakdown of eager steps (max over
ranks per phase) and a bitwise check that every rank ends the timed steps with the same params.
"""

from __future__ import annotations

import contextlib
import datetime
import json
import statistics

import torch
import torch.distributed as dist

from . import configs
from .distributed import ShardedStep, capture, cuda_compute, make_plan
from .measure import METRIC, ClockSampler, bench_config, load_peaks, step_roofline, streamed_e2e

PHASES = ["reduce_scatter", "grad_norm", "owned_update", "exchange", "apply_all"]


def checksum(*tensors: torch.Tensor) -> int:
    """A bitwise checksum of fp32 tensors (the int32 words summed with position weights, in int64), equal on two
    ranks exactly when their bits agree (up to a 2^-64 collision chance of the weighted sum)."""
    total = 0
    for t in tensors:
        w = t.contiguous().view(torch.int32).to(torch.int64)
        idx = torch.arange(1, w.numel() + 1, device=w.device, dtype=torch.int64)
        total = (total + int((w * (idx % 1000003 + 1)).sum().item()) * 31 + int(w.sum().item())) & ((1 << 63) - 1)
    return total


def _sharded_setup(w, plan, rank, dev, grad_seed):
    nd = len(w.adam_decay_shapes)
    pm = torch.zeros(plan.muon_len, dtype=torch.float32, device=dev)
    pa = torch.zeros(plan.adam_len, dtype=torch.float32, device=dev)
    st = ShardedStep(plan, rank, pm, pa, torch.zeros(plan.muon_len, dtype=torch.bfloat16, device=dev),
                     torch.zeros(plan.adam_len, dtype=torch.bfloat16, device=dev),
                     cuda_compute(ns_steps=w.ns_steps, betas=w.betas, eps=w.eps), muon_lr=w.muon_lr,
                     muon_wd=w.muon_wd, momentum=w.muon_momentum, adam_lr=w.adam_lr,
                     adam_wd=[w.adam_wd if i < nd else 0.0 for i in range(len(w.adam_shapes))])
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)   # identical params on every rank
    for i in range(len(w.muon_shapes)):
        st.muon_view(pm, i).normal_(0.0, 0.02, generator=gen)
    for i in range(len(w.adam_shapes)):
        st.adam_view(pa, i).normal_(0.0, 0.02, generator=gen)
    gen.manual_seed(grad_seed + rank)   # local grads differ per rank
    if plan.muon_len:
        st.gm.copy_(torch.randn(plan.muon_len, generator=gen, device=dev) * 1e-3)
    if plan.adam_len:
        st.ga.copy_(torch.randn(plan.adam_len, generator=gen, device=dev) * 1e-3)
    return st


def _phases(st, w, n: int, dev, gate_ms: float = 20.0) -> dict:
    """Mean ms of each phase of `n` eager steps on this rank (events recorded after each phase). Each step is queued
    behind a bounded GPU sleep (torch.cuda._sleep, a clock-counting kernel of about gate_ms) issued right after a
    barrier on every rank, so the host has enqueued the whole step, collectives included, before the GPU starts it:
    the phase times are GPU time, not the host's launch work."""
    acc = {p: [] for p in PHASES}
    cycles = int(gate_ms * 2.0e6)   # SM cycles at up to 2 GHz: at least gate_ms
    for _ in range(n):
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda._sleep(cycles)
        marks = []
        st.step(max_norm=w.clip, marks=marks)
        torch.cuda.synchronize(dev)
        for (_, a), (name, b) in zip(marks, marks[1:]):
            acc[name].append(a.elapsed_time(b))
    return {p: statistics.mean(v) for p, v in acc.items() if v}


def _zero1_sweep(world: int, rank: int, dev, peaks: dict, sizes=(100_000_000, 1_000_000_000), steps: int = 5) -> dict:
    """Config c4 at N GPUs: AdamW-only flat fp32 params, ZeRO-1 (reduce-scatter of the bf16 grads, the global clip from
    per-rank sums, AdamW on the owned slice, all-gather of the fp32 params), the whole step as a CUDA graph. Per size:
    ms per step (max over ranks) and the step roofline (28 B/elem of state per GPU at HBM rate + the grad
    reduce-scatter and the param all-gather at the NVLink rate)."""
    rows = []
    for n in sizes:
        free = torch.cuda.mem_get_info(dev)[0]
        if (6 + 12.0 / world) * n > 0.7 * free:   # p fp32 + g bf16 + the owned slice's grads, m, v
            continue
        w = configs.c4(n)
        plan = make_plan([], w.adam_shapes, world)
        st = _sharded_setup(w, plan, rank, dev, grad_seed=3000)
        held = {"graph": None}   # released before anything else can end the process group
        try:
            for _ in range(2):
                st.step(max_norm=1.0)
            held["graph"], _ = capture(st, max_norm=1.0)
            for _ in range(2):
                held["graph"].replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(dev)
            dist.barrier()
            e0.record()
            for _ in range(steps):
                held["graph"].replay()
            e1.record()
            torch.cuda.synchronize(dev)
        finally:
            held["graph"] = None
        ms_local = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        dist.all_reduce(ms_local, op=dist.ReduceOp.MAX)
        ms = float(ms_local.item())
        link = (2.0 + 4.0) * n * (world - 1) / world   # bytes each GPU receives: bf16 grads in, fp32 params back
        rows.append({"elems": n, "ms": round(ms, 4),
                     "step_roofline": step_roofline(0.0, 28.0 * n / world, link, peaks, ms)})
        del st
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
        dist.barrier()
    return {"unit": "ms/step", "step": "ZeRO-1 AdamW + clip (CUDA graph, NCCL reduce-scatter / all-gather)",
            "rows": rows}


def run(args, rank: int, world: int, local_rank: int):
    from . import _lib as L
    from .ops import read_status

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    held = {"graph": None}   # the only reference to the captured graph: dropped before destroy_process_group
    try:
        w = configs.CONFIGS[args.config]()
        plan = make_plan(w.muon_shapes, w.adam_shapes, world, ns_steps=w.ns_steps)
        st = _sharded_setup(w, plan, rank, dev, grad_seed=1000)
        stream = torch.cuda.current_stream(dev)
        peer_error = ""
        try:
            st.enable_peer_updates()
        except Exception as exc:  # noqa: BLE001  (recorded in the JSON line; the all-gather exchange is used instead)
            peer_error = f"{type(exc).__name__}: {exc}"[:200]

        for _ in range(args.warmup):
            st.step(max_norm=w.clip)
        torch.cuda.synchronize(dev)
        dist.barrier()
        # eager steps with the library's Newton-Schulz event hook (the roofline's kernel time)
        n_eager = max(3, min(20, args.steps))
        ns_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_eager)]
        for a, b in ns_ev:
            a.record(stream)
            b.record(stream)
        torch.cuda.synchronize(dev)
        for k in range(n_eager):
            L.check(L.lib.moteopt_profile_ns_events(ns_ev[k][0].cuda_event, ns_ev[k][1].cuda_event), "events")
            st.step(max_norm=w.clip)
        torch.cuda.synchronize(dev)
        L.check(L.lib.moteopt_profile_ns_events(None, None), "events")
        ns_local = statistics.mean(a.elapsed_time(b) for a, b in ns_ev) if st.mine else 0.0
        phases_local = _phases(st, w, max(3, min(10, args.steps)), dev)
        # the whole sharded step (NCCL collectives + kernels) captured in a CUDA graph and replayed
        capture_error = ""
        _norm = None
        l0 = L.lib.moteopt_launch_count()
        try:
            held["graph"], _norm = capture(st, max_norm=w.clip)
        except Exception as exc:  # noqa: BLE001  (recorded in the JSON line; the eager step is timed instead)
            held["graph"] = None
            capture_error = f"{type(exc).__name__}: {exc}"[:200]
        per_step = L.lib.moteopt_launch_count() - l0
        captured = held["graph"] is not None

        def run_step():
            if captured:
                held["graph"].replay()
                return _norm
            return st.step(max_norm=w.clip)
        for _ in range(3):
            run_step()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gpu_id = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
        # clocks sampled by rank 0 alone (one nvidia-smi for the node; the line reports rank 0's GPU). The sampler
        # starts before the barrier: every rank enters the timed region together, so no rank's collectives wait
        # for rank 0's sampler to come up inside another rank's timed region
        with ClockSampler(gpu_id) if rank == 0 else contextlib.nullcontext() as clk:
            torch.cuda.synchronize(dev)
            dist.barrier()
            if clk is not None:
                clk.restart()
            l1 = L.lib.moteopt_launch_count()
            e0.record(stream)
            for _ in range(args.steps):
                run_step()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        launches = per_step * args.steps if captured else L.lib.moteopt_launch_count() - l1
        ms_local = e0.elapsed_time(e1) / args.steps
        status, _ = read_status(dev)
        if status & 3:
            raise RuntimeError(f"rank {rank}: kernel status {status}")
        # every rank must hold the same params after the timed steps (each applies every update itself)
        sums = [None] * world
        dist.all_gather_object(sums, checksum(st.pm, st.pa))
        ranks_equal = all(s == sums[0] for s in sums)

        # end to end: this rank's local grads copied in from pinned host memory, the grad norm read back
        host_m = st.gm.cpu().pin_memory()
        host_a = st.ga.cpu().pin_memory()
        host_norm = torch.empty((), dtype=torch.float32).pin_memory()
        e2e_steps = max(5, min(30, args.steps // 6))
        pairs = [(st.gm, host_m), (st.ga, host_a)]
        streamed_e2e(run_step, pairs, host_norm, 2, stream)
        dist.barrier()
        e2e_local = streamed_e2e(run_step, pairs, host_norm, e2e_steps, stream)

        my_flops = sum(w.ns_steps * _ns_flops(w.muon_shapes[i]) for i in st.mine)
        vals = torch.tensor([ms_local, e2e_local, ns_local, float(launches), my_flops]
                            + [phases_local.get(p, 0.0) for p in PHASES], dtype=torch.float64, device=dev)
        allv = [torch.zeros_like(vals) for _ in range(world)]
        dist.all_gather(allv, vals)
        allv = torch.stack(allv).cpu()
        ms = float(allv[:, 0].max())
        e2e = float(allv[:, 1].max())
        slow = int(allv[:, 2].argmax())
        peaks, src = load_peaks()
        ns_ms = float(allv[slow, 2])
        achieved = float(allv[slow, 4]) / (ns_ms * 1e-3) / 1e12 if ns_ms > 0 else 0.0
        phases = {p: {"max": round(float(allv[:, 5 + k].max()), 4), "mean": round(float(allv[:, 5 + k].mean()), 4)}
                  for k, p in enumerate(PHASES)}
        phases["owned_update"]["per_rank"] = [round(float(x), 4) for x in allv[:, 5 + PHASES.index("owned_update")]]
        phases["newton_schulz_per_rank"] = [round(float(x), 4) for x in allv[:, 2]]
        # per GPU: 1/N of the reference FLOPs and state bytes; received in the exchange: the other ranks' bf16 O
        o_bytes = 2.0 * w.numel()[0]
        roof = step_roofline(w.ns_flops() / world, w.state_bytes() / world, o_bytes * (world - 1) / world, peaks, ms)
        h2d = int((st.gm.numel() + st.ga.numel()) * 2)
        peer_grads = st._peer_pieces is not None
        held["graph"] = None
        st.close()
        zero1 = None if args.no_other_configs else _zero1_sweep(world, rank, dev, peaks)
        line = {
            "metric": METRIC, "value": round(ms, 4), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded params N(0,0.02^2) fp32 (same on every rank), local grads N(0,1e-3^2) bf16 per rank",
            "config": bench_config(w, world),
            "launch": {"timed": "CUDA graph of the whole sharded step" if captured
                       else f"eager (graph capture failed: {capture_error})", "collectives":
                       ("grads reduced by reading every rank's grads over NVLink (CUDA IPC mappings, one-element "
                        "all-reduce as the ordering barrier; per-tensor sums of squares in the same pass)"
                        if peer_grads else "NCCL reduce-scatter (grads)") +
                       ", all-gather (per-rank per-tensor sums of squares), all-gather (AdamW fp32 "
                       "params); Muon updates: " + ("every rank's bf16 O read over NVLink by the apply kernel (CUDA "
                       "IPC mappings, one-element all-reduce as the ordering barrier)" if not peer_error
                       else f"NCCL all-gather of bf16 O ({peer_error})")},
            "ranks_equal": ranks_equal,
            "phases_ms": {"how": "eager steps queued behind a GPU sleep (so host launch work is hidden), CUDA events "
                                 "after each phase on every rank; max and mean over ranks", **phases},
            "roofline": {"bound": "tensor", "kernel": "ns_gemm_kernel", "achieved": round(achieved, 1),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops"], 4), "traffic": None,
                         "peak_source": f"{src} (burst bf16)",
                         "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4),
                         "rank": slow, "ns_ms_per_step": round(ns_ms, 4),
                         "achieved_of": "the reference algorithm's FLOPs of the slowest rank's matrices"},
            "step_roofline": roof,
            "e2e": {"value": round(e2e, 4), "unit": "ms/step", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                    "h2d_aggregate_gbs": round(world * h2d / (e2e * 1e-3) / 1e9, 1),
                    "how": "host-fed loop per rank: each step's local grads uploaded from pinned memory on a copy "
                           "stream while the previous step computes, then moved to the grad regions; norm read back. "
                           "Every rank uploads its own grads at once, so the aggregate host-to-device rate "
                           "(h2d_aggregate_gbs) bounds the loop as N grows"},
            "clocks": clk.summary() if rank == 0 else None,
            "gpu_launches": int(allv[:, 3].sum()),
            "zero1_adamw_sweep": zero1,
        }
        return line
    finally:
        held["graph"] = None   # a graph holding NCCL calls must be gone before destroy_process_group, or the exit waits
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()


def _ns_flops(shape) -> float:
    """The reference algorithm's FLOPs of one Newton-Schulz iteration of one parameter."""
    return configs.Workload("one", [tuple(shape)], [], [], ns_steps=1).ns_flops()


if __name__ == "__main__":
    print(json.dumps({"note": "run through bench.py under torch.distributed.run"}))
