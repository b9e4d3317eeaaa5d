"""bench.py's N > 1 leg: the sharded optimizer step of mote_b200.distributed on N GPUs of one node, one process per
GPU (launched by torch.distributed.run), NCCL over NVLink.

Each rank holds the whole c1 model in its flat param regions and its own local bf16 grads; one step is the
reduce-scatter of the grads, the global clip from per-rank sums, the owned updates, and the exchange and apply of
the Muon updates (read from their owners over NVLink) with the AdamW slices all-gathered. Time is measured with CUDA
events on each rank and the maximum over ranks is reported.
"""

from __future__ import annotations

import datetime
import json
import os
import statistics
from pathlib import Path

import torch
import torch.distributed as dist

from . import configs
from .distributed import ShardedStep, capture, cuda_compute, make_plan

ROOT = Path(__file__).resolve().parent.parent
METRIC = "ms/optimizer step (96M set)"


def run(args, rank: int, world: int, local_rank: int):
    from bench import ClockSampler, load_peaks, step_roofline, streamed_e2e   # driver-facing helpers live in bench.py
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
        gen = torch.Generator(device=dev)
        gen.manual_seed(0)   # identical params on every rank
        pm = torch.zeros(plan.muon_len, dtype=torch.float32, device=dev)
        pa = torch.zeros(plan.adam_len, dtype=torch.float32, device=dev)
        nd = len(w.adam_decay_shapes)
        st = ShardedStep(plan, rank, pm, pa, torch.zeros(plan.muon_len, dtype=torch.bfloat16, device=dev),
                         torch.zeros(plan.adam_len, dtype=torch.bfloat16, device=dev),
                         cuda_compute(ns_steps=w.ns_steps, betas=w.betas, eps=w.eps), muon_lr=w.muon_lr,
                         muon_wd=w.muon_wd, momentum=w.muon_momentum, adam_lr=w.adam_lr,
                         adam_wd=[w.adam_wd if i < nd else 0.0 for i in range(len(w.adam_shapes))])
        for i in range(len(w.muon_shapes)):
            st.muon_view(pm, i).normal_(0.0, 0.02, generator=gen)
        for i in range(len(w.adam_shapes)):
            st.adam_view(pa, i).normal_(0.0, 0.02, generator=gen)
        gen.manual_seed(1000 + rank)   # local grads differ per rank
        st.gm.copy_(torch.randn(plan.muon_len, generator=gen, device=dev) * 1e-3)
        st.ga.copy_(torch.randn(plan.adam_len, generator=gen, device=dev) * 1e-3)
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
        torch.cuda.synchronize(dev)
        dist.barrier()
        l1 = L.lib.moteopt_launch_count()
        with ClockSampler(gpu_id) as clk:
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

        # end to end: this rank's local grads copied in from pinned host memory, the grad norm read back
        host_m = st.gm.cpu().pin_memory()
        host_a = st.ga.cpu().pin_memory()
        host_norm = torch.empty((), dtype=torch.float32).pin_memory()
        e2e_steps = max(5, min(30, args.steps // 6))
        pairs = [(st.gm, host_m), (st.ga, host_a)]
        streamed_e2e(run_step, pairs, host_norm, 2, stream)
        dist.barrier()
        e2e_local = streamed_e2e(run_step, pairs, host_norm, e2e_steps, stream)

        my_flops = sum(w.ns_steps * _ns_flops_issued(w.muon_shapes[i]) for i in st.mine)
        vals = torch.tensor([ms_local, e2e_local, ns_local, float(launches), my_flops], dtype=torch.float64, device=dev)
        allv = [torch.zeros_like(vals) for _ in range(world)]
        dist.all_gather(allv, vals)
        allv = torch.stack(allv).cpu()
        ms = float(allv[:, 0].max())
        e2e = float(allv[:, 1].max())
        slow = int(allv[:, 2].argmax())
        peaks, src = load_peaks()
        ns_ms = float(allv[slow, 2])
        achieved = float(allv[slow, 4]) / (ns_ms * 1e-3) / 1e12 if ns_ms > 0 else 0.0
        # per GPU: 1/N of the reference FLOPs and state bytes; received in the exchange: the other ranks' bf16 O
        o_bytes = 2.0 * w.numel()[0]
        roof = step_roofline(w.ns_flops() / world, w.state_bytes() / world, o_bytes * (world - 1) / world, peaks, ms)
        line = {
            "metric": METRIC, "value": round(ms, 4), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded params N(0,0.02^2) fp32 (same on every rank), local grads N(0,1e-3^2) bf16 per rank",
            "config": {"workload": w.name, "parallelism": f"muon-owner+zero1 x{world}",
                       "launch": "CUDA graph of the whole sharded step" if captured
                       else f"eager (graph capture failed: {capture_error})", "collectives":
                       "NCCL reduce-scatter (grads), all-gather (per-rank sums of squares), all-gather (AdamW fp32 "
                       "params); Muon updates: " + ("every rank's bf16 O read over NVLink by the apply kernel (CUDA "
                       "IPC mappings, one-element all-reduce as the ordering barrier)" if st.peer_ptrs is not None
                       else f"NCCL all-gather of bf16 O ({peer_error or 'peer mapping off'})"),
                       "l2": "inputs larger than L2; no flush"},
            "roofline": {"bound": "tensor", "kernel": "ns_gemm_kernel", "achieved": round(achieved, 1),
                         "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops_sustained"], 4), "traffic": None,
                         "peak_source": f"{src} (sustained bf16)", "frac_of_burst": round(achieved / peaks["bf16_tflops"], 4),
                         "rank": slow,
                         "ns_ms_per_step": round(ns_ms, 4)},
            "step_roofline": roof,
            "e2e": {"value": round(e2e, 4), "unit": "ms/step",
                    "h2d_bytes_per_step": int((st.gm.numel() + st.ga.numel()) * 2), "d2h_bytes_per_step": 4,
                    "how": "host-fed loop per rank: each step's local grads uploaded from pinned memory on a copy "
                           "stream while the previous step computes, then moved to the grad regions; norm read back"},
            "clocks": clk.summary(),
            "gpu_launches": int(allv[:, 3].sum()),
        }
        st.close()
        return line
    finally:
        held["graph"] = None   # a graph holding NCCL calls must be gone before destroy_process_group, or the exit waits
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()


def _ns_flops_issued(shape) -> float:
    """Tensor-core FLOPs of one Newton-Schulz iteration of one parameter (upper-triangle Gram / A A blocks)."""
    return configs.Workload("one", [tuple(shape)], [], [], ns_steps=1).ns_flops_issued()


if __name__ == "__main__":
    print(json.dumps({"note": "run through bench.py under torch.distributed.run"}))
