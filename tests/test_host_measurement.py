"""The measurement arithmetic on the CPU: the per-step algorithmic work of each workload (the units the roofline
figures in bench.py divide by) against the figures the reference's step is quoted with, the issued tensor-core work
against an explicit enumeration of the kernel's tile schedule, and the step roofline's formula."""

import pytest

from mote_b200 import configs


@pytest.mark.parametrize("name,tflop,gb,elems", [
    ("c1", 1.727, 1.877, 93.3e6),    # 12 x {4 x 768^2, 768 x 3072, 3072 x 768} + 8 x 512 x 2048 Muon, ~0.36 M AdamW
    ("c2", 14.43, 10.74, 536.9e6),   # 256 x 1024^2 + 64 x 1024 x 4096
    ("c3", 3.67, 4.03, 201.3e6),     # 64 x 768 x 2048 + 64 x 2048 x 768 expert stacks
])
def test_workload_figures(name, tflop, gb, elems):
    """FLOPs = sum 5 (4 s^2 l + 2 s^3) over the matrices (s, l = short, long side); bytes = 20 per Muon element and
    28 per AdamW element."""
    w = configs.CONFIGS[name]()
    assert w.ns_flops() / 1e12 == pytest.approx(tflop, rel=1e-3)
    assert w.state_bytes() / 1e9 == pytest.approx(gb, rel=1e-3)
    assert w.numel()[0] == pytest.approx(elems, rel=1e-3)


def _issued_by_enumeration(w, tile=256):
    """Walk the kernel's schedule tile by tile: per iteration the Gram (X X^T, K = l) and polynomial (A A, K = s)
    phases compute the output blocks on and above the diagonal, the update (B X, K = s) every block of X; a block
    clipped at the matrix edge does only its valid rows and columns."""
    tot = 0.0
    for shape in w.muon_shapes:
        batch = shape[0] if len(shape) == 3 else 1
        s, l = min(shape[-2:]), max(shape[-2:])
        rows = [min(tile, s - i) for i in range(0, s, tile)]
        cols = [min(tile, l - j) for j in range(0, l, tile)]
        for bi, r in enumerate(rows):
            for bj, c in enumerate(rows):
                if bj >= bi:
                    tot += batch * w.ns_steps * (2.0 * r * c * l + 2.0 * r * c * s)
            for c in cols:
                tot += batch * w.ns_steps * 2.0 * r * c * s
    return tot


@pytest.mark.parametrize("name", ["c0", "c1", "c2", "c3"])
def test_issued_tensor_work_matches_the_tile_schedule(name):
    w = configs.CONFIGS[name]()
    assert w.ns_flops_issued() == pytest.approx(_issued_by_enumeration(w), rel=1e-12)
    assert w.ns_flops_issued() <= w.ns_flops()


def test_c1_issued_work_and_tiles():
    w = configs.c1()
    assert w.ns_flops_issued() == pytest.approx(1.3878e12, rel=1e-4)   # the figure the NS profile divides by
    assert w.ns_tiles_per_iter() == 2336


def test_step_roofline_formula():
    from mote_b200.measure import step_roofline
    peaks = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0}
    r = step_roofline(1.727e12, 1.877e9, 0.0, peaks, ms=2.0)
    assert r["sustained"]["roofline_ms"] == pytest.approx(1.727e12 / 1.4e15 * 1e3, rel=1e-3)   # FLOP-bound
    assert r["burst"]["frac"] == pytest.approx(1.727e12 / 1.6e15 * 1e3 / 2.0, rel=1e-3)
    # an exchange adds its NVLink time (770 GB/s per direction) on top of the slower of the two bounds
    r = step_roofline(1e9, 6.5e9, 0.77e9, peaks, ms=2.0)
    assert r["sustained"]["roofline_ms"] == pytest.approx(1.0 + 1.0, rel=1e-3)


@pytest.mark.parametrize("config", ["c0", "c4_small"])
def test_reference_arm_line(config, monkeypatch):
    """`bench.py --impl reference`: the reference's own torch step on the host (oracle/torch_port.py), whole steps,
    one JSON line with the contract's keys and the same `config` dict as the library's line for that workload; a
    workload without Muon matrices times its clip + AdamW step."""
    import argparse

    import bench
    if config == "c4_small":
        monkeypatch.setitem(configs.CONFIGS, "c4_small", lambda: configs.c4(200_000))
    args = argparse.Namespace(steps=4, warmup=1, config=config)
    line = bench.run_reference(args, rank=0, world=1)
    assert line["impl"] == "reference" and line["unit"] == "ms/step" and line["higher_is_better"] is False
    assert line["value"] > 0 and line["value"] == line["ms_per_step"] == line["e2e"]["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and "torch_port" in cb["sample"]
    assert "4 whole steps" in cb["sample"]
    from mote_b200.measure import bench_config
    assert line["config"] == bench_config(configs.CONFIGS[config](), 1)


def test_cpu_baseline_times_whole_reference_steps():
    """The GPU arm's cpu_baseline: whole reference steps over every Muon param and AdamW tensor of the workload,
    whose momentum buffers and AdamW state exist after the step (every tensor was stepped)."""
    import bench
    w = configs.c0()
    cb = bench.cpu_baseline_sample(w, steps=2)
    assert cb["value"] > 0 and cb["unit"] == "ms/step" and cb["kind"] == "port" and "2 whole steps" in cb["sample"]
    ref = bench.TorchReference(w)
    ref.time_step()
    assert all(b is not None for b in ref.bufs) and len(ref.bufs) == len(w.muon_shapes)
    assert all(len(ref.adam.state[p]) == 3 for p in ref.adam_p)


def test_reference_arm_under_torchrun_prints_on_rank_zero_only():
    """Under torchrun (N > 1) rank 0 alone times and prints the reference line; the other ranks exit 0 without work."""
    import json
    import os
    import subprocess
    import sys
    from tests.conftest import ROOT
    cmd = [sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "0", "--config", "c0"]
    for rank in (1, 0):
        env = {**os.environ, "RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": "2"}
        r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        if rank:
            assert lines == []
        else:
            line = json.loads(lines[-1])
            assert line["impl"] == "reference" and line["n_gpus"] == 2
