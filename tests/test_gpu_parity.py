"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and the reference's golden outputs.

Tolerances: the measured distance on a B200 plus a margin (the oracle runs on the CPU, whose fp32 matmul sums in
another order than the tensor cores; the library against the reference's own iteration on the B200 is bit for bit,
tests/test_gpu_ns_reference.py):
  * Newton-Schulz vs the oracle and the reference's CPU fixtures, golden shapes: 1 iteration <= 1e-4 (measured 0),
    2 iterations <= 5e-4 (measured 5.0e-5), 5 iterations <= 2e-2 (measured <= 1.5e-2), and no farther from the
    exact fp64 iteration than the oracle + 1e-3 (measured <= 4.2e-5 farther)
  * the benchmark shapes of c1/c2/c3: 1 iteration <= 1e-4 (measured <= 2.8e-5), 5 iterations <= 2e-2 (measured
    <= 1.3e-2). 5 iterations amplify the CPU's fp32 summation order 5-10x per iteration; north star's 1e-2 bar is
    stated against the reference's bf16 iteration on the B200, where the distance is 0.
  * AdamW exp_avg / exp_avg_sq and Muon momentum: 1e-6 relative per element (RMS-floored)
  * params after 10 steps: AdamW 1e-6 (RMS-floored, 1e-9 absolute); Muon 1e-2 relative Frobenius against the CPU
    oracle (the 5-iteration summation-order distance carried through 10 steps)
"""

import numpy as np
import pytest
import torch

from oracle import moteopt_oracle as O
from tests.conftest import golden, record
from tests.golden.cases import ADAM_SHAPES, ADAM_WDS, NS_CASES, ns_input
from mote_b200 import configs

pytestmark = pytest.mark.gpu

P_ATOL = 1e-9


def _close(a, b, rel, atol=0.0):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    rms = float(np.sqrt(np.mean(b * b))) if b.size else 0.0
    return int((np.abs(a - b) > rel * np.maximum(np.abs(b), rms) + atol).sum())


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mote_b200 import ops  # noqa: F401  (loads libmoteopt.so: fails loudly if it is missing)
    return torch.device("cuda", 0)


def _ns_gpu(u: np.ndarray, steps: int, dev) -> np.ndarray:
    from mote_b200 import ops
    out = ops.newton_schulz(torch.from_numpy(u).to(dev), steps=steps)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def _status_ok(dev):
    from mote_b200 import ops
    st, _ = ops.read_status(dev)
    assert st & 3 == 0, f"kernel status {st}"


@pytest.mark.parametrize("name,shape,seed", NS_CASES)
def test_newton_schulz_matches_oracle_and_reference(dev, name, shape, seed):
    ref = golden("ns_reference")
    u = ns_input(shape, seed)
    exact = O.newton_schulz_f64(u, 5)
    seen = {}
    for steps, tol in ((1, 1e-4), (2, 5e-4), (5, 2e-2)):
        g = _ns_gpu(u, steps, dev)
        o = O.newton_schulz(u, steps)
        r = O.bf16_from_bits(ref[f"{name}_s{steps}"]).reshape(shape)
        seen.update({f"k_o_{steps}": O.rel_frob(g, o), f"k_ref_{steps}": O.rel_frob(g, r)})
        if steps == 5:
            seen.update(k_e=O.rel_frob(g, exact), o_e=O.rel_frob(o, exact), ref_e=O.rel_frob(r, exact))
        record("ns_vs_oracle_and_fixture", name, seen)
        assert O.rel_frob(g, o) <= tol, (name, steps, O.rel_frob(g, o))
        assert O.rel_frob(g, r) <= tol, (name, steps, O.rel_frob(g, r))
        if steps == 5:
            assert O.rel_frob(g, exact) <= O.rel_frob(o, exact) + 1e-3
    _status_ok(dev)


@pytest.mark.parametrize("shape", [(4, 768, 768), (2, 768, 3072), (2, 3072, 768), (2, 512, 2048), (1, 1000, 264),
                                   (1, 1100, 1300),
                                   # the c2 (1024^2, 1024 x 4096) and c3 (768 x 2048 expert) matrix shapes
                                   (2, 1024, 1024), (1, 1024, 4096), (1, 4096, 1024), (1, 768, 2048), (1, 2048, 768)])
def test_newton_schulz_benchmark_shapes(dev, shape):
    u = ns_input(shape, 123)
    seen = {}
    for steps, tol in ((1, 1e-4), (5, 2e-2)):
        g = _ns_gpu(u, steps, dev)
        o = O.newton_schulz(u, steps)
        seen[f"k_o_{steps}"] = O.rel_frob(g, o)
        record("ns_benchmark_shapes_vs_oracle", "x".join(map(str, shape)), seen)
        assert O.rel_frob(g, o) <= tol, (shape, steps, O.rel_frob(g, o))
    assert O.rel_frob(g, O.newton_schulz_f64(u, 5)) <= O.rel_frob(o, O.newton_schulz_f64(u, 5)) + 3e-3
    _status_ok(dev)


@pytest.mark.parametrize("shape", [(4, 768, 768), (2, 768, 3072), (1, 1100, 1300), (3, 130, 72), (37, 768, 3072)])
def test_newton_schulz_launch_modes_agree(dev, shape):
    """One persistent cooperative launch (completion counters between phases) and one launch per phase compute
    the same bits, for 1 and 5 iterations. 37 x 768 x 3072 is an iteration of 24 waves of tiles, where the
    persistent launch takes the matrices in two runs (18 and 19)."""
    from mote_b200 import _lib as L
    from mote_b200 import ops
    u = torch.from_numpy(ns_input(shape, 77)).to(dev)
    prev = L.lib.moteopt_ns_set_persistent(0)
    try:
        a = [ops.newton_schulz(u, s) for s in (1, 5)]
        L.lib.moteopt_ns_set_persistent(1)
        b = [ops.newton_schulz(u, s) for s in (1, 5)]
    finally:
        L.lib.moteopt_ns_set_persistent(prev)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    _status_ok(dev)


@pytest.mark.parametrize("shape", [(2, 3072, 768), (1, 4096, 1024), (3, 2048, 768), (2, 520, 264), (4, 136, 72),
                                   (3, 130, 72)])
def test_tall_matrices_iterated_as_stored_equal_the_transposed_iteration(dev, shape):
    """A matrix with more rows than columns iterated in its stored layout (A = X^T X, X' = a X + X B; the default)
    gives the bits of its transpose's iteration, for 1 and 5 iterations and both launch modes; shapes not a multiple
    of 8 (130 x 72) keep the transposed path either way."""
    from mote_b200 import _lib as L
    from mote_b200 import ops
    u = torch.from_numpy(ns_input(shape, 91)).to(dev)
    prev_tall = L.lib.moteopt_ns_set_tall(1)
    prev_mode = L.lib.moteopt_ns_set_persistent(-1)
    try:
        out = {}
        for tall in (1, 0):
            L.lib.moteopt_ns_set_tall(tall)
            for mode in (1, 0):
                L.lib.moteopt_ns_set_persistent(mode)
                out[(tall, mode)] = [ops.newton_schulz(u, s) for s in (1, 5)]
    finally:
        L.lib.moteopt_ns_set_tall(prev_tall)
        L.lib.moteopt_ns_set_persistent(prev_mode)
    for key, v in out.items():
        for x, y in zip(v, out[(0, 1)]):
            assert torch.equal(x, y), key
    _status_ok(dev)


def test_c1_muon_set_tall_and_transposed_agree(dev):
    """c1's Muon step (12 of its 80 matrices are 3072 x 768) with tall matrices iterated as stored (flat normalise and
    apply passes) equals the step with them transposed, bit for bit, params and momentum."""
    from mote_b200 import _lib as L
    from mote_b200 import configs
    from mote_b200.functional import MuonItem, muon_step
    w = configs.CONFIGS["c1"]()
    gen = torch.Generator(device=dev)
    gen.manual_seed(8)
    base = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in w.muon_shapes]
    grads = [(torch.randn(s, generator=gen, device=dev) * 1e-3).to(torch.bfloat16) for s in w.muon_shapes]
    out = []
    prev = L.lib.moteopt_ns_set_tall(1)
    try:
        for tall in (1, 0):
            L.lib.moteopt_ns_set_tall(tall)
            ps = [b.clone() for b in base]
            bufs = [torch.zeros_like(p) for p in ps]
            items = [MuonItem(p, g, m, 0.02, 0.002) for p, g, m in zip(ps, grads, bufs)]
            for _ in range(2):
                muon_step(items, ns_steps=5)
            torch.cuda.synchronize()
            out.append((ps, bufs))
    finally:
        L.lib.moteopt_ns_set_tall(prev)
    for a, b in zip(out[0][0] + out[0][1], out[1][0] + out[1][1]):
        assert torch.equal(a, b)
    _status_ok(dev)


def test_c1_muon_set_launch_modes_agree(dev):
    """c1's 80 matrices (three shape groups, 32 waves of tiles per iteration: the persistent launch runs them in two
    runs) step to the same bits in both launch modes."""
    from mote_b200 import _lib as L
    from mote_b200 import configs
    from mote_b200.functional import MuonItem, muon_step
    w = configs.CONFIGS["c1"]()
    gen = torch.Generator(device=dev)
    gen.manual_seed(6)
    base = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in w.muon_shapes]
    grads = [(torch.randn(s, generator=gen, device=dev) * 1e-3).to(torch.bfloat16) for s in w.muon_shapes]
    out = []
    prev = L.lib.moteopt_ns_set_persistent(0)
    try:
        for mode in (0, 1):
            L.lib.moteopt_ns_set_persistent(mode)
            ps = [b.clone() for b in base]
            items = [MuonItem(p, g, torch.zeros_like(p), 0.02, 0.002) for p, g in zip(ps, grads)]
            muon_step(items, ns_steps=5)
            torch.cuda.synchronize()
            out.append(ps)
    finally:
        L.lib.moteopt_ns_set_persistent(prev)
    for a, b in zip(*out):
        assert torch.equal(a, b)
    _status_ok(dev)


def test_muon_step_many_groups_launch_modes_agree(dev):
    """More shape groups than one launch holds (8) and a 600-matrix stack (groups of <= 512): several launch sets,
    each with its own counters, in both modes."""
    from mote_b200 import _lib as L
    from mote_b200.functional import MuonItem, muon_step
    shapes = [(64, 64), (64, 96), (96, 64), (128, 64), (64, 128), (200, 72), (72, 200), (256, 256), (40, 300),
              (600, 32, 32), (3, 520, 264)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    base = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in shapes]
    grads = [torch.randn(s, generator=gen, device=dev) * 1e-3 for s in shapes]
    out = []
    prev = L.lib.moteopt_ns_set_persistent(0)
    try:
        for mode in (0, 1):
            L.lib.moteopt_ns_set_persistent(mode)
            ps = [b.clone() for b in base]
            bufs = [torch.zeros_like(b) for b in base]
            items = [MuonItem(p, g, m, 0.02, 0.002) for p, g, m in zip(ps, grads, bufs)]
            for _ in range(2):
                muon_step(items, ns_steps=5)
            torch.cuda.synchronize()
            out.append(ps)
    finally:
        L.lib.moteopt_ns_set_persistent(prev)
    for a, b in zip(*out):
        assert torch.equal(a, b)
    _status_ok(dev)


def test_muon_step_forty_shapes_matches_oracle(dev):
    """40 distinct shapes, wide (flat normalise / apply) and tall (tiled, transposing) mixed, through muon_step,
    against the oracle's Muon step after one Newton-Schulz iteration."""
    from mote_b200.functional import MuonItem, muon_step
    rng = np.random.default_rng(11)
    shapes = [(8 + 3 * k, 16 + 5 * (k % 7)) if k % 2 else (24 + 5 * (k % 9), 8 + 3 * k) for k in range(40)]
    shapes += [(64, 16384 + 64), (16384 + 64, 64)]   # more than one 16K-element chunk, ragged last chunk
    p0 = [(rng.standard_normal(sh, dtype=np.float32) * np.float32(0.02)) for sh in shapes]
    gr = [O.bf16_round(rng.standard_normal(sh, dtype=np.float32) * np.float32(1e-3)) for sh in shapes]
    ps = _to(dev, p0)
    gs = _to(dev, gr)
    bufs = [torch.zeros_like(p) for p in ps]
    muon_step([MuonItem(p, g, b, 0.02, 0.002, 0.95, True) for p, g, b in zip(ps, gs, bufs)], ns_steps=1)
    torch.cuda.synchronize()
    ref = [p.copy() for p in p0]
    rbufs = [None] * len(ref)
    O.muon_step(ref, gr, rbufs, O.MuonGroup(lr=0.02, weight_decay=0.1, ns_steps=1))
    for i in range(len(shapes)):
        d_gpu = ps[i].cpu().numpy() - p0[i]
        d_ref = ref[i] - p0[i]
        assert O.rel_frob(d_gpu, d_ref) <= 2e-3, (shapes[i], O.rel_frob(d_gpu, d_ref))
        assert _close(bufs[i].cpu().numpy(), rbufs[i], 1e-6) == 0
    _status_ok(dev)


def test_expert_stacks_with_zipf_grads_match_oracle(dev):
    """c3's 3-D MoE expert stacks (mote/train/muon.py:59-72 reshapes them to (-1, m, n)), both orientations, with each
    expert's grad scaled by its Zipf(1.1) token factor, through the whole step: momentum buffers to 1e-6, param
    deltas to 2e-3 after one Newton-Schulz iteration."""
    from mote_b200.functional import MuonItem, muon_step
    w = configs.c3()
    e = 4
    shapes = [(e,) + s[1:] for s in w.muon_shapes]
    scale = np.asarray(w.grad_scale[:e], np.float32)[:, None, None]
    rng = np.random.default_rng(31)
    p0 = [rng.standard_normal(sh, dtype=np.float32) * np.float32(0.02) for sh in shapes]
    gr = [O.bf16_round(rng.standard_normal(sh, dtype=np.float32) * np.float32(1e-3) * scale) for sh in shapes]
    ps, gs = _to(dev, p0), _to(dev, gr)
    bufs = [torch.zeros_like(p) for p in ps]
    for _ in range(2):   # the second step runs on a non-zero momentum buffer
        muon_step([MuonItem(p, g, b, 0.02, 0.002, 0.95, True) for p, g, b in zip(ps, gs, bufs)], ns_steps=1)
    torch.cuda.synchronize()
    ref = [p.copy() for p in p0]
    rbufs = [None] * len(ref)
    for _ in range(2):
        O.muon_step(ref, gr, rbufs, O.MuonGroup(lr=0.02, weight_decay=0.1, ns_steps=1))
    for i in range(len(shapes)):
        d_gpu = ps[i].cpu().numpy() - p0[i]
        d_ref = ref[i] - p0[i]
        assert O.rel_frob(d_gpu, d_ref) <= 2e-3, (shapes[i], O.rel_frob(d_gpu, d_ref))
        assert _close(bufs[i].cpu().numpy(), rbufs[i], 1e-6) == 0
    _status_ok(dev)


def test_update_out_then_apply_equals_in_step_apply(dev):
    """The sharded step's exchange: Muon updates written out (moteopt_optimizer_step_with_coef_out) and applied by
    moteopt_muon_apply give the same bits as moteopt_optimizer_step's own apply (wide, tall, padded, 3-D)."""
    from mote_b200.distributed import cuda_compute
    from mote_b200.functional import AdamWItem, MuonItem, optimizer_step
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    shapes = [(40, 96), (96, 40), (37, 53), (2, 48, 64), (768, 3072), (3072, 768)]
    p0 = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in shapes]
    g = [(torch.randn(s, generator=gen, device=dev) * 1e-3).to(torch.bfloat16) for s in shapes]
    a0 = torch.randn(300, generator=gen, device=dev) * 0.02
    ag = (torch.randn(300, generator=gen, device=dev) * 1e-3).to(torch.bfloat16)

    def items(ps, bufs, pa, m, v):
        return ([MuonItem(p, gr, b, 0.02, 0.002) for p, gr, b in zip(ps, g, bufs)],
                [AdamWItem(pa, ag, m, v, 3e-4, 0.1, 1)])
    ps1, bufs1 = [p.clone() for p in p0], [torch.zeros_like(p) for p in p0]
    pa1, m1, v1 = a0.clone(), torch.zeros_like(a0), torch.zeros_like(a0)
    mu, ad = items(ps1, bufs1, pa1, m1, v1)
    optimizer_step(mu, ad, betas=(0.9, 0.95))
    ps2, bufs2 = [p.clone() for p in p0], [torch.zeros_like(p) for p in p0]
    pa2, m2, v2 = a0.clone(), torch.zeros_like(a0), torch.zeros_like(a0)
    mu2, ad2 = items(ps2, bufs2, pa2, m2, v2)
    outs = [torch.empty(s, dtype=torch.bfloat16, device=dev) for s in shapes]
    comp = cuda_compute(betas=(0.9, 0.95))
    comp.update(mu2, ad2, None, None, outs)
    for p, q in zip(ps2, p0):   # the params are not touched before the apply
        assert torch.equal(p, q)
    comp.apply(mu2, outs)
    torch.cuda.synchronize()
    for x, y in zip(ps1 + bufs1 + [pa1, m1, v1], ps2 + bufs2 + [pa2, m2, v2]):
        assert torch.equal(x, y)
    _status_ok(dev)


def test_muon_step_without_iterations_matches_oracle(dev):
    """ns_steps = 0: Muon applies the normalised momentum itself (muon.py:32-36 with no iteration), wide, tall, padded
    and 3-D parameters."""
    from mote_b200.functional import MuonItem, muon_step
    rng = np.random.default_rng(21)
    shapes = [(64, 96), (96, 64), (37, 53), (2, 40, 72)]
    p0 = [(rng.standard_normal(sh, dtype=np.float32) * np.float32(0.02)) for sh in shapes]
    gr = [O.bf16_round(rng.standard_normal(sh, dtype=np.float32) * np.float32(1e-3)) for sh in shapes]
    ps, gs = _to(dev, p0), _to(dev, gr)
    bufs = [torch.zeros_like(p) for p in ps]
    muon_step([MuonItem(p, g, b, 0.02, 0.002, 0.95, True) for p, g, b in zip(ps, gs, bufs)], ns_steps=0)
    torch.cuda.synchronize()
    ref = [p.copy() for p in p0]
    rbufs = [None] * len(ref)
    O.muon_step(ref, gr, rbufs, O.MuonGroup(lr=0.02, weight_decay=0.1, ns_steps=0))
    for i in range(len(shapes)):
        d_gpu, d_ref = ps[i].cpu().numpy() - p0[i], ref[i] - p0[i]
        assert O.rel_frob(d_gpu, d_ref) <= 1e-3, (shapes[i], O.rel_frob(d_gpu, d_ref))   # bf16 X0: a norm ulp can flip a rounding
    _status_ok(dev)


def test_captured_step_with_a_learning_rate_schedule(dev):
    """CapturedStep(dynamic_lr=True): one graph replayed under a changing lr (set_lrs before each replay, plain and
    Muon-SW decay rules) == eager steps built with each step's lr and decay as the reference computes them
    (muon.py:76-79), bit for bit."""
    from mote_b200.functional import AdamWItem, CapturedStep, MuonItem, optimizer_step
    w = configs.c0()
    sets = []
    for _ in range(2):
        inp = configs.make_params(w, seed=4)
        mp, ap = _to(dev, inp.muon_params), _to(dev, inp.adam_params)
        ag_np, mg_np = configs.make_grads(w, seed=4, step=0)
        mg = [torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in mg_np]
        ag = [torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in ag_np]
        sets.append((mp, ap, mg, ag, [torch.zeros_like(p) for p in mp], [torch.zeros_like(p) for p in ap],
                     [torch.zeros_like(p) for p in ap]))
    wd, lr_max = 0.1, 0.05
    sw = [i % 2 == 1 for i in range(len(w.muon_shapes))]   # every other Muon param on the Muon-SW rule
    sched = [(0.02, 3e-4), (0.015, 2e-4), (0.03, 1e-4), (0.005, 5e-5)]

    def decay(e, i):
        return (e * e / lr_max if sw[i] else e) * wd

    mp, ap, mg, ag, mb, am, av = sets[0]
    for k, (lm, la) in enumerate(sched):
        optimizer_step([MuonItem(p, g, b, lm, decay(lm, i)) for i, (p, g, b) in enumerate(zip(mp, mg, mb))],
                       [AdamWItem(p, g, m, v, la, 0.1, k + 1) for p, g, m, v in zip(ap, ag, am, av)],
                       betas=(0.9, 0.95), max_norm=0.01)
    mp2, ap2, mg2, ag2, mb2, am2, av2 = sets[1]
    lm0, la0 = sched[0]
    cs = CapturedStep([MuonItem(p, g, b, lm0, decay(lm0, i), wd=wd, lr_max=lr_max if sw[i] else 0.0)
                       for i, (p, g, b) in enumerate(zip(mp2, mg2, mb2))],
                      [AdamWItem(p, g, m, v, la0, 0.1, 0) for p, g, m, v in zip(ap2, ag2, am2, av2)],
                      betas=(0.9, 0.95), max_norm=0.01, dynamic_lr=True)
    for lm, la in sched:
        cs.set_lrs([la] * len(ap2), [lm] * len(mp2))
        cs()
    torch.cuda.synchronize()
    assert cs.graph is not None
    for a, b in zip(mp + ap + mb + am + av, mp2 + ap2 + mb2 + am2 + av2):
        assert torch.equal(a, b)


def test_newton_schulz_fp32_and_bf16_inputs_agree(dev):
    from mote_b200 import ops
    u = torch.from_numpy(O.bf16_round(ns_input((3, 96, 200), 9))).to(dev)
    a = ops.newton_schulz(u, 5)
    b = ops.newton_schulz(u.to(torch.bfloat16), 5)
    assert torch.equal(a, b)


def _to(dev, xs):
    return [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in xs]


def test_full_step_c0_ten_steps_matches_oracle(dev):
    """train.py:944-947 on the c0 workload through the C ABI (bf16 grads), 10 steps, against the oracle."""
    from mote_b200.functional import AdamWItem, MuonItem, optimizer_step
    w = configs.c0()
    inp = configs.make_params(w, seed=0)
    ap = _to(dev, inp.adam_params)
    mp = _to(dev, inp.muon_params)
    am = [torch.zeros_like(p) for p in ap]
    av = [torch.zeros_like(p) for p in ap]
    mb = [torch.zeros_like(p) for p in mp]
    nd = len(w.adam_decay_shapes)
    st = O.StepState()
    st.muon_bufs = [None] * len(mp)
    st.exp_avgs = [np.zeros_like(p) for p in inp.adam_params]
    st.exp_avg_sqs = [np.zeros_like(p) for p in inp.adam_params]
    st.adam_steps = [0] * len(ap)
    mg = O.MuonGroup(lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True, weight_decay=w.muon_wd, ns_steps=w.ns_steps)
    div = 4.0
    for step in range(10):
        ag_np, mg_np = configs.make_grads(w, seed=0, step=step)
        ag = [torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in ag_np]
        mgg = [torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in mg_np]
        muon = [MuonItem(p, g, b, w.muon_lr, w.muon_lr * w.muon_wd, w.muon_momentum, True) for p, g, b in zip(mp, mgg, mb)]
        adam = [AdamWItem(p, g, m, v, w.adam_lr, w.adam_wd if i < nd else 0.0, step + 1)
                for i, (p, g, m, v) in enumerate(zip(ap, ag, am, av))]
        norm = optimizer_step(muon, adam, ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip,
                              grad_divisor=div)
        # oracle
        allg = [x.copy() for x in ag_np] + [x.copy() for x in mg_np]
        for x in allg:
            x[...] = (x / np.float32(div)).astype(np.float32)
        total = O.clip_grad_norm(allg, w.clip)
        for i in range(len(ap)):
            st.adam_steps[i] += 1
            O.adamw_update(inp.adam_params[i], allg[i], st.exp_avgs[i], st.exp_avg_sqs[i], w.adam_lr, w.betas[0],
                           w.betas[1], w.eps, w.adam_wd if i < nd else 0.0, st.adam_steps[i])
        O.muon_step(inp.muon_params, allg[len(ap):], st.muon_bufs, mg)
        assert _close(norm.item(), total, 1e-6) == 0, (norm.item(), total)
        if step in (0, 9):
            for i in range(len(ap)):
                assert _close(am[i].cpu().numpy(), st.exp_avgs[i], 1e-6) == 0
                assert _close(av[i].cpu().numpy(), st.exp_avg_sqs[i], 1e-6) == 0
                assert _close(ap[i].cpu().numpy(), inp.adam_params[i], 1e-6, atol=P_ATOL) == 0
            for i in range(len(mp)):
                assert _close(mb[i].cpu().numpy(), st.muon_bufs[i], 1e-6) == 0
                assert O.rel_frob(mp[i].cpu().numpy(), inp.muon_params[i]) < 1e-2, (step, i)
    _status_ok(dev)


def test_adamw_and_clip_match_reference(dev):
    """The AdamW/clip fixture of the reference (5 steps, clip active) through the C ABI."""
    from mote_b200.functional import AdamWItem, optimizer_step
    g = golden("adamw_reference")
    n = len(ADAM_SHAPES)
    ps = _to(dev, [g[f"p0_{i}"] for i in range(n)])
    ms = [torch.zeros_like(p) for p in ps]
    vs = [torch.zeros_like(p) for p in ps]
    for step in range(5):
        grads = _to(dev, [g[f"g{step}_{i}"] for i in range(n)])
        items = [AdamWItem(ps[i], grads[i], ms[i], vs[i], 3e-4, ADAM_WDS[i], step + 1) for i in range(n)]
        norm = optimizer_step((), items, betas=(0.9, 0.95), eps=1e-8, max_norm=0.05)
        assert _close(norm.item(), g[f"norm{step}"], 1e-5) == 0
        if step in (0, 4):
            for i in range(n):
                # torch's CPU norm sits a few ulp off the exact one; through v ~ coef^2 that is ~1e-6 (test docstring)
                assert _close(ms[i].cpu().numpy(), g[f"m{step + 1}_{i}"], 1e-5) == 0
                assert _close(vs[i].cpu().numpy(), g[f"v{step + 1}_{i}"], 1e-5) == 0
                assert _close(ps[i].cpu().numpy(), g[f"p{step + 1}_{i}"], 1e-5, atol=P_ATOL) == 0
    _status_ok(dev)


def test_clip_grad_norm_matches_oracle(dev):
    from mote_b200 import ops
    rng = np.random.default_rng(5)
    shapes = [(1000, 3), (17,), (4, 4, 4), (70000,)]
    gs = [O.bf16_round(rng.standard_normal(s).astype(np.float32)) for s in shapes]
    for dt in (torch.float32, torch.bfloat16):
        params = [torch.nn.Parameter(torch.zeros(s, device=dev, dtype=dt)) for s in shapes]
        for p, x in zip(params, gs):
            p.grad = torch.from_numpy(x).to(dev).to(dt)
        ref = [x.copy() for x in gs]
        tot = O.clip_grad_norm(ref, 1.0)
        n = ops.clip_grad_norm_(params, 1.0)
        assert _close(n.item(), tot, 1e-6) == 0
        for p, r in zip(params, ref):
            got = p.grad.float().cpu().numpy()
            want = r if dt == torch.float32 else O.bf16_round(r)
            assert _close(got, want, 1e-6 if dt == torch.float32 else 1e-2) == 0


def test_muon_batched_reference_case(dev):
    """tests/test_muon_batched.py:46-67 of the reference through the C ABI, against its stored result."""
    from mote_b200.functional import MuonItem, muon_step
    g = golden("muon_reference")
    for sw in (0, 1):
        ps = _to(dev, [g[f"batched_p0_{i}"] for i in range(6)])
        bufs = [torch.zeros_like(p) for p in ps]
        for it in range(3):
            grads = _to(dev, [(g[f"batched_g_{i}"] * np.float32(1.0 + 0.1 * it)).astype(np.float32) for i in range(6)])
            lr, wd, lr_max = 1e-2, 0.1, 2e-2
            decay = (lr * lr / lr_max if sw else lr) * wd
            muon_step([MuonItem(p, gr, b, lr, decay, 0.95, True) for p, gr, b in zip(ps, grads, bufs)])
        for i in range(6):
            ref_p = g[f"batched_sw{sw}_p3_{i}"]
            got = ps[i].cpu().numpy()
            assert np.allclose(got, ref_p, atol=2e-3, rtol=1e-2)
            assert _close(bufs[i].cpu().numpy(), g[f"batched_sw{sw}_buf_{i}"], 1e-6) == 0


def test_step_is_bitwise_deterministic(dev):
    from mote_b200.functional import AdamWItem, MuonItem, optimizer_step
    w = configs.c0()
    outs = []
    for _ in range(2):
        inp = configs.make_params(w, seed=1)
        mp = _to(dev, inp.muon_params)
        ap = _to(dev, inp.adam_params)
        mb = [torch.zeros_like(p) for p in mp]
        am = [torch.zeros_like(p) for p in ap]
        av = [torch.zeros_like(p) for p in ap]
        norms = []
        for step in range(3):
            ag, mg = configs.make_grads(w, seed=1, step=step)
            muon = [MuonItem(p, torch.from_numpy(x).to(dev), b, 0.02, 0.002) for p, x, b in zip(mp, mg, mb)]
            adam = [AdamWItem(p, torch.from_numpy(x).to(dev), m, v, 3e-4, 0.1, step + 1)
                    for p, x, m, v in zip(ap, ag, am, av)]
            norms.append(optimizer_step(muon, adam, betas=(0.9, 0.95), max_norm=0.01).item())
        outs.append(([p.cpu() for p in mp + ap + mb + am + av], norms))
    for a, b in zip(outs[0][0], outs[1][0]):
        assert torch.equal(a, b)
    assert outs[0][1] == outs[1][1]


def test_captured_step_replays_equal_eager_steps(dev):
    """CapturedStep (one CUDA graph of the whole step, AdamW's step count on the device) == eager optimizer_step."""
    from mote_b200.functional import AdamWItem, CapturedStep, MuonItem, optimizer_step
    w = configs.c0()
    sets = []
    for _ in range(2):
        inp = configs.make_params(w, seed=3)
        mp = _to(dev, inp.muon_params)
        ap = _to(dev, inp.adam_params)
        ag_np, mg_np = configs.make_grads(w, seed=3, step=0)
        mg = [torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in mg_np]
        ag = [torch.from_numpy(x).to(dev).to(torch.bfloat16) for x in ag_np]
        sets.append((mp, ap, mg, ag, [torch.zeros_like(p) for p in mp], [torch.zeros_like(p) for p in ap],
                     [torch.zeros_like(p) for p in ap]))
    mp, ap, mg, ag, mb, am, av = sets[0]
    norms_eager = []
    for k in range(4):
        norms_eager.append(optimizer_step([MuonItem(p, g, b, 0.02, 0.002) for p, g, b in zip(mp, mg, mb)],
                                          [AdamWItem(p, g, m, v, 3e-4, 0.1, k + 1) for p, g, m, v in zip(ap, ag, am, av)],
                                          betas=(0.9, 0.95), max_norm=0.01).item())
    mp2, ap2, mg2, ag2, mb2, am2, av2 = sets[1]
    cs = CapturedStep([MuonItem(p, g, b, 0.02, 0.002) for p, g, b in zip(mp2, mg2, mb2)],
                      [AdamWItem(p, g, m, v, 3e-4, 0.1, 0) for p, g, m, v in zip(ap2, ag2, am2, av2)],
                      betas=(0.9, 0.95), max_norm=0.01)
    norms_graph = [cs().item() for _ in range(4)]
    assert cs.graph is not None and cs.launches_per_step > 0
    assert norms_graph == norms_eager
    for a, b in zip(mp + ap + mb + am + av, mp2 + ap2 + mb2 + am2 + av2):
        assert torch.equal(a, b)
    assert cs.device_step.item() == 4.0


def test_adamw_large_launch_equals_small_launches(dev):
    """AdamW picks its work unit per launch: 16K-element units when the launch fills the GPU in them, 2K otherwise.
    A 10.5M-element tensor in one call (16K units) and the same tensor in four calls of 2.6M (2K units) must give
    the same bits, with a grad divisor and the fused EMA, over three steps."""
    from mote_b200.functional import AdamWItem, optimizer_step
    n, parts = 10_500_000, 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(31)
    p0 = torch.randn(n, generator=gen, device=dev) * 0.02
    ga = [(torch.randn(n, generator=gen, device=dev) * 1e-3).to(torch.bfloat16) for _ in range(3)]
    big = [p0.clone(), torch.zeros(n, device=dev), torch.zeros(n, device=dev), p0.clone()]
    small = [t.clone() for t in big]
    cut = [k * (n // parts) for k in range(parts)] + [n]
    for step in range(3):
        p, m, v, e = big
        optimizer_step((), [AdamWItem(p, ga[step], m, v, 3e-4, 0.1, step + 1)], betas=(0.9, 0.95),
                       grad_divisor=3.0, ema=[e], ema_weight=0.1)
        for a, b in zip(cut, cut[1:]):
            p, m, v, e = (t[a:b] for t in small)
            optimizer_step((), [AdamWItem(p, ga[step][a:b], m, v, 3e-4, 0.1, step + 1)], betas=(0.9, 0.95),
                           grad_divisor=3.0, ema=[e], ema_weight=0.1)
    torch.cuda.synchronize()
    for x, y in zip(big, small):
        assert torch.equal(x, y)
