"""Pin the CPU oracle (oracle/moteopt_oracle.py) against the reference's own outputs stored in tests/golden/.

Tolerances:
  * Newton-Schulz at 1 and 2 iterations: <= 2e-4 / 2e-3 relative Frobenius. The oracle rounds to bf16 at every op
    exactly where the reference does; only the fp32 summation order inside a matmul differs, which flips about one
    output in 10^4 by one bf16 ulp.
  * Newton-Schulz at 5 iterations: <= 4e-2 relative Frobenius, and no farther from the exact (fp64) iteration than
    the reference itself plus 2e-3. The bf16 iteration is chaotic: a single-ulp flip grows 5-10x per iteration, so
    two correct bf16 implementations end ~1e-2 apart. The reference disagrees with itself by the same amount
    (batched vs per-matrix 8.6e-3, transposed input 2.7e-2 on 768x768; see test_reference_noise_floor_is_recorded).
  * AdamW state, params and clip norms: 1e-6 relative per element, with the tensor's RMS as the floor of the scale
    (and 1e-9 absolute for params, half an fp32 ulp at |p| = 0.02). The oracle mirrors torch's rounding op by op,
    but torch's CPU sqrt is not correctly rounded and its norm sums in another order, so a few values differ by
    one ulp, which is large relative to an element that has just cancelled to ~0.
  * Muon momentum buffers: 1e-6 relative per element; Muon params after 3 (10) steps: the reference test's own
    tolerance (atol 2e-3, rtol 1e-2, tests/test_muon_batched.py:67) and 1e-3 relative Frobenius.
"""

import numpy as np
import pytest

from tests.conftest import golden
from oracle import moteopt_oracle as O

from tests.golden.cases import (ADAM_SHAPES, ADAM_WDS, C0_DIVISOR, MOE_CASES, MOE_GAMMA, MOE_STEPS, NS_CASES, moe_bias0,
                                moe_loads, ns_input, sample_index)
from mote_b200 import configs


P_ATOL = 1e-9


def _close_rel(a, b, rel, atol=0.0):
    """Count elements with |a-b| > rel * max(|b|, rms(b)) + atol: `rel` relative per element, with the tensor's RMS
    as the floor of the scale, so an element that cancels to ~0 is judged against the tensor's own magnitude."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    rms = float(np.sqrt(np.mean(b * b))) if b.size else 0.0
    bad = np.abs(a - b) > rel * np.maximum(np.abs(b), rms) + atol
    return int(bad.sum())


@pytest.mark.parametrize("name,shape,seed", NS_CASES)
def test_ns_matches_reference(name, shape, seed):
    ref = golden("ns_reference")
    u = ns_input(shape, seed)
    exact = O.newton_schulz_f64(u, 5)
    for steps, tol in ((1, 2e-4), (2, 2e-3), (5, 4e-2)):
        r = O.bf16_from_bits(ref[f"{name}_s{steps}"]).reshape(shape)
        o = O.newton_schulz(u, steps=steps)
        err = O.rel_frob(o, r)
        assert err <= tol, (name, steps, err)
        if steps == 5:
            # the oracle is as accurate as the reference: no farther from the exact iteration
            assert O.rel_frob(o, exact) <= O.rel_frob(r, exact) + 2e-3, (name, O.rel_frob(o, exact), O.rel_frob(r, exact))


def test_muon_batched_matches_reference():
    """tests/test_muon_batched.py:46-67 through the oracle vs the reference's stored result."""
    g = golden("muon_reference")
    n = 6
    params0 = [g[f"batched_p0_{i}"] for i in range(n)]
    grads = [g[f"batched_g_{i}"] for i in range(n)]
    for sw in (0, 1):
        ps = [p.copy() for p in params0]
        bufs = [None] * n
        grp = O.MuonGroup(lr=1e-2, momentum=0.95, nesterov=True, weight_decay=0.1, sw_decay=bool(sw), lr_max=2e-2)
        for it in range(3):
            O.muon_step(ps, [(x * np.float32(1.0 + 0.1 * it)).astype(np.float32) for x in grads], bufs, grp)
        for i in range(n):
            ref_p = g[f"batched_sw{sw}_p3_{i}"]
            assert np.allclose(ps[i], ref_p, atol=2e-3, rtol=1e-2)
            assert O.rel_frob(ps[i], ref_p) < 1e-3
            assert _close_rel(bufs[i], g[f"batched_sw{sw}_buf_{i}"], 1e-6) == 0


def test_muon_stack_matches_reference():
    g = golden("muon_reference")
    p = g["stack_p0"].copy()
    bufs = [None]
    grp = O.MuonGroup(lr=1e-2, weight_decay=0.1)
    for it in range(3):
        O.muon_step([p], [(g["stack_g"] * np.float32(1 + 0.1 * it)).astype(np.float32)], bufs, grp)
    assert np.allclose(p, g["stack_p3"], atol=2e-3, rtol=1e-2)
    assert O.rel_frob(p, g["stack_p3"]) < 1e-3


def test_muon_param_lr_decay_matches_reference():
    g = golden("muon_reference")
    p = (np.eye(8, dtype=np.float32) * 3.0)
    grp = O.MuonGroup(lr=1e-2, weight_decay=0.1, param_lr={0: 5e-2})
    O.muon_step([p], [np.zeros_like(p)], [None], grp)
    assert np.array_equal(p, g["elr_decay_p1"])


def test_adamw_and_clip_match_reference():
    g = golden("adamw_reference")
    n = len(ADAM_SHAPES)
    ps = [g[f"p0_{i}"].copy() for i in range(n)]
    ms, vs, steps = [None] * n, [None] * n, [0] * n
    wds = ADAM_WDS
    for step in range(5):
        grads = [g[f"g{step}_{i}"].copy() for i in range(n)]
        total = O.grad_total_norm(grads)
        assert _close_rel(total, g[f"norm{step}"], 1e-6) == 0
        # pin the AdamW arithmetic on its own: scale by the coefficient of the reference's own norm (torch's CPU
        # norm sums in fp32 and lands a few ulp from the oracle's fp64 sum; v ~ coef^2 would carry that along)
        coef = O.clip_coef(g[f"norm{step}"], 0.05)
        for x in grads:
            x[...] = (x * coef).astype(np.float32)
        for i in range(n):
            if ms[i] is None:
                ms[i], vs[i] = np.zeros_like(ps[i]), np.zeros_like(ps[i])
            steps[i] += 1
            O.adamw_update(ps[i], grads[i], ms[i], vs[i], 3e-4, 0.9, 0.95, 1e-8, wds[i], steps[i])
        if step in (0, 4):
            for i in range(n):
                assert _close_rel(ms[i], g[f"m{step + 1}_{i}"], 1e-6) == 0, ("m", step, i)
                assert _close_rel(vs[i], g[f"v{step + 1}_{i}"], 1e-6) == 0, ("v", step, i)
                assert _close_rel(ps[i], g[f"p{step + 1}_{i}"], 1e-6, atol=P_ATOL) == 0, ("p", step, i)


def test_c0_ten_steps_match_reference():
    """The whole step of train.py:944-947 on the c0 workload, 10 steps, against the reference's stored samples.
    End to end the oracle uses its own clip norm, so AdamW state is held to 1e-5 here (the norm's few-ulp offset
    enters v squared); each piece is pinned at 1e-6 by the tests above. Params: 1e-3 relative."""
    g = golden("c0_reference")
    w = configs.c0()
    inp = configs.make_params(w, seed=0)
    st = O.StepState()
    mg = O.MuonGroup(lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True, weight_decay=w.muon_wd, ns_steps=w.ns_steps)
    for step in range(10):
        ag, mgr = configs.make_grads(w, seed=0, step=step)
        total = c0_step(inp, ag, mgr, st, mg, w)
        # torch's CPU norm accumulates in fp32 (~2e-6 off the exact value at c0's 0.8 M elements); the oracle's is
        # the fp64 sum rounded once
        assert _close_rel(total, g[f"norm{step}"], 1e-5) == 0, (step, total, g[f"norm{step}"])
        if step in (0, 9):
            for i, p in enumerate(inp.adam_params):
                idx = sample_index(p.size)
                assert _close_rel(p.ravel()[idx], g[f"ap{step + 1}_{i}"], 1e-5, atol=P_ATOL) == 0
                assert _close_rel(st.exp_avgs[i].ravel()[idx], g[f"am{step + 1}_{i}"], 1e-5) == 0
                assert _close_rel(st.exp_avg_sqs[i].ravel()[idx], g[f"av{step + 1}_{i}"], 1e-5) == 0
            for i, p in enumerate(inp.muon_params):
                idx = sample_index(p.size)
                assert _close_rel(st.muon_bufs[i].ravel()[idx], g[f"mbuf{step + 1}_{i}"], 1e-5) == 0
                ssq = float((p.astype(np.float64) ** 2).sum())
                assert abs(ssq - float(g[f"mp{step + 1}_{i}_ssq"])) <= 2e-3 * float(g[f"mp{step + 1}_{i}_ssq"])
                assert np.allclose(p.ravel()[idx], g[f"mp{step + 1}_{i}"], atol=2e-3, rtol=1e-2)
                assert O.rel_frob(p.ravel()[idx], g[f"mp{step + 1}_{i}"]) < 1e-3 * 10


def c0_step(inp, ag, mgr, st, mg, w):
    """train.py:944-947 with the c0 workload's two AdamW groups (decayed >= 2-D, undecayed vectors)."""
    n_a = len(inp.adam_params)
    if not st.muon_bufs:
        st.muon_bufs = [None] * len(inp.muon_params)
        st.exp_avgs = [np.zeros_like(p) for p in inp.adam_params]
        st.exp_avg_sqs = [np.zeros_like(p) for p in inp.adam_params]
        st.adam_steps = [0] * n_a
    allg = [x.copy() for x in ag] + [x.copy() for x in mgr]
    for x in allg:
        x[...] = (x / np.float32(C0_DIVISOR)).astype(np.float32)
    total = O.clip_grad_norm(allg, w.clip)
    nd = len(w.adam_decay_shapes)
    for i in range(n_a):
        st.adam_steps[i] += 1
        O.adamw_update(inp.adam_params[i], allg[i], st.exp_avgs[i], st.exp_avg_sqs[i], w.adam_lr, w.betas[0],
                       w.betas[1], w.eps, w.adam_wd if i < nd else 0.0, st.adam_steps[i])
    O.muon_step(inp.muon_params, allg[n_a:], st.muon_bufs, mg)
    return total


def test_reference_noise_floor_is_recorded():
    """The 5-iteration tolerance rests on the bf16 iteration's own chaos: the oracle run on the same input with the
    matrix transposed (mathematically identical) lands about as far away as the reference does from the oracle."""
    u = ns_input((2, 128, 128), 7)
    a = O.newton_schulz(u, 5)
    b = np.swapaxes(O.newton_schulz(np.ascontiguousarray(np.swapaxes(u, -1, -2)), 5), -1, -2)
    assert O.rel_frob(a, b) > 1e-3   # not bitwise: the noise floor is real


@pytest.mark.parametrize("name,experts,kind,seed", MOE_CASES)
def test_moe_update_bias_matches_reference(name, experts, kind, seed):
    """The lossfree router's bias step (mote/model/moe.py:147-159), MOE_STEPS steps: bit for bit, bias and load."""
    ref = golden("moe_reference")
    bias = moe_bias0(experts, seed)
    for step in range(MOE_STEPS):
        load = moe_loads(experts, kind, seed, step)
        O.moe_update_bias(load, bias, MOE_GAMMA)
        assert np.array_equal(bias.view(np.uint32), ref[f"{name}_bias{step}"].view(np.uint32)), (name, step)
        assert np.array_equal(load.view(np.uint32), ref[f"{name}_load{step}"].view(np.uint32)), (name, step)


@pytest.mark.parametrize("weight", [0.001, 0.25, 0.5, 0.9])
def test_ema_lerp_matches_torch(weight):
    """train.py:950-953 is torch._foreach_lerp_ (third-party, run here on the CPU): both of its weight branches."""
    import torch
    rng = np.random.default_rng(int(weight * 1000))
    e = rng.standard_normal(4099).astype(np.float32) * np.float32(0.02)
    p = rng.standard_normal(4099).astype(np.float32) * np.float32(0.02)
    ref = torch.from_numpy(e.copy())
    torch._foreach_lerp_([ref], [torch.from_numpy(p)], weight)
    O.ema_lerp(e, p, weight)
    assert np.array_equal(e.view(np.uint32), ref.numpy().view(np.uint32))


def test_clip_coefficient_is_torchs_expression():
    """torch's clip coefficient, max_norm / (total + 1e-6) with a Python float over a tensor (torch.nn.utils.clip_grad's
    _clip_grads_with_norm_), is Tensor.__rdiv__: reciprocal(total + 1e-6) * max_norm, two fp32 roundings. The
    oracle's clip_coef reproduces it bit for bit (the library's norm kernels do the same two operations); a single
    correctly rounded division would differ for max_norm != 1."""
    import torch
    rng = np.random.default_rng(3)
    totals = (10.0 ** rng.uniform(-4, 4, 20000)).astype(np.float32)
    t = torch.from_numpy(totals)
    differs = 0
    for max_norm in (1.0, 0.05, 0.3, 2.5, 7.0):
        ref = torch.clamp(max_norm / (t + 1e-6), max=1.0).numpy()
        got = np.array([O.clip_coef(x, max_norm) for x in totals], dtype=np.float32)
        assert np.array_equal(got, ref), max_norm
        one_div = np.minimum(np.float32(max_norm) / (totals + np.float32(1e-6)), np.float32(1.0)).astype(np.float32)
        differs += int((one_div != ref).sum())
    assert differs > 0
