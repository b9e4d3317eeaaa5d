"""Pin oracle/torch_port.py, the reference step that bench.py's reference arm times on the host CPU, against the
reference's own outputs (tests/golden/, made by running mote/train/muon.py and train.py:944-947). It performs the
reference's torch operations in the reference's order, so the outputs are equal bit for bit."""

import os

import numpy as np
import pytest
import torch

from oracle import torch_port as TP
from tests.conftest import golden
from tests.golden.cases import C0_DIVISOR, NS_CASES, ns_input, sample_index
from mote_b200 import configs


@pytest.fixture(autouse=True, scope="module")
def _fixture_threads():
    """The fixtures were made with min(8, cores) torch threads (make_golden.py); the CPU matmuls' blocking, and so
    their summation order, follows the thread count, so the port runs with the same count."""
    before = torch.get_num_threads()
    torch.set_num_threads(max(1, min(8, os.cpu_count() or 1)))
    yield
    torch.set_num_threads(before)


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("name,shape,seed", NS_CASES)
def test_newton_schulz_equals_the_reference(name, shape, seed):
    ref = golden("ns_reference")
    u = torch.from_numpy(ns_input(shape, seed))
    for steps in (1, 2, 5):
        assert np.array_equal(_bits16(TP.newton_schulz(u, steps)), ref[f"{name}_s{steps}"].reshape(shape))


@pytest.mark.parametrize("sw", [0, 1])
def test_batched_muon_equals_the_reference(sw):
    """reference tests/test_muon_batched.py:46-67: six matrices in three shape groups, three steps."""
    g = golden("muon_reference")
    ps = [torch.from_numpy(g[f"batched_p0_{i}"].copy()) for i in range(6)]
    grads = [torch.from_numpy(g[f"batched_g_{i}"].copy()) for i in range(6)]
    bufs = [None] * 6
    for it in range(3):
        for p, gr in zip(ps, grads):
            p.grad = gr * (1.0 + 0.1 * it)
        TP.muon_update(ps, bufs, lr=1e-2, momentum=0.95, nesterov=True, weight_decay=0.1, sw_decay=bool(sw),
                       lr_max=2e-2)
    for i in range(6):
        assert np.array_equal(ps[i].numpy(), g[f"batched_sw{sw}_p3_{i}"])
        assert np.array_equal(bufs[i].numpy(), g[f"batched_sw{sw}_buf_{i}"])


def test_expert_stack_equals_the_reference():
    """reference tests/test_moe.py:105-123: a 3-D [3, 24, 40] stack, three steps."""
    g = golden("muon_reference")
    p = torch.from_numpy(g["stack_p0"].copy())
    bufs = [None]
    for it in range(3):
        p.grad = torch.from_numpy(g["stack_g"].copy()) * (1 + 0.1 * it)
        TP.muon_update([p], bufs, lr=1e-2, weight_decay=0.1)
    assert np.array_equal(p.numpy(), g["stack_p3"])


def test_c0_ten_steps_equal_the_reference():
    """train.py:944-947 on the c0 workload for 10 steps: norms, sampled params and optimizer state."""
    g = golden("c0_reference")
    w = configs.c0()
    inp = configs.make_params(w, seed=0)
    ap = [torch.nn.Parameter(torch.from_numpy(p.copy())) for p in inp.adam_params]
    mp = [torch.nn.Parameter(torch.from_numpy(p.copy())) for p in inp.muon_params]
    nd = len(w.adam_decay_shapes)
    adam = torch.optim.AdamW([{"params": ap[:nd], "weight_decay": w.adam_wd}, {"params": ap[nd:], "weight_decay": 0.0}],
                             lr=w.adam_lr, betas=w.betas, eps=w.eps, fused=False)
    bufs = [None] * len(mp)
    kw = dict(lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True, weight_decay=w.muon_wd, ns_steps=w.ns_steps)
    for step in range(10):
        ag, mg = configs.make_grads(w, seed=0, step=step)
        for p, x in zip(ap + mp, ag + mg):
            p.grad = torch.from_numpy(x.copy())
        n = TP.optimizer_step(adam, mp, bufs, ap + mp, divisor=torch.tensor(C0_DIVISOR), max_norm=w.clip, muon_kw=kw)
        assert np.float32(n.item()) == g[f"norm{step}"], step
        if step in (0, 9):
            for kind, ps in (("a", ap), ("m", mp)):
                for i, p in enumerate(ps):
                    x = p.detach().numpy().ravel()
                    idx = sample_index(x.size)
                    assert np.array_equal(x[idx], g[f"{kind}p{step + 1}_{i}"]), (kind, step, i)
                    if kind == "m":
                        assert np.array_equal(bufs[i].numpy().ravel()[idx], g[f"mbuf{step + 1}_{i}"])
                    else:
                        st = adam.state[p]
                        assert np.array_equal(st["exp_avg"].numpy().ravel()[idx], g[f"am{step + 1}_{i}"])


def test_stack_plan_follows_the_cap():
    """muon.py:81-90 at c1: 768^2 fp32 stacks of 14 matrices, 768 x 3072 of 3, 512 x 2048 of 8."""
    plan = TP.stacks([tuple(s) for s in configs.c1().muon_shapes])
    sizes = {}
    for shape, idx in plan:
        sizes.setdefault(shape, []).append(len(idx))
    assert sizes[(768, 768)] == [14, 14, 14, 6]
    assert sizes[(768, 3072)] == [3, 3, 3, 3] and sizes[(3072, 768)] == [3, 3, 3, 3]
    assert sizes[(512, 2048)] == [8]
