"""Generate the golden fixtures by running the REFERENCE optimizer itself (noahsabaj/mote, imported from a local
checkout) on seeded inputs. Run in a container that has the reference checkout:

    MOTE_REFERENCE=/path/to/mote python tests/golden/make_golden.py

It writes `tests/golden/*.npz` and `groups_reference.json`. The fixtures pin `oracle/moteopt_oracle.py`
(tests/test_oracle_golden.py) and `oracle/torch_port.py` (tests/test_oracle_torch_port.py, bit for bit), and are the
reference side of the GPU parity tests and of the optimizer-construction test (tests/test_host_optim.py). The
reference is never needed at test time.

What is run (reference file:line):
  * `mote.train.muon.newton_schulz` (muon.py:26-43) on assorted shapes at 1, 2 and 5 iterations;
  * `mote.train.muon.Muon` (muon.py:46-100): the batched-step case of tests/test_muon_batched.py:46-67, the 3-D stack
    of tests/test_moe.py:105-123 and the per-matrix-lr cases of tests/test_elr.py:145-182;
  * `torch.optim.AdamW` (constructed as at train.py:98) and `torch.nn.utils.clip_grad_norm_` (train.py:946);
  * the whole step of train.py:944-947 (grads /= n, clip, AdamW then Muon) on the c0 workload for 10 steps;
  * `mote.model.moe.MoESwiGLU.update_bias` (moe.py:147-159), the lossfree router's bias step of train.py:948-949;
  * `split_muon_params` (muon.py:103-126), `build_optimizer` (train.py:76-105) and `set_lr` (train.py:177-179) on a
    model with every kind of parameter the split distinguishes (groups_reference.json).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
REF = os.environ.get("MOTE_REFERENCE")
if not REF:
    raise SystemExit("set MOTE_REFERENCE to a checkout of noahsabaj/mote (the generator runs the reference itself)")
sys.path.insert(0, REF)

from mote.train.muon import Muon, newton_schulz  # noqa: E402  (the reference)

from mote_b200 import configs  # noqa: E402
from tests.golden.cases import (ADAM_SHAPES, C0_DIVISOR, GROUP_KINDS, GROUP_LR, GROUP_MULTS,  # noqa: E402
                                GROUP_SET_LR, GROUP_WD, MOE_CASES, MOE_GAMMA, MOE_STEPS, NS_CASES, NS_STEPS,
                                describe_optimizer, group_model, mixer_parts, moe_bias0, moe_loads, ns_input,
                                sample_index)

torch.set_num_threads(max(1, min(8, os.cpu_count() or 1)))


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


# ---------------------------------------------------------------------------------------------------------------
def make_ns():
    out = {}
    for name, shape, seed in NS_CASES:
        u = torch.from_numpy(ns_input(shape, seed))
        for steps in NS_STEPS:
            out[f"{name}_s{steps}"] = bf16_bits(newton_schulz(u, steps=steps))
    np.savez_compressed(HERE / "ns_reference.npz", **out)


# ---------------------------------------------------------------------------------------------------------------
def make_muon():
    out = {}
    # tests/test_muon_batched.py:46-67 with its shapes and hyperparameters
    torch.manual_seed(0)
    shapes = [(64, 48), (64, 48), (64, 48), (32, 96), (40, 40), (32, 96)]
    params = [torch.randn(*s) * 0.1 for s in shapes]
    grads = [torch.randn(*s) * 0.01 for s in shapes]
    for i, (p, g) in enumerate(zip(params, grads)):
        out[f"batched_p0_{i}"] = p.numpy().copy()
        out[f"batched_g_{i}"] = g.numpy().copy()
    for sw in (False, True):
        ps = [torch.nn.Parameter(p.clone()) for p in params]
        opt = Muon(ps, lr=1e-2, momentum=0.95, nesterov=True, weight_decay=0.1, sw_decay=sw, lr_max=2e-2)
        for it in range(3):
            for p, g in zip(ps, grads):
                p.grad = g * (1.0 + 0.1 * it)
            opt.step()
        for i, p in enumerate(ps):
            out[f"batched_sw{int(sw)}_p3_{i}"] = p.detach().numpy().copy()
            out[f"batched_sw{int(sw)}_buf_{i}"] = opt.state[p]["momentum_buffer"].numpy().copy()
    # tests/test_moe.py:105-123: a 3-D stack
    torch.manual_seed(0)
    stack = torch.randn(3, 24, 40) * 0.1
    g = torch.randn(3, 24, 40) * 0.01
    out["stack_p0"], out["stack_g"] = stack.numpy().copy(), g.numpy().copy()
    ps = torch.nn.Parameter(stack.clone())
    opt = Muon([ps], lr=1e-2, weight_decay=0.1)
    for it in range(3):
        ps.grad = g * (1 + 0.1 * it)
        opt.step()
    out["stack_p3"] = ps.detach().numpy().copy()
    # tests/test_elr.py:174-182: decay follows the per-matrix rate
    p = torch.nn.Parameter(torch.eye(8) * 3.0)
    p.grad = torch.zeros_like(p)
    o = Muon([p], lr=1e-2, weight_decay=0.1)
    o.param_groups[0]["param_lr"] = {id(p): 5e-2}
    o.step()
    out["elr_decay_p1"] = p.detach().numpy().copy()
    np.savez_compressed(HERE / "muon_reference.npz", **out)


# ---------------------------------------------------------------------------------------------------------------
def make_adamw_clip():
    out = {}
    rng = np.random.default_rng(11)
    ps = [torch.nn.Parameter(torch.from_numpy(rng.standard_normal(size=s, dtype=np.float32) * np.float32(0.02)))
          for s in ADAM_SHAPES]
    for i, p in enumerate(ps):
        out[f"p0_{i}"] = p.detach().numpy().copy()
    decay = [ps[0], ps[2], ps[4]]
    nodecay = [ps[1], ps[3]]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1}, {"params": nodecay, "weight_decay": 0.0}],
                            lr=3e-4, betas=(0.9, 0.95), eps=1e-8, fused=False)
    for step in range(5):
        for i, p in enumerate(ps):
            g = configs._bf16_round(rng.standard_normal(size=p.shape, dtype=np.float32) * np.float32(1e-3))
            out[f"g{step}_{i}"] = g
            p.grad = torch.from_numpy(g.copy())
        n = torch.nn.utils.clip_grad_norm_(ps, 0.05)   # small max_norm so the clip is active
        out[f"norm{step}"] = np.float32(n.item())
        opt.step()
        if step in (0, 4):
            for i, p in enumerate(ps):
                st = opt.state[p]
                out[f"p{step + 1}_{i}"] = p.detach().numpy().copy()
                out[f"m{step + 1}_{i}"] = st["exp_avg"].numpy().copy()
                out[f"v{step + 1}_{i}"] = st["exp_avg_sq"].numpy().copy()
    np.savez_compressed(HERE / "adamw_reference.npz", **out)


# ---------------------------------------------------------------------------------------------------------------
def make_c0():
    """train.py:944-947 on the c0 workload: grads / n, clip_grad_norm_(1.0), AdamW, then Muon; 10 steps."""
    w = configs.c0()
    inp = configs.make_params(w, seed=0)
    ap = [torch.nn.Parameter(torch.from_numpy(p.copy())) for p in inp.adam_params]
    mp = [torch.nn.Parameter(torch.from_numpy(p.copy())) for p in inp.muon_params]
    nd = len(w.adam_decay_shapes)
    adam = torch.optim.AdamW([{"params": ap[:nd], "weight_decay": w.adam_wd}, {"params": ap[nd:], "weight_decay": 0.0}],
                             lr=w.adam_lr, betas=w.betas, eps=w.eps, fused=False)
    muon = Muon(mp, lr=w.muon_lr, momentum=w.muon_momentum, nesterov=True, weight_decay=w.muon_wd, ns_steps=w.ns_steps)
    out = {}
    divisor = C0_DIVISOR
    for step in range(10):
        ag, mg = configs.make_grads(w, seed=0, step=step)
        for p, g in zip(ap, ag):
            p.grad = torch.from_numpy(g.copy())
        for p, g in zip(mp, mg):
            p.grad = torch.from_numpy(g.copy())
        grads = [p.grad for p in ap + mp]
        torch._foreach_div_(grads, torch.tensor(divisor))
        n = torch.nn.utils.clip_grad_norm_(ap + mp, w.clip)
        out[f"norm{step}"] = np.float32(n.item())
        adam.step()
        muon.step()
        if step in (0, 9):
            for kind, ps in (("a", ap), ("m", mp)):
                for i, p in enumerate(ps):
                    x = p.detach().numpy().ravel()
                    idx = sample_index(x.size)
                    out[f"{kind}p{step + 1}_{i}"] = x[idx].copy()
                    out[f"{kind}p{step + 1}_{i}_sum"] = np.float64(x.astype(np.float64).sum())
                    out[f"{kind}p{step + 1}_{i}_ssq"] = np.float64((x.astype(np.float64) ** 2).sum())
                    if kind == "m":
                        b = muon.state[p]["momentum_buffer"].numpy().ravel()
                        out[f"mbuf{step + 1}_{i}"] = b[idx].copy()
                    else:
                        st = adam.state[p]
                        out[f"am{step + 1}_{i}"] = st["exp_avg"].numpy().ravel()[idx].copy()
                        out[f"av{step + 1}_{i}"] = st["exp_avg_sq"].numpy().ravel()[idx].copy()
    np.savez_compressed(HERE / "c0_reference.npz", **out)


# ---------------------------------------------------------------------------------------------------------------
def make_moe():
    """mote/model/moe.py:147-159 (MoESwiGLU.update_bias) on the MOE_CASES loads, MOE_STEPS steps per case."""
    from mote.model.moe import MoESwiGLU   # the reference
    out = {}
    for name, experts, kind, seed in MOE_CASES:
        torch.manual_seed(0)
        m = MoESwiGLU(16, 32, experts, top_k=1, router="lossfree", bias_gamma=MOE_GAMMA)
        with torch.no_grad():
            m.expert_bias.copy_(torch.from_numpy(moe_bias0(experts, seed)))
        for step in range(MOE_STEPS):
            with torch.no_grad():
                m._load_acc.copy_(torch.from_numpy(moe_loads(experts, kind, seed, step)))
            m.update_bias()
            out[f"{name}_bias{step}"] = m.expert_bias.numpy().copy()
            out[f"{name}_load{step}"] = m._load_acc.numpy().copy()
    np.savez_compressed(HERE / "moe_reference.npz", **out)


# ---------------------------------------------------------------------------------------------------------------
def make_groups():
    """The reference's split_muon_params (muon.py:103-126), build_optimizer (train.py:76-105) and set_lr
    (train.py:177-179) on cases.group_model for each optimizer kind: which parameter lands in which group, every
    group key, and the param_groups a checkpoint stores. Written as JSON (tests/golden/groups_reference.json)."""
    import json
    from mote.model.mamba3 import Mamba3Mixer as RefMixer   # the reference
    from mote.train.muon import split_muon_params
    from mote.train.train import build_optimizer, set_lr

    class Mamba3Mixer(RefMixer):   # an instance of the reference's class, without its full construction
        def __init__(self):
            torch.nn.Module.__init__(self)
            mixer_parts(self)

    model = group_model(Mamba3Mixer)
    names = {id(p): n for n, p in model.named_parameters()}
    muon, other = split_muon_params(model)
    out = {"split": {"muon": [names[id(p)] for p in muon], "other": [names[id(p)] for p in other]},
           "cuda": torch.cuda.is_available()}
    for kind in GROUP_KINDS:
        opt = build_optimizer(model, GROUP_LR, GROUP_WD, GROUP_MULTS, optimizer=kind)
        d = describe_optimizer(opt, model)
        set_lr(opt, GROUP_SET_LR)
        d["set_lr"] = [g["lr"] for g in opt.param_groups]
        out[kind] = d
    (HERE / "groups_reference.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    make_groups()
    make_ns()
    make_muon()
    make_adamw_clip()
    make_c0()
    make_moe()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
