"""The sharded (multi-GPU) step's host logic on CPU ranks: 2 gloo processes run mote_b200.distributed.ShardedStep
with the oracle as the compute, and must end bitwise equal to one process running the oracle step on the summed
grads; both ranks must hold identical params. Also: the shard plan's ownership and layout rules."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mote_b200 import configs
from mote_b200.distributed import Compute, ShardedStep, make_plan, muon_cost
from oracle import moteopt_oracle as O

DIV = 3.0
CLIP = 0.02
STEPS = 3
EMA_DECAY = 0.75   # weight 0.25: the lerp's small-weight branch; the GPU tests cover the other


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _coef(norm: np.float32, max_norm):
    if max_norm is None:
        return norm, np.float32(1.0)
    return norm, O.clip_coef(norm, max_norm)


def oracle_compute(w):
    """The step's compute as the oracle (numpy on CPU tensors' memory)."""
    def sumsq(views, tensors, n_tensors, divisor):   # per grad tensor: its sum of squares over the views here
        s = np.zeros(n_tensors, dtype=np.float64)
        for v, t in zip(views, tensors):
            g = v.numpy().astype(np.float32)
            if divisor:
                g = (g / np.float32(divisor)).astype(np.float32)
            s[t] = float((g.astype(np.float64) ** 2).sum())
        return torch.from_numpy(s)

    def coef(sums, n_tensors, max_norm):   # per tensor the ranks' sums in rank order, then the norm of the norms
        per_rank = sums.numpy().reshape(-1, n_tensors)
        tot = np.zeros(n_tensors, dtype=np.float64)
        for row in per_rank:
            tot = tot + row
        norms = np.sqrt(tot).astype(np.float32)
        norm, c = _coef(np.float32(np.sqrt(np.sum(np.square(norms.astype(np.float64))))), max_norm)
        return torch.tensor([norm, c], dtype=torch.float32)

    def update(muon, adam, coef_t, divisor, muon_out):
        c = np.float32(coef_t.item()) if coef_t is not None else None

        def eff(g):
            x = g.numpy().astype(np.float32).copy()
            if divisor:
                x = (x / np.float32(divisor)).astype(np.float32)
            if c is not None:
                x = (x * c).astype(np.float32)
            return x
        for it in adam:
            O.adamw_update(it.param.numpy(), eff(it.grad), it.exp_avg.numpy(), it.exp_avg_sq.numpy(), it.lr,
                           w.betas[0], w.betas[1], w.eps, it.weight_decay, it.step)
        for it, out in zip(muon, muon_out):   # momentum + Newton-Schulz; the update O goes to `out`
            u = O.muon_momentum(it.momentum_buffer.numpy(), eff(it.grad), it.momentum, it.nesterov)
            m, n = it.param.shape[-2], it.param.shape[-1]
            o = O.newton_schulz(u.reshape(-1, m, n), steps=w.ns_steps).reshape(it.param.shape)
            out.copy_(torch.from_numpy(np.ascontiguousarray(o, dtype=np.float32)).to(torch.bfloat16))

    def apply(muon, updates, ema=None, ema_weight=0.0, norms=None):   # the item carries decay = lr * wd (muon.py:78)
        for k, (it, o) in enumerate(zip(muon, updates)):
            m, n = it.param.shape[-2], it.param.shape[-1]
            decay = it.lr * (it.decay / it.lr) if it.decay else 0.0   # as muon_lr_decay forms lr * wd
            O.muon_apply(it.param.numpy(), o.float().numpy(), 0.2 * max(m, n) ** 0.5, it.lr, decay)
            if ema is not None:
                O.ema_lerp(ema[k].numpy(), it.param.numpy(), ema_weight)
            if norms is not None:
                norms[k] = float(O.frob_norm32(it.param.numpy()))

    def ema(emas, params, weight):
        for e, p in zip(emas, params):
            O.ema_lerp(e.numpy(), p.numpy(), weight)
    return Compute(sumsq, coef, update, apply, None, ema)


def small_workload():
    return configs.Workload("dist_test", [(48, 64), (64, 48), (2, 32, 40), (40, 40), (16, 80)],
                            [(30, 16)], [(16,), (7,)], muon_wd=0.1, adam_wd=0.1, ns_steps=3)


def _grads(w, rank, step, world):
    """A rank's local grads. With more than two ranks the reduction's summation order is the collective's own, so
    the grads are put on a 2^-20 grid: every partial sum is then exact in fp32 and any order gives the same bits."""
    ag, mg = configs.make_grads(w, seed=100 + rank, step=step)
    if world > 2:
        ag = [(np.round(g * 2.0 ** 20) / 2.0 ** 20).astype(np.float32) for g in ag]
        mg = [(np.round(g * 2.0 ** 20) / 2.0 ** 20).astype(np.float32) for g in mg]
    return ag, mg


def _rank_main(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = small_workload()
        plan = make_plan(w.muon_shapes, w.adam_shapes, world, ns_steps=w.ns_steps)
        inp = configs.make_params(w, seed=0)
        pm = torch.zeros(plan.muon_len)
        pa = torch.zeros(plan.adam_len)
        gm = torch.zeros(plan.muon_len)
        ga = torch.zeros(plan.adam_len)
        nd = len(w.adam_decay_shapes)
        st = ShardedStep(plan, rank, pm, pa, gm, ga, oracle_compute(w), muon_lr=w.muon_lr, muon_wd=w.muon_wd,
                         adam_lr=w.adam_lr, adam_wd=[w.adam_wd if i < nd else 0.0 for i in range(len(w.adam_shapes))])
        for i, p in enumerate(inp.muon_params):
            st.muon_view(pm, i).copy_(torch.from_numpy(p))
        for i, p in enumerate(inp.adam_params):
            st.adam_view(pa, i).copy_(torch.from_numpy(p))
        st.enable_ema(EMA_DECAY)
        norms = []
        wnorms = torch.zeros(len(w.muon_shapes))
        for step in range(STEPS):
            ag, mg = _grads(w, rank, step, world)   # local grads differ per rank
            for i, g in enumerate(mg):
                st.muon_view(gm, i).copy_(torch.from_numpy(g))
            for i, g in enumerate(ag):
                st.adam_view(ga, i).copy_(torch.from_numpy(g))
            norms.append(float(st.step(max_norm=CLIP, grad_divisor=DIV, norms=wnorms)))
        ema = {f"em{i}": st.muon_view(st.em, i).numpy().copy() for i in range(len(w.muon_shapes))}
        ema.update({f"ea{i}": st.adam_view(st.ea, i).numpy().copy() for i in range(len(w.adam_shapes))})
        # the sharded checkpoint: the whole state on every rank, then a fresh step object resumed from it must
        # continue bit for bit like the original
        pm_after, pa_after = pm.clone(), pa.clone()
        sd = st.state_dict()
        adam_sd, muon_sd = sd["multi"]
        idx = {i: k for g in adam_sd["param_groups"] for k, i in zip(g["params"], g["plan_index"])}
        ckpt = {f"m{i}": adam_sd["state"][idx[i]]["exp_avg"].numpy().copy() for i in range(len(w.adam_shapes))}
        ckpt.update({f"v{i}": adam_sd["state"][idx[i]]["exp_avg_sq"].numpy().copy() for i in range(len(w.adam_shapes))})
        ckpt.update({f"b{i}": muon_sd["state"][i]["momentum_buffer"].numpy().copy() for i in range(len(w.muon_shapes))})
        st2 = ShardedStep(plan, rank, pm.clone(), pa.clone(), gm, ga, oracle_compute(w), muon_lr=w.muon_lr,
                          muon_wd=w.muon_wd, adam_lr=w.adam_lr,
                          adam_wd=[w.adam_wd if i < nd else 0.0 for i in range(len(w.adam_shapes))])
        st2.load_state_dict(sd)
        ag, mg = _grads(w, rank, STEPS, world)
        for i, g in enumerate(mg):
            st.muon_view(gm, i).copy_(torch.from_numpy(g))
        for i, g in enumerate(ag):
            st.adam_view(ga, i).copy_(torch.from_numpy(g))
        st.step(max_norm=CLIP, grad_divisor=DIV)
        st2.step(max_norm=CLIP, grad_divisor=DIV)
        resumed = bool(torch.equal(st.pm, st2.pm) and torch.equal(st.pa, st2.pa))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), pm=pm_after.numpy(), pa=pa_after.numpy(), norms=np.array(norms),
                 muon_off=np.array(plan.muon_off), adam_off=np.array(plan.adam_off), resumed=resumed,
                 wnorms=wnorms.numpy().copy(), **ckpt, **ema)
    finally:
        dist.destroy_process_group()


def _reference(world):
    """One process: grads summed over the ranks, then the oracle step with the same norm arithmetic."""
    w = small_workload()
    inp = configs.make_params(w, seed=0)
    nd = len(w.adam_decay_shapes)
    ms, vs = [np.zeros_like(p) for p in inp.adam_params], [np.zeros_like(p) for p in inp.adam_params]
    bufs = [None] * len(inp.muon_params)
    emas = [np.zeros_like(p) for p in inp.adam_params + inp.muon_params]   # train.py:721 starts the average at 0
    norms = []
    for step in range(STEPS):
        tot_a = [np.zeros_like(p) for p in inp.adam_params]
        tot_m = [np.zeros_like(p) for p in inp.muon_params]
        for r in range(world):
            ag, mg = _grads(w, r, step, world)
            tot_a = [(x + y).astype(np.float32) for x, y in zip(tot_a, ag)]
            tot_m = [(x + y).astype(np.float32) for x, y in zip(tot_m, mg)]
        allg = [(g / np.float32(DIV)).astype(np.float32) for g in tot_a + tot_m]
        norm, c = _coef(O.grad_total_norm(allg), CLIP)   # torch's get_total_norm, AdamW grads first
        norms.append(float(norm))
        allg = [(g * c).astype(np.float32) for g in allg]
        for i in range(len(inp.adam_params)):
            O.adamw_update(inp.adam_params[i], allg[i], ms[i], vs[i], w.adam_lr, w.betas[0], w.betas[1], w.eps,
                           w.adam_wd if i < nd else 0.0, step + 1)
        O.muon_step(inp.muon_params, allg[len(inp.adam_params):], bufs,
                    O.MuonGroup(lr=w.muon_lr, momentum=w.muon_momentum, weight_decay=(w.muon_lr * w.muon_wd) / w.muon_lr,
                                ns_steps=w.ns_steps))
        for e, p in zip(emas, inp.adam_params + inp.muon_params):   # train.py:950-953 after the step
            O.ema_lerp(e, p, 1.0 - EMA_DECAY)
    return inp, norms, ms, vs, bufs, emas


def test_plan_owns_every_matrix_once_and_balances_cost():
    w = configs.c1()
    for world in (2, 4, 8):
        plan = make_plan(w.muon_shapes, w.adam_shapes, world)
        assert sorted(set(plan.owner)) == list(range(world))
        loads = [sum(muon_cost(w.muon_shapes[i]) for i in plan.owned_muon(r)) for r in range(world)]
        assert max(loads) <= 1.25 * (sum(loads) / world)
        # segments never overlap and every offset is aligned
        spans = sorted((plan.muon_off[i], plan.muon_off[i] + int(np.prod(s))) for i, s in enumerate(w.muon_shapes))
        assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
        assert all(o % 64 == 0 for o in plan.muon_off)
        got = sum(n for r in range(world) for _, _, n in plan.adam_pieces(r))
        assert got == plan.a_total


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 3, 6])
def test_cpu_ranks_match_one_process(tmp_path, world):
    """gloo ranks with the oracle as the compute: params, optimizer state, checkpoint/resume, the weights' EMA and
    the per-matrix norms all equal the single-process oracle step on the summed grads, bit for bit. Three ranks
    split the five matrices unevenly; six ranks are more than there are matrices, so one rank owns none."""
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    outs = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(outs[0]["pm"], outs[r]["pm"]) and np.array_equal(outs[0]["pa"], outs[r]["pa"])
        assert np.array_equal(outs[0]["norms"], outs[r]["norms"])
    inp, norms, ms, vs, bufs, emas = _reference(world)
    assert np.allclose(outs[0]["norms"], norms, rtol=1e-6, atol=0)
    w = small_workload()
    for i, (p, s) in enumerate(zip(inp.muon_params, w.muon_shapes)):
        o = int(outs[0]["muon_off"][i])
        got = outs[0]["pm"][o:o + p.size].reshape(s)
        assert np.array_equal(got, p), (i, float(np.abs(got - p).max()))
    for i, (p, s) in enumerate(zip(inp.adam_params, w.adam_shapes)):
        o = int(outs[0]["adam_off"][i])
        assert np.array_equal(outs[0]["pa"][o:o + p.size].reshape(s), p), i
    # the EMA (train.py:950-953) and the ELR norms (elr.py:85-87) kept by the sharded step, on every rank
    na = len(w.adam_shapes)
    for r in range(world):
        for i in range(na):
            assert np.array_equal(outs[r][f"ea{i}"], emas[i]), (r, i)
        for i, p in enumerate(inp.muon_params):
            assert np.array_equal(outs[r][f"em{i}"], emas[na + i]), (r, i)
            assert outs[r]["wnorms"][i] == O.frob_norm32(p), (r, i)
    # the sharded checkpoint holds the single-process optimizer state, and resuming from it is bitwise
    for r in range(world):
        assert bool(outs[r]["resumed"])
        for i in range(len(w.adam_shapes)):
            assert np.array_equal(outs[r][f"m{i}"], ms[i]) and np.array_equal(outs[r][f"v{i}"], vs[i]), i
        for i in range(len(w.muon_shapes)):
            assert np.array_equal(outs[r][f"b{i}"], bufs[i]), i


def _rank_fault(rank, world, port, out_dir, mode):
    """One step on both ranks, then rank 1 either dies before the second step ("dead") or enters it late ("late")."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))
    w = small_workload()
    plan = make_plan(w.muon_shapes, w.adam_shapes, world, ns_steps=w.ns_steps)
    inp = configs.make_params(w, seed=0)
    pm, pa = torch.zeros(plan.muon_len), torch.zeros(plan.adam_len)
    gm, ga = torch.zeros(plan.muon_len), torch.zeros(plan.adam_len)
    nd = len(w.adam_decay_shapes)
    st = ShardedStep(plan, rank, pm, pa, gm, ga, oracle_compute(w), muon_lr=w.muon_lr, muon_wd=w.muon_wd,
                     adam_lr=w.adam_lr, adam_wd=[w.adam_wd if i < nd else 0.0 for i in range(len(w.adam_shapes))])
    for i, p in enumerate(inp.muon_params):
        st.muon_view(pm, i).copy_(torch.from_numpy(p))
    for i, p in enumerate(inp.adam_params):
        st.adam_view(pa, i).copy_(torch.from_numpy(p))
    for step in range(2):
        ag, mg = configs.make_grads(w, seed=100 + rank, step=step)
        for i, g in enumerate(mg):
            st.muon_view(gm, i).copy_(torch.from_numpy(g))
        for i, g in enumerate(ag):
            st.adam_view(ga, i).copy_(torch.from_numpy(g))
        if step == 1 and rank == 1:
            if mode == "dead":
                os._exit(0)   # leaves between steps, with nothing in flight
            time.sleep(2.0)
        t0 = time.time()
        try:
            st.step(max_norm=CLIP, grad_divisor=DIV)
        except Exception as exc:  # noqa: BLE001  (the surviving rank records how its collective ended)
            with open(os.path.join(out_dir, f"fault{rank}.txt"), "w") as f:
                f.write(f"error {type(exc).__name__} {time.time() - t0:.1f}")
            os._exit(0)   # the group is broken: no destroy_process_group
    np.save(os.path.join(out_dir, f"late{rank}.npy"), pm.numpy())
    dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_a_dead_rank_ends_the_step_with_an_error_not_a_hang(tmp_path):
    """Failure detection on the host: a rank that leaves between steps makes the survivor's next
    collective fail within the process group's timeout (15 s here) instead of waiting forever."""
    mp.spawn(_rank_fault, args=(2, _free_port(), str(tmp_path), "dead"), nprocs=2, join=True)
    msg = (tmp_path / "fault0.txt").read_text().split()
    assert msg[0] == "error" and float(msg[2]) < 60.0, msg


@pytest.mark.timeout(180)
def test_a_late_rank_only_delays_the_step(tmp_path):
    """A rank that enters the step 2 s late: the collectives wait for it and both ranks end with the same params."""
    mp.spawn(_rank_fault, args=(2, _free_port(), str(tmp_path), "late"), nprocs=2, join=True)
    a, b = np.load(tmp_path / "late0.npy"), np.load(tmp_path / "late1.npy")
    assert np.array_equal(a, b)
