"""The sharded step on 2 GPUs (NCCL): both ranks end with identical params, and they match the single-GPU fused step
run on the summed grads (AdamW to 1e-5; Muon to the Newton-Schulz noise floor, 1e-2 relative Frobenius, since the
sharded clip sums squares in another order and a one-ulp coefficient change is amplified by the bf16 iteration).
The step also keeps the weights' EMA and the per-matrix norms, checked against torch's lerp and fp64 norms.
Skipped with fewer than 2 GPUs."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
EMA_DECAY = 0.3   # weight 0.7: the lerp's large-weight branch


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _workload():
    from mote_b200 import configs
    return configs.Workload("dist_gpu_test", [(256, 256)] * 3 + [(256, 1024), (1024, 256), (2, 128, 384)],
                            [(271, 64)], [(64,)] * 3)


def _rank(rank, world, port, out, peer):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from mote_b200 import configs
        from mote_b200.distributed import ShardedStep, cuda_compute, make_plan
        w = _workload()
        plan = make_plan(w.muon_shapes, w.adam_shapes, world)
        inp = configs.make_params(w, seed=0)
        pm = torch.zeros(plan.muon_len, device=dev)
        pa = torch.zeros(plan.adam_len, device=dev)
        gm = torch.zeros(plan.muon_len, device=dev, dtype=torch.bfloat16)
        ga = torch.zeros(plan.adam_len, device=dev, dtype=torch.bfloat16)
        nd = len(w.adam_decay_shapes)
        st = ShardedStep(plan, rank, pm, pa, gm, ga, cuda_compute(betas=w.betas), muon_lr=w.muon_lr, muon_wd=w.muon_wd,
                         adam_lr=w.adam_lr, adam_wd=[w.adam_wd if i < nd else 0.0 for i in range(len(w.adam_shapes))])
        if peer:
            st.enable_peer_updates()
        for i, p in enumerate(inp.muon_params):
            st.muon_view(pm, i).copy_(torch.from_numpy(p))
        for i, p in enumerate(inp.adam_params):
            st.adam_view(pa, i).copy_(torch.from_numpy(p))
        st.enable_ema(EMA_DECAY)
        snaps = {"pm_init": pm.cpu().numpy(), "pa_init": pa.cpu().numpy()}
        wnorms = torch.zeros(len(w.muon_shapes), device=dev)
        norms = []
        for step in range(3):
            ag, mg = configs.make_grads(w, seed=50 + rank, step=step)
            for i, g in enumerate(mg):
                st.muon_view(gm, i).copy_(torch.from_numpy(g))
            for i, g in enumerate(ag):
                st.adam_view(ga, i).copy_(torch.from_numpy(g))
            norms.append(st.step(max_norm=0.05, grad_divisor=2.0, norms=wnorms).item())
            snaps[f"pm{step}"], snaps[f"pa{step}"] = pm.cpu().numpy(), pa.cpu().numpy()
        torch.cuda.synchronize()
        st.close()
        np.savez(os.path.join(out, f"r{rank}_{int(peer)}.npz"), pm=pm.cpu().numpy(), pa=pa.cpu().numpy(),
                 norms=np.array(norms), moff=np.array(plan.muon_off), aoff=np.array(plan.adam_off),
                 em=st.em.cpu().numpy(), ea=st.ea.cpu().numpy(), wnorms=wnorms.cpu().numpy(), **snaps)
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_step_matches_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from mote_b200 import configs
    from mote_b200.functional import AdamWItem, MuonItem, optimizer_step
    from oracle import moteopt_oracle as O
    world = 2
    for peer in (False, True):   # NCCL all-gather of the updates, then the peer (NVLink) reads of them
        mp.spawn(_rank, args=(world, _port(), str(tmp_path), peer), nprocs=world, join=True)
    r0, r1 = (np.load(tmp_path / f"r{r}_0.npz") for r in range(world))
    assert np.array_equal(r0["pm"], r1["pm"]) and np.array_equal(r0["pa"], r1["pa"])
    for r in range(world):   # the two exchanges give the same bits
        q = np.load(tmp_path / f"r{r}_1.npz")
        assert np.array_equal(q["pm"], r0["pm"]) and np.array_equal(q["pa"], r0["pa"])
    # the weights' EMA (train.py:950-953) and the ELR norms (elr.py:85-87) kept by the sharded step: the same on every
    # rank and exchange, the EMA bit for bit torch's lerp of each step's params, the norms those of the final params
    w = _workload()
    for r in range(world):
        for peer in (0, 1):
            q = np.load(tmp_path / f"r{r}_{peer}.npz")
            for key in ("em", "ea", "wnorms"):
                assert np.array_equal(q[key], r0[key]), (r, peer, key)
    em = torch.zeros(r0["pm_init"].shape)   # train.py:721 starts the average at 0
    ea = torch.zeros(r0["pa_init"].shape)
    for step in range(3):
        torch._foreach_lerp_([em, ea], [torch.from_numpy(r0[f"pm{step}"]), torch.from_numpy(r0[f"pa{step}"])],
                             1.0 - EMA_DECAY)
    for i, s in enumerate(w.muon_shapes):
        o, n = int(r0["moff"][i]), int(np.prod(s))
        assert np.array_equal(r0["em"][o:o + n], em.numpy()[o:o + n]), i
        exact = float(np.linalg.norm(r0["pm"][o:o + n].astype(np.float64)))
        assert abs(float(r0["wnorms"][i]) - exact) <= 1e-6 * exact, i
    for i, s in enumerate(w.adam_shapes):
        o, n = int(r0["aoff"][i]), int(np.prod(s))
        assert np.array_equal(r0["ea"][o:o + n], ea.numpy()[o:o + n]), i
    # one GPU, grads summed over the ranks (bf16 sum, as NCCL's bf16 reduction of two values)
    dev = torch.device("cuda", 0)
    inp = configs.make_params(w, seed=0)
    mp_ = [torch.from_numpy(p).to(dev) for p in inp.muon_params]
    ap = [torch.from_numpy(p).to(dev) for p in inp.adam_params]
    mb = [torch.zeros_like(p) for p in mp_]
    am, av = [torch.zeros_like(p) for p in ap], [torch.zeros_like(p) for p in ap]
    nd = len(w.adam_decay_shapes)
    for step in range(3):
        gs = [configs.make_grads(w, seed=50 + r, step=step) for r in range(world)]
        ag = [(torch.from_numpy(gs[0][0][i]).to(dev).bfloat16() + torch.from_numpy(gs[1][0][i]).to(dev).bfloat16())
              for i in range(len(ap))]
        mg = [(torch.from_numpy(gs[0][1][i]).to(dev).bfloat16() + torch.from_numpy(gs[1][1][i]).to(dev).bfloat16())
              for i in range(len(mp_))]
        n = optimizer_step([MuonItem(p, g, b, w.muon_lr, w.muon_lr * w.muon_wd) for p, g, b in zip(mp_, mg, mb)],
                           [AdamWItem(p, g, m, v, w.adam_lr, w.adam_wd if i < nd else 0.0, step + 1)
                            for i, (p, g, m, v) in enumerate(zip(ap, ag, am, av))],
                           betas=w.betas, max_norm=0.05, grad_divisor=2.0)
        assert abs(n.item() - r0["norms"][step]) <= 1e-5 * n.item()
    for i, (p, s) in enumerate(zip(mp_, w.muon_shapes)):
        o = int(r0["moff"][i])
        got = r0["pm"][o:o + p.numel()].reshape(s)
        assert O.rel_frob(got, p.cpu().numpy()) < 1e-2, i
    for i, (p, s) in enumerate(zip(ap, w.adam_shapes)):
        o = int(r0["aoff"][i])
        got = r0["pa"][o:o + p.numel()].reshape(s)
        ref = p.cpu().numpy()
        assert np.allclose(got, ref, rtol=1e-5, atol=1e-8), i
