"""The sharded step on 2, 4 and 8 GPUs (NCCL, and the peer-memory grad reduction and update exchange): every rank ends
with identical params, equal bit for bit to the single-GPU fused step on the summed grads with the clip active (the
sharded clip forms the same per-tensor norms and the same norm of norms). The step also keeps the weights' EMA and
the per-matrix norms, checked against torch's lerp and fp64 norms. Skipped where the box has fewer GPUs."""

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
CLIP = 0.05


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
        assert n.item() == r0["norms"][step], (step, n.item(), r0["norms"][step])
    for i, (p, s) in enumerate(zip(mp_, w.muon_shapes)):
        o = int(r0["moff"][i])
        got = r0["pm"][o:o + p.numel()].reshape(s)
        assert np.array_equal(got, p.cpu().numpy()), (i, O.rel_frob(got, p.cpu().numpy()))
    for i, (p, s) in enumerate(zip(ap, w.adam_shapes)):
        o = int(r0["aoff"][i])
        assert np.array_equal(r0["pa"][o:o + p.numel()].reshape(s), p.cpu().numpy()), i


# ---------------------------------------------------------------------------------------------------------------
# N = 2, 4, 8 GPUs: the sharded step bit for bit against one GPU, and the sharded checkpoint round trip over NCCL
def _grid_workload():
    from mote_b200 import configs
    return configs.Workload("dist_grid_test", [(256, 256)] * 5 + [(256, 1024), (1024, 256), (2, 128, 384), (384, 640)],
                            [(271, 64)], [(64,)] * 5)


def _grid_grads(w, rank, step):
    """fp32 grads on the 2^-20 grid with |g| < 2^-10: a sum over up to 8 ranks is exact in fp32 in any order, so
    NCCL's reduction order cannot change a bit and one GPU can reproduce the reduced grads exactly."""
    rng = np.random.default_rng([77, rank, step])
    out = []
    for s in list(w.adam_shapes) + list(w.muon_shapes):
        out.append((rng.integers(-1023, 1024, size=s).astype(np.float32) * np.float32(2.0 ** -20)))
    return out[: len(w.adam_shapes)], out[len(w.adam_shapes):]


def _grid_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from mote_b200 import configs
        from mote_b200.distributed import ShardedStep, cuda_compute, make_plan
        w = _grid_workload()
        plan = make_plan(w.muon_shapes, w.adam_shapes, world)
        inp = configs.make_params(w, seed=5)
        nd = len(w.adam_decay_shapes)
        wds = [w.adam_wd if i < nd else 0.0 for i in range(len(w.adam_shapes))]

        def new_step(pm, pa):
            gm = torch.zeros(plan.muon_len, device=dev)
            ga = torch.zeros(plan.adam_len, device=dev)
            return ShardedStep(plan, rank, pm, pa, gm, ga, cuda_compute(betas=w.betas), muon_lr=w.muon_lr,
                               muon_wd=w.muon_wd, adam_lr=w.adam_lr, adam_wd=wds)

        def load_grads(st, step):
            ag, mg = _grid_grads(w, rank, step)
            for i, g in enumerate(mg):
                st.muon_view(st.gm, i).copy_(torch.from_numpy(g))
            for i, g in enumerate(ag):
                st.adam_view(st.ga, i).copy_(torch.from_numpy(g))

        pm = torch.zeros(plan.muon_len, device=dev)
        pa = torch.zeros(plan.adam_len, device=dev)
        st = new_step(pm, pa)
        for i, p in enumerate(inp.muon_params):
            st.muon_view(pm, i).copy_(torch.from_numpy(p))
        for i, p in enumerate(inp.adam_params):
            st.adam_view(pa, i).copy_(torch.from_numpy(p))
        st.enable_peer_updates(peer_grads=True)   # grads reduced and updates read over NVLink at every world size
        for step in range(2):
            load_grads(st, step)
            st.step(max_norm=CLIP)
        sd = st.state_dict()       # collective: the ZeRO-1 slices and the owners' momentum buffers, gathered
        # resume: a fresh step object on copies of the params takes the checkpoint (NCCL all-gather exchange)
        st2 = new_step(pm.clone(), pa.clone())
        st2.load_state_dict(sd)
        for s in (st, st2):   # st2: NCCL reduce-scatter and all-gather exchange
            load_grads(s, 2)
            s.step(max_norm=CLIP)
        torch.cuda.synchronize()
        sd3 = st.state_dict()
        sd3b = st2.state_dict()
        st.close()
        flat = {"pm": pm.cpu().numpy(), "pa": pa.cpu().numpy(), "pm2": st2.pm.cpu().numpy(), "pa2": st2.pa.cpu().numpy(),
                "moff": np.array(plan.muon_off), "aoff": np.array(plan.adam_off)}
        for tag, d in (("sd2", sd), ("sd3", sd3), ("sd3b", sd3b)):
            adam_sd, muon_sd = d["multi"]
            for g in adam_sd["param_groups"]:
                for k, i in zip(g["params"], g["plan_index"]):
                    flat[f"{tag}_m{i}"] = adam_sd["state"][k]["exp_avg"].cpu().numpy()
                    flat[f"{tag}_v{i}"] = adam_sd["state"][k]["exp_avg_sq"].cpu().numpy()
                    flat[f"{tag}_step{i}"] = np.array(float(adam_sd["state"][k]["step"]))
            for i in range(len(w.muon_shapes)):
                flat[f"{tag}_b{i}"] = muon_sd["state"][i]["momentum_buffer"].cpu().numpy()
        np.savez(os.path.join(out, f"grid_r{rank}.npz"), **flat)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_step_and_checkpoint_bitwise_against_one_gpu(tmp_path, world):
    """`world` ranks over NCCL (grads reduced and updates read over NVLink), 3 steps with the clip active on
    exact-grid fp32 grads: every rank holds the same params, and they equal one GPU's optimizer_step on the summed
    grads bit for bit; the sharded
    checkpoint after step 2 (ShardedStep.state_dict, train.py:68-73's {"multi": [adamw, muon]} layout) equals that
    GPU's optimizer state bit for bit, and a fresh ShardedStep that loads it continues bit for bit (step 3)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from mote_b200 import configs
    from mote_b200.functional import AdamWItem, MuonItem, optimizer_step
    mp.spawn(_grid_rank, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    rs = [np.load(tmp_path / f"grid_r{r}.npz") for r in range(world)]
    for r in rs[1:]:
        for key in rs[0].files:
            assert np.array_equal(r[key], rs[0][key]), key
    r0 = rs[0]
    assert np.array_equal(r0["pm2"], r0["pm"]) and np.array_equal(r0["pa2"], r0["pa"])   # the resumed step
    # one GPU on the summed grads
    w = _grid_workload()
    dev = torch.device("cuda", 0)
    inp = configs.make_params(w, seed=5)
    mps = [torch.from_numpy(p).to(dev) for p in inp.muon_params]
    aps = [torch.from_numpy(p).to(dev) for p in inp.adam_params]
    mb = [torch.zeros_like(p) for p in mps]
    am, av = [torch.zeros_like(p) for p in aps], [torch.zeros_like(p) for p in aps]
    nd = len(w.adam_decay_shapes)
    snap = {}
    for step in range(3):
        gs = [_grid_grads(w, r, step) for r in range(world)]
        ag = [torch.from_numpy(sum(g[0][i] for g in gs)).to(dev) for i in range(len(aps))]
        mg = [torch.from_numpy(sum(g[1][i] for g in gs)).to(dev) for i in range(len(mps))]
        optimizer_step([MuonItem(p, g, b, w.muon_lr, w.muon_lr * w.muon_wd) for p, g, b in zip(mps, mg, mb)],
                       [AdamWItem(p, g, m, v, w.adam_lr, w.adam_wd if i < nd else 0.0, step + 1)
                        for i, (p, g, m, v) in enumerate(zip(aps, ag, am, av))], betas=w.betas, max_norm=CLIP)
        if step == 1:
            snap = {"m": [x.cpu().numpy() for x in am], "v": [x.cpu().numpy() for x in av],
                    "b": [x.cpu().numpy() for x in mb]}
    for tag, ref in (("sd2", snap), ("sd3", {"m": [x.cpu().numpy() for x in am], "v": [x.cpu().numpy() for x in av],
                                             "b": [x.cpu().numpy() for x in mb]})):
        for i in range(len(aps)):
            assert np.array_equal(r0[f"{tag}_m{i}"], ref["m"][i]), (tag, "exp_avg", i)
            assert np.array_equal(r0[f"{tag}_v{i}"], ref["v"][i]), (tag, "exp_avg_sq", i)
            assert float(r0[f"{tag}_step{i}"]) == (2.0 if tag == "sd2" else 3.0)
        for i in range(len(mps)):
            assert np.array_equal(r0[f"{tag}_b{i}"], ref["b"][i]), (tag, "momentum_buffer", i)
            assert np.array_equal(r0[f"sd3b_b{i}"], r0[f"sd3_b{i}"])
    for i, (p, s) in enumerate(zip(mps, w.muon_shapes)):
        o = int(r0["moff"][i])
        assert np.array_equal(r0["pm"][o:o + p.numel()].reshape(s), p.cpu().numpy()), ("muon param", i)
    for i, (p, s) in enumerate(zip(aps, w.adam_shapes)):
        o = int(r0["aoff"][i])
        assert np.array_equal(r0["pa"][o:o + p.numel()].reshape(s), p.cpu().numpy()), ("adamw param", i)
