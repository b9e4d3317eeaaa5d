"""The step's fused extras on the GPU: the weights' EMA (mote/train/train.py:950-953, torch._foreach_lerp_ after the
step) and the Muon params' Frobenius norms (mote/train/elr.py:85-87, NormTracker.sample), both computed in the
passes that write the params. The EMA must equal torch's lerp of the same inputs bit for bit (torch on the CPU is
the oracle), the params must be unchanged by the extras, and the norms must match the fp64 norm of the updated
params to 1e-6 relative."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(96, 160), (160, 96), (37, 53), (2, 48, 64), (256, 2048), (2048, 256), (8, 16392)]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


def _setup(dev, seed):
    from mote_b200.functional import AdamWItem, MuonItem
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    ps = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in SHAPES]
    gs = [(torch.randn(s, generator=gen, device=dev) * 1e-3).to(torch.bfloat16) for s in SHAPES]
    bufs = [torch.zeros_like(p) for p in ps]
    pa = [torch.randn(300, generator=gen, device=dev) * 0.02, torch.randn(7, 33, generator=gen, device=dev) * 0.02]
    ga = [(torch.randn(p.shape, generator=gen, device=dev) * 1e-3).to(torch.bfloat16) for p in pa]
    m = [torch.zeros_like(p) for p in pa]
    v = [torch.zeros_like(p) for p in pa]
    muon = [MuonItem(p, g, b, 0.02, 0.002) for p, g, b in zip(ps, gs, bufs)]
    adam = [AdamWItem(p, g, mm, vv, 3e-4, 0.1, 1) for p, g, mm, vv in zip(pa, ga, m, v)]
    return muon, adam


@pytest.mark.parametrize("weight", [0.01, 0.7])
def test_fused_ema_equals_torch_lerp_and_leaves_params_unchanged(dev, weight):
    from mote_b200.functional import optimizer_step
    muon_a, adam_a = _setup(dev, 7)
    optimizer_step(muon_a, adam_a, ns_steps=2, betas=(0.9, 0.95), max_norm=1.0)
    muon_b, adam_b = _setup(dev, 7)
    items = adam_b + muon_b
    gen = torch.Generator(device=dev)
    gen.manual_seed(8)
    ema = [it.param.clone() + torch.randn(it.param.shape, generator=gen, device=dev) * 1e-3 for it in items]
    ema[1] = None   # a tensor without an EMA
    ema_old = [e.cpu() if e is not None else None for e in ema]
    optimizer_step(muon_b, adam_b, ns_steps=2, betas=(0.9, 0.95), max_norm=1.0, ema=ema, ema_weight=weight)
    torch.cuda.synchronize()
    for x, y in zip(adam_a + muon_a, items):   # the extras do not change the step
        assert torch.equal(x.param, y.param)
    for it, e, e0 in zip(items, ema, ema_old):
        if e is None:
            continue
        ref = [e0.clone()]
        torch._foreach_lerp_(ref, [it.param.cpu()], weight)
        assert torch.equal(e.cpu(), ref[0])


def test_fused_muon_norms_match_the_updated_params(dev):
    from mote_b200.functional import optimizer_step
    muon, adam = _setup(dev, 9)
    norms = torch.full((len(muon),), -1.0, device=dev)
    optimizer_step(muon, adam, ns_steps=2, betas=(0.9, 0.95), muon_norms=norms)
    torch.cuda.synchronize()
    for it, n in zip(muon, norms.cpu().tolist()):
        exact = float(np.linalg.norm(it.param.cpu().numpy().astype(np.float64)))
        assert abs(n - exact) <= 1e-6 * exact, (tuple(it.param.shape), n, exact)
        tn = float(torch.linalg.vector_norm(it.param.cpu()))   # what NormTracker computes (fp32)
        assert abs(n - tn) <= 1e-5 * tn


@pytest.mark.parametrize("weight", [0.01, 0.7])
def test_standalone_ema_lerp_equals_torch(dev, weight):
    """moteopt_ema_lerp (the EMA pass for params no fused pass writes): full 16K chunks, ragged tails and a tensor
    starting off the 16-byte grid, bit for bit torch._foreach_lerp_ on the CPU."""
    from mote_b200.functional import ema_lerp
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    sizes = [16384 * 3, 16384 * 2 + 77, 5, 1]
    ps = [torch.randn(n, generator=gen, device=dev) * 0.02 for n in sizes]
    es = [torch.randn(n, generator=gen, device=dev) * 0.02 for n in sizes]
    base = torch.randn(16384 + 1, generator=gen, device=dev)
    ps.append(base[1:])   # 4-byte aligned only: the element path
    es.append(torch.randn(16384, generator=gen, device=dev)[:16384])
    ref = [e.cpu() for e in es]
    torch._foreach_lerp_(ref, [p.cpu() for p in ps], weight)
    ema_lerp(es, ps, weight)
    torch.cuda.synchronize()
    for e, r in zip(es, ref):
        assert torch.equal(e.cpu(), r)


@pytest.mark.parametrize("weight", [0.01, 0.7])
def test_muon_apply_with_ema_and_norms(dev, weight):
    """moteopt_muon_apply_ex (the sharded step's apply): the same params as the plain apply, the EMA bit for bit
    torch's lerp of the updated params, and the norms within 1e-6 of the fp64 norms."""
    from mote_b200.distributed import cuda_compute
    from mote_b200.functional import MuonItem
    comp = cuda_compute()
    gen = torch.Generator(device=dev)
    gen.manual_seed(12)
    shapes = [(96, 160), (160, 96), (37, 53), (2, 48, 64), (256, 2048)]
    p0 = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in shapes]
    us = [(torch.randn(s, generator=gen, device=dev) * 0.05).to(torch.bfloat16) for s in shapes]
    e0 = [p + torch.randn(p.shape, generator=gen, device=dev) * 1e-3 for p in p0]
    pa = [p.clone() for p in p0]
    pb = [p.clone() for p in p0]
    eb = [e.clone() for e in e0]
    comp.apply([MuonItem(p, None, None, 0.02, 0.002) for p in pa], us)
    norms = torch.full((len(shapes),), -1.0, device=dev)
    comp.apply([MuonItem(p, None, None, 0.02, 0.002) for p in pb], us, ema=eb, ema_weight=weight, norms=norms)
    torch.cuda.synchronize()
    for a, b, e, e_old, n in zip(pa, pb, eb, e0, norms.cpu().tolist()):
        assert torch.equal(a, b)
        ref = [e_old.cpu()]
        torch._foreach_lerp_(ref, [b.cpu()], weight)
        assert torch.equal(e.cpu(), ref[0])
        exact = float(np.linalg.norm(b.cpu().numpy().astype(np.float64)))
        assert abs(n - exact) <= 1e-6 * exact


def test_captured_step_with_ema_norms_and_moe_equals_eager(dev):
    """CapturedStep carrying the trainer's after-step work (EMA, per-matrix norms, MoE bias step) in its graph:
    three replays give the same bits as three eager steps with the same extras."""
    import types

    from mote_b200.functional import CapturedStep, moe_update_bias, optimizer_step

    def mk(seed):
        muon, adam = _setup(dev, seed)
        ema = [it.param.clone() for it in adam + muon]
        norms = torch.zeros(len(muon), device=dev)
        gen = torch.Generator(device=dev)
        gen.manual_seed(3)
        layer = types.SimpleNamespace(router_kind="lossfree", bias_gamma=1e-3,
                                      _load_acc=torch.zeros(16, device=dev), expert_bias=torch.zeros(16, device=dev))
        loads = [torch.randint(0, 500, (16,), generator=gen, device=dev).float() for _ in range(3)]
        return muon, adam, ema, norms, layer, loads
    ma, aa, ea, na, la, lda = mk(21)
    mb, ab, eb, nb, lb, ldb = mk(21)
    for k in range(3):
        la._load_acc.copy_(lda[k])
        optimizer_step(ma, aa, ns_steps=2, betas=(0.9, 0.95), max_norm=1.0, ema=ea, ema_weight=0.3, muon_norms=na,
                       device_step=torch.full((), float(k), device=dev))
        moe_update_bias([la])
    cs = CapturedStep(mb, ab, ns_steps=2, betas=(0.9, 0.95), max_norm=1.0, ema=eb, ema_weight=0.3, muon_norms=nb,
                      moe=[lb])
    for k in range(3):
        lb._load_acc.copy_(ldb[k])
        cs()
    torch.cuda.synchronize()
    assert cs.graph is not None
    for x, y in zip(aa + ma, ab + mb):
        assert torch.equal(x.param, y.param)
    for x, y in zip(ea, eb):
        assert torch.equal(x, y)
    assert torch.equal(na, nb)
    assert torch.equal(la.expert_bias, lb.expert_bias) and float(lb._load_acc.abs().sum()) == 0.0


def test_standalone_ema_lerp_over_many_tensors(dev):
    """More tensors than one argument block holds (600 > 512): the lerp is split over launches, same bits as torch."""
    from mote_b200.functional import ema_lerp
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    ps = [torch.randn(int(n), generator=gen, device=dev) for n in torch.randint(1, 3000, (600,), generator=gen, device=dev).tolist()]
    es = [torch.randn(p.shape, generator=gen, device=dev) for p in ps]
    ref = [e.cpu() for e in es]
    torch._foreach_lerp_(ref, [p.cpu() for p in ps], 0.02)
    ema_lerp(es, ps, 0.02)
    torch.cuda.synchronize()
    assert all(torch.equal(e.cpu(), r) for e, r in zip(es, ref))
