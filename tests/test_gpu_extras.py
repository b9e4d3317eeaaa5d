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
