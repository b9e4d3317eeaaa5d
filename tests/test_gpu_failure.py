"""Failure detection that faults no GPU: a non-finite grad norm is reported in the library's status word (the step
itself proceeds, as torch's clip_grad_norm_ + step do, mote/train/train.py:946-947), and the degenerate all-zero
step is exact. The bounded waits of the Newton-Schulz kernel report MOTEOPT_STATUS_WAIT_TIMEOUT instead of hanging;
no test provokes one (there is no fault injector), the parity tests check the word stays clear."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


def _setup(dev, seed):
    from mote_b200.functional import AdamWItem, MuonItem
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    mp = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in [(64, 96), (96, 64), (2, 32, 48)]]
    mg = [torch.randn(p.shape, generator=gen, device=dev) * 1e-3 for p in mp]
    ap = [torch.randn(100, generator=gen, device=dev) * 0.02]
    ag = [torch.randn(100, generator=gen, device=dev) * 1e-3]
    muon = [MuonItem(p, g, torch.zeros_like(p), 0.02, 0.02 * 0.1) for p, g in zip(mp, mg)]
    adam = [AdamWItem(p, g, torch.zeros_like(p), torch.zeros_like(p), 3e-4, 0.1, 1) for p, g in zip(ap, ag)]
    return muon, adam


def test_nan_grad_sets_the_nonfinite_status_and_the_step_proceeds_like_torch(dev):
    """A NaN grad: the total norm is NaN, torch's clip coefficient is NaN, every grad becomes NaN, so every param does.
    The library does the same and raises MOTEOPT_STATUS_NONFINITE (4) in its status word."""
    from mote_b200 import ops
    from mote_b200.functional import optimizer_step
    ops.read_status(dev, clear=True)
    muon, adam = _setup(dev, 1)
    adam[0].grad[17] = float("nan")
    norm = optimizer_step(muon, adam, ns_steps=2, betas=(0.9, 0.95), max_norm=1.0)
    st, (total, coef) = ops.read_status(dev, clear=True)
    assert st & 4 and not st & 3
    assert np.isnan(norm.item()) and np.isnan(total) and np.isnan(coef)
    for it in muon + adam:
        assert bool(torch.isnan(it.param).all())
    # a clean step afterwards leaves the word clear
    muon, adam = _setup(dev, 2)
    optimizer_step(muon, adam, ns_steps=2, betas=(0.9, 0.95), max_norm=1.0)
    st, _ = ops.read_status(dev, clear=True)
    assert st == 0


def test_inf_grad_zeroes_the_other_grads_like_torch(dev):
    """An Inf grad: the norm is Inf and the coefficient max_norm / (Inf + 1e-6) = 0, so every finite grad becomes 0
    and the Inf one NaN (Inf * 0), as torch's clip does: the Muon params only decay, the AdamW param is NaN at that
    element and decayed elsewhere."""
    from mote_b200 import ops
    from mote_b200.functional import optimizer_step
    ops.read_status(dev, clear=True)
    muon, adam = _setup(dev, 3)
    p_m0 = [it.param.clone() for it in muon]
    p_a0 = adam[0].param.clone()
    adam[0].grad[5] = float("inf")
    norm = optimizer_step(muon, adam, ns_steps=2, betas=(0.9, 0.95), max_norm=1.0)
    st, (total, coef) = ops.read_status(dev, clear=True)
    assert st & 4 and np.isinf(norm.item()) and coef == 0.0
    keep = np.float32(1.0 - 0.02 * 0.1)   # p * (1 - decay): the items carry decay = lr * wd (muon.py:78)
    for it, p0 in zip(muon, p_m0):
        assert torch.equal(it.param.cpu(), torch.from_numpy(p0.cpu().numpy() * keep))
    a = adam[0].param.cpu().numpy()
    assert np.isnan(a[5]) and np.isfinite(np.delete(a, 5)).all()
    # AdamW with a zero grad: m = v = 0, the update term is 0 / eps, only the decoupled decay moves the param
    exp = p_a0.cpu().numpy() * np.float32(1.0 - 3e-4 * 0.1)
    assert np.array_equal(np.delete(a, 5), np.delete(exp, 5))


def test_all_zero_grads_only_decay(dev):
    """All grads zero: norm 0, coefficient 1, momentum 0, X0 = 0 / (0 + eps) = 0, Newton-Schulz keeps 0, so every
    param is exactly p * (1 - decay) and the status stays clear."""
    from mote_b200 import ops
    from mote_b200.functional import optimizer_step
    ops.read_status(dev, clear=True)
    muon, adam = _setup(dev, 4)
    for it in muon + adam:
        it.grad.zero_()
    p0 = [it.param.clone() for it in muon + adam]
    norm = optimizer_step(muon, adam, ns_steps=5, betas=(0.9, 0.95), max_norm=1.0)
    st, _ = ops.read_status(dev, clear=True)
    assert st == 0 and norm.item() == 0.0
    for it, p in zip(muon, p0):
        assert torch.equal(it.param.cpu(), torch.from_numpy(p.cpu().numpy() * np.float32(1.0 - 0.02 * 0.1)))
    for it, p in zip(adam, p0[len(muon):]):
        assert torch.equal(it.param.cpu(), torch.from_numpy(p.cpu().numpy() * np.float32(1.0 - 3e-4 * 0.1)))
