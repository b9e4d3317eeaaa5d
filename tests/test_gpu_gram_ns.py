"""The opt-in Gram Newton-Schulz variant on the GPU (moteopt_muon_config::ns_variant 1; the reference's research
notes, docs/research/efficiency-campaign-2026-08-23.md:903-911; not the reference's iteration).

Against its specification with the kernel's storage (oracle.gram_newton_schulz_blocked): the same rounding points
(every product rounded once with its a*Y / b*R term) and the same storage (R exactly symmetric, B and the final Q read
through their upper 256 x 256 tiles), so only the fp32 summation order inside a product differs (the CPU's against
the tensor cores'). Measured on a B200: at most 8e-5, 2.2e-4 and 3.4e-3 after 1, 2 and 5 iterations over the shapes
below; the bars are those plus a margin. The measured distances are recorded with the session's parity record
(tests/conftest.py). Its accuracy bar is the one the reference's own iteration is held to: no farther from the exact
fp64 iteration than the library's reference iteration (measured: about half as far, 1.2-1.5e-2 against 2.3-3.4e-2).
Matrices the variant does not take (long side under twice the short one) keep the reference iteration bit for bit.
"""

import numpy as np
import pytest
import torch

from oracle import moteopt_oracle as O
from tests.conftest import record

pytestmark = pytest.mark.gpu

EXACT_SLACK = 0.0

# every Gram-eligible matrix shape of c1 (768x3072 both ways, 512x2048), c2 (1024x4096 both ways), c3 (768x2048 both
# ways), and odd, padded and multi-block ones
SHAPES = [(2, 768, 3072), (2, 3072, 768), (2, 512, 2048), (1, 1024, 4096), (1, 4096, 1024), (2, 768, 2048),
          (2, 2048, 768), (1, 600, 1800), (3, 130, 1000), (1, 520, 1100), (2, 64, 256)]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mote_b200 import ops  # noqa: F401
    return torch.device("cuda", 0)


def _input(shape, seed):
    rng = np.random.default_rng(seed)
    g = O.bf16_round(rng.standard_normal(size=shape, dtype=np.float32) * np.float32(1e-3))
    return (g + np.float32(0.95) * g).astype(np.float32)


def _ns(u, steps, dev, variant):
    from mote_b200 import ops
    return ops.newton_schulz(torch.from_numpy(u).to(dev), steps=steps, variant=variant).float().cpu().numpy()


@pytest.mark.parametrize("shape", SHAPES)
def test_gram_variant_matches_its_specification(dev, shape):
    from mote_b200 import ops
    u = _input(shape, sum(shape))
    exact = O.newton_schulz_f64(u, 5)
    d = {}
    for steps, tol in ((1, 5e-4), (2, 1e-3), (5, 1e-2)):
        g = _ns(u, steps, dev, 1)
        o = O.gram_newton_schulz_blocked(u, steps)
        d[f"k_o_{steps}"] = O.rel_frob(g, o)
        assert np.array_equal(g, O.bf16_round(g))
        assert d[f"k_o_{steps}"] <= tol, (steps, d)
    ref = _ns(u, 5, dev, 0)
    d.update(k_e=O.rel_frob(g, exact), ref_e=O.rel_frob(ref, exact), o_e=O.rel_frob(o, exact),
             k_ref=O.rel_frob(g, ref))
    record("gram_ns_vs_blocked_oracle", "x".join(map(str, shape)), d)
    st, _ = ops.read_status(dev)
    assert st & 3 == 0, st
    assert d["k_e"] <= d["ref_e"] + EXACT_SLACK, d


@pytest.mark.parametrize("shape", [(4, 768, 768), (2, 1024, 1024), (3, 130, 72), (2, 600, 1100)])
def test_matrices_the_variant_does_not_take_keep_the_reference_iteration(dev, shape):
    u = _input(shape, 5)
    assert np.array_equal(_ns(u, 5, dev, 1), _ns(u, 5, dev, 0))


def test_muon_step_with_the_variant_mixes_both_iterations(dev):
    """One Muon step over square and rectangular matrices with ns_variant 1: the square ones are bit for bit the
    reference iteration's step, the rectangular ones the variant's (against the oracle's step built on
    gram_newton_schulz_blocked, 1e-2 relative Frobenius on the update)."""
    from mote_b200.functional import MuonItem, muon_step
    rng = np.random.default_rng(9)
    shapes = [(256, 256), (768, 768), (768, 3072), (3072, 768), (512, 2048), (2, 128, 512)]
    p0 = [rng.standard_normal(s, dtype=np.float32) * np.float32(0.02) for s in shapes]
    g0 = [O.bf16_round(rng.standard_normal(s, dtype=np.float32) * np.float32(1e-3)) for s in shapes]
    out = {}
    for variant in (0, 1):
        ps = [torch.from_numpy(p.copy()).to(dev) for p in p0]
        bufs = [torch.zeros_like(p) for p in ps]
        muon_step([MuonItem(p, torch.from_numpy(g).to(dev), b, 0.02, 0.002) for p, g, b in zip(ps, g0, bufs)],
                  ns_variant=variant)
        torch.cuda.synchronize()
        out[variant] = [p.cpu().numpy() for p in ps]
    for i, s in enumerate(shapes):
        if not O.gram_ns_eligible(s[-2], s[-1]):
            assert np.array_equal(out[0][i], out[1][i]), s
            continue
        u = O.fma32(np.float32(0.95), g0[i], g0[i])   # Nesterov on a zero buffer: g + 0.95 (0.95 * 0 + g), fused
        o = O.gram_newton_schulz_blocked(u.reshape((-1,) + s[-2:]), 5).reshape(s)
        scale = np.float32(0.2 * max(s[-2], s[-1]) ** 0.5)
        want = (p0[i] * np.float32(1 - 0.002)) - np.float32(0.02) * (o * scale)
        got = out[1][i]
        assert O.rel_frob(got - p0[i], want - p0[i]) <= 1e-2, (s, O.rel_frob(got - p0[i], want - p0[i]))
        assert not np.array_equal(out[0][i], out[1][i])


def test_muon_class_opts_in(dev):
    """Muon(..., gram_ns=True) steps its eligible matrices with the variant; its param groups keep the reference's
    keys (the option is not a group key)."""
    from mote_b200 import Muon
    torch.manual_seed(0)
    a = [torch.nn.Parameter((torch.randn(s) * 0.02).to(dev)) for s in [(128, 512), (96, 96)]]
    b = [torch.nn.Parameter(p.detach().clone()) for p in a]
    for p, q in zip(a, b):
        p.grad = (torch.randn(p.shape) * 1e-3).to(dev)
        q.grad = p.grad.clone()
    o1 = Muon(a, lr=0.02, weight_decay=0.1, gram_ns=True)
    o2 = Muon(b, lr=0.02, weight_decay=0.1)
    o1.step()
    o2.step()
    assert not torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert set(o1.param_groups[0]) == set(o2.param_groups[0])
