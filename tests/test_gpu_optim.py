"""The drop-in classes on the GPU: the reference's own optimizer tests replayed through mote_b200.Muon / AdamW /
MultiOpt (reference tests/test_muon_batched.py, tests/test_moe.py:105-123, tests/test_elr.py:145-195,
tests/test_resume_bitwise.py), and AdamW against torch.optim.AdamW itself."""

import io

import numpy as np
import pytest
import torch

from tests.conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _pair(shapes, dev, seed=0):
    torch.manual_seed(seed)
    ps = [torch.nn.Parameter(torch.randn(*s).to(dev)) for s in shapes]
    for p in ps:
        p.grad = torch.randn_like(p)
    return ps


def test_muon_batched_step_matches_reference_fixture(dev):
    """reference tests/test_muon_batched.py:46-67 through the Muon class (3 steps, Muon-SW off and on)."""
    from mote_b200 import Muon
    g = golden("muon_reference")
    for sw in (0, 1):
        ps = [torch.nn.Parameter(torch.from_numpy(g[f"batched_p0_{i}"].copy()).to(dev)) for i in range(6)]
        opt = Muon(ps, lr=1e-2, momentum=0.95, nesterov=True, weight_decay=0.1, sw_decay=bool(sw), lr_max=2e-2)
        for it in range(3):
            for i, p in enumerate(ps):
                p.grad = (torch.from_numpy(g[f"batched_g_{i}"].copy()) * (1.0 + 0.1 * it)).to(dev)
            opt.step()
        for i, p in enumerate(ps):
            assert torch.allclose(p.detach().cpu(), torch.from_numpy(g[f"batched_sw{sw}_p3_{i}"]), atol=2e-3, rtol=1e-2)


def test_muon_stack_equals_its_slices(dev):
    """reference tests/test_moe.py:105-123: a 3-D [3,24,40] stack steps like its three slices."""
    from mote_b200 import Muon
    torch.manual_seed(0)
    stack = torch.nn.Parameter((torch.randn(3, 24, 40) * 0.1).to(dev))
    g = (torch.randn(3, 24, 40) * 0.01).to(dev)
    slices = [torch.nn.Parameter(stack[i].detach().clone()) for i in range(3)]
    o1 = Muon([stack], lr=1e-2, weight_decay=0.1)
    o2 = Muon(slices, lr=1e-2, weight_decay=0.1)
    for it in range(3):
        stack.grad = g * (1 + 0.1 * it)
        for i, s in enumerate(slices):
            s.grad = (g[i] * (1 + 0.1 * it)).contiguous()
        o1.step()
        o2.step()
    for i in range(3):
        # same matrices, same batch position rules: identical, not just close
        assert torch.equal(stack[i], slices[i]), i
    gref = golden("muon_reference")
    assert np.allclose(stack.detach().cpu().numpy(), gref["stack_p3"], atol=2e-3, rtol=1e-2)


def test_param_lr_matching_the_group_lr_is_a_no_op(dev):
    """reference tests/test_elr.py:145-157: bit-identical."""
    from mote_b200 import Muon
    a = _pair([(8, 8), (8, 16), (16, 8)], dev)
    b = [torch.nn.Parameter(p.detach().clone()) for p in a]
    for p, q in zip(a, b):
        q.grad = p.grad.clone()
    o1 = Muon(a, lr=1e-2, weight_decay=0.1, lr_max=1e-2)
    o2 = Muon(b, lr=1e-2, weight_decay=0.1, lr_max=1e-2)
    o2.param_groups[0]["param_lr"] = {id(q): 1e-2 for q in b}
    o1.step()
    o2.step()
    for p, q in zip(a, b):
        assert torch.equal(p, q)


def test_param_lr_gives_each_matrix_its_own_rate(dev):
    """reference tests/test_elr.py:159-172."""
    from mote_b200 import Muon
    a = _pair([(8, 8), (8, 8)], dev)
    b = [torch.nn.Parameter(p.detach().clone()) for p in a]
    for p, q in zip(a, b):
        q.grad = p.grad.clone()
    o1 = Muon(a, lr=1e-2, weight_decay=0.0)
    o2 = Muon(b, lr=1e-2, weight_decay=0.0)
    o2.param_groups[0]["param_lr"] = {id(b[0]): 1e-2, id(b[1]): 2e-2}
    o1.step()
    o2.step()
    assert torch.equal(a[0], b[0])
    assert not torch.allclose(a[1], b[1])
    start = _pair([(8, 8), (8, 8)], dev)[1]
    assert torch.allclose(b[1] - start, 2.0 * (a[1] - start), atol=1e-6)


def test_param_lr_scales_the_decay_with_the_rate(dev):
    """reference tests/test_elr.py:174-182."""
    from mote_b200 import Muon
    p = torch.nn.Parameter((torch.eye(8) * 3.0).to(dev))
    p.grad = torch.zeros_like(p)
    o = Muon([p], lr=1e-2, weight_decay=0.1)
    o.param_groups[0]["param_lr"] = {id(p): 5e-2}
    o.step()
    assert p[0, 0].item() == pytest.approx(3.0 * (1 - 5e-2 * 0.1), rel=1e-6)


def test_adamw_class_matches_torch_adamw(dev):
    """Our AdamW (GPU kernel) against torch.optim.AdamW's own CPU single-tensor update, 5 steps, two groups."""
    from mote_b200 import AdamW
    rng = np.random.default_rng(3)
    shapes = [(271, 64), (64,), (3, 5, 7)]
    p0 = [rng.standard_normal(s).astype(np.float32) * np.float32(0.02) for s in shapes]
    ours = [torch.nn.Parameter(torch.from_numpy(x.copy()).to(dev)) for x in p0]
    ref = [torch.nn.Parameter(torch.from_numpy(x.copy())) for x in p0]
    mk = lambda ps, cls, **kw: cls([{"params": [ps[0], ps[2]], "weight_decay": 0.1},  # noqa: E731
                                   {"params": [ps[1]], "weight_decay": 0.0}], lr=3e-4, betas=(0.9, 0.95), eps=1e-8, **kw)
    o1 = mk(ours, AdamW)
    o2 = mk(ref, torch.optim.AdamW, fused=False, foreach=False)
    for _ in range(5):
        gs = [rng.standard_normal(s).astype(np.float32) * np.float32(1e-3) for s in shapes]
        for p, q, x in zip(ours, ref, gs):
            p.grad = torch.from_numpy(x.copy()).to(dev)
            q.grad = torch.from_numpy(x.copy())
        o1.step()
        o2.step()
    for p, q in zip(ours, ref):
        a, b = o1.state[p], o2.state[q]
        assert float(a["step"]) == float(b["step"]) == 5.0
        for k in ("exp_avg", "exp_avg_sq"):
            x, y = a[k].cpu().numpy().astype(np.float64), b[k].numpy().astype(np.float64)
            rms = np.sqrt(np.mean(y * y))
            assert (np.abs(x - y) <= 1e-6 * np.maximum(np.abs(y), rms)).all(), k
        x, y = p.detach().cpu().numpy().astype(np.float64), q.detach().numpy().astype(np.float64)
        assert (np.abs(x - y) <= 1e-6 * np.maximum(np.abs(y), np.sqrt(np.mean(y * y))) + 1e-9).all()
    # the state_dict layout is torch's
    s1, s2 = o1.state_dict(), o2.state_dict()
    assert set(s1["state"][0]) == set(s2["state"][0])
    assert set(s1["param_groups"][0]) == set(s2["param_groups"][0])


def _tiny_model(dev):
    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.embeddings = torch.nn.Embedding(271, 32)
            self.lm_head = torch.nn.Linear(32, 271, bias=False)
            self.lm_head.weight = self.embeddings.weight
            self.w1 = torch.nn.Linear(32, 64, bias=False)
            self.w2 = torch.nn.Linear(64, 32, bias=False)
            self.norm = torch.nn.Parameter(torch.ones(32))
            self.experts = torch.nn.Parameter(torch.randn(4, 32, 48) * 0.02)
            self.experts._muon_stack = True

        def stage_param_groups(self):
            return {0: [self.embeddings.weight, self.norm], 1: [self.w1.weight, self.w2.weight, self.experts]}

    torch.manual_seed(0)
    return M().to(dev)


def _grads(model, step):
    g = torch.Generator().manual_seed(100 + step)
    for p in model.parameters():
        p.grad = (torch.randn(p.shape, generator=g) * 1e-2).to(p.device)


def test_fused_step_equals_clip_then_step(dev):
    """fused_step(opt, clip, n) == torch._foreach_div_ + clip_grad_norm_ + opt.step() (train.py:944-947)."""
    from mote_b200 import build_optimizer, fused_step
    m1, m2 = _tiny_model(dev), _tiny_model(dev)
    o1 = build_optimizer(m1, 1e-2, 0.1, [2.0, 1.0], optimizer="muon")
    o2 = build_optimizer(m2, 1e-2, 0.1, [2.0, 1.0], optimizer="muon")
    for step in range(3):
        _grads(m1, step)
        _grads(m2, step)
        n1 = fused_step(o1, max_norm=0.05, grad_divisor=3.0)
        grads = [p.grad for p in m2.parameters()]
        torch._foreach_div_(grads, 3.0)
        n2 = torch.nn.utils.clip_grad_norm_(m2.parameters(), 0.05)
        o2.step()
        assert abs(n1.item() - n2.item()) <= 1e-5 * n2.item()
    for p, q in zip(m1.parameters(), m2.parameters()):
        assert torch.allclose(p, q, rtol=1e-5, atol=1e-6)


def test_resume_is_bitwise(dev):
    """reference tests/test_resume_bitwise.py: N straight steps == k steps + state_dict save/load + N-k steps."""
    from mote_b200 import build_optimizer, fused_step

    def run(steps, resume_at=None):
        m = _tiny_model(dev)
        o = build_optimizer(m, 1e-2, 0.1, [2.0, 1.0], optimizer="muon")
        for s in range(steps):
            if resume_at is not None and s == resume_at:
                buf = io.BytesIO()
                torch.save({"model": m.state_dict(), "optimizer": o.state_dict()}, buf)
                buf.seek(0)
                ck = torch.load(buf, weights_only=True)
                m = _tiny_model(dev)
                o = build_optimizer(m, 1e-2, 0.1, [2.0, 1.0], optimizer="muon")
                m.load_state_dict(ck["model"])
                o.load_state_dict(ck["optimizer"])
            _grads(m, s)
            fused_step(o, max_norm=1.0)
        return m, o

    a, _ = run(6)
    b, _ = run(6, resume_at=3)
    for p, q in zip(a.parameters(), b.parameters()):
        assert torch.equal(p, q)


def test_state_dict_layout_matches_the_reference(dev):
    from mote_b200 import build_optimizer
    m = _tiny_model(dev)
    o = build_optimizer(m, 1e-3, 0.1, [2.0, 1.0], optimizer="muonsw")
    _grads(m, 0)
    o.step()
    sd = o.state_dict()
    assert list(sd) == ["multi"] and len(sd["multi"]) == 2
    adam_sd, muon_sd = sd["multi"]
    for st in adam_sd["state"].values():
        assert set(st) == {"step", "exp_avg", "exp_avg_sq"} and st["step"].dtype == torch.float32 and st["step"].ndim == 0
    for st in muon_sd["state"].values():
        assert set(st) == {"momentum_buffer"} and st["momentum_buffer"].dtype == torch.float32
    g = muon_sd["param_groups"][0]
    for k in ("lr", "momentum", "nesterov", "weight_decay", "ns_steps", "rms_scale", "sw_decay", "lr_max", "lr_mult", "stage"):
        assert k in g
    assert g["sw_decay"] is True


def test_multiopt_step_is_one_library_call_with_the_separate_steps_bits(dev, monkeypatch):
    """MultiOpt.step (train.py:64-66) over this package's AdamW + Muon runs as one library call (one optimizer_step:
    AdamW, then Muon), and gives the same bits as AdamW.step() followed by Muon.step(), over 3 steps."""
    from mote_b200 import build_optimizer
    from mote_b200 import functional as F
    m1, m2 = _tiny_model(dev), _tiny_model(dev)
    o1 = build_optimizer(m1, 1e-2, 0.1, [2.0, 1.0], optimizer="muonsw")
    o2 = build_optimizer(m2, 1e-2, 0.1, [2.0, 1.0], optimizer="muonsw")
    calls = {"step": 0, "adamw": 0, "muon": 0}
    real = F.optimizer_step

    def counting(*a, **k):
        calls["step"] += 1
        return real(*a, **k)
    monkeypatch.setattr(F, "optimizer_step", counting)
    for step in range(3):
        _grads(m1, step)
        _grads(m2, step)
        o1.step()
        for o in o2.opts:   # the two optimizers one after the other, as the reference's MultiOpt steps them
            o.step()
    assert calls["step"] == 3
    for p, q in zip(m1.parameters(), m2.parameters()):
        assert torch.equal(p, q)
    for s1, s2 in zip(o1.state_dict()["multi"], o2.state_dict()["multi"]):
        for k in s1["state"]:
            for name, t in s1["state"][k].items():
                assert torch.equal(t, s2["state"][k][name]), (k, name)


def test_device_divisor_equals_the_host_divisor_and_never_syncs(dev, monkeypatch):
    """train.py:945 divides by total_n, a GPU tensor: fused_step(grad_divisor=tensor) reads it on the device (no
    .item(), no host synchronisation) and gives the same bits as the same divisor passed as a number; an int64
    total_n is converted on the device. A CapturedStep reads an fp32 device divisor in place at every replay."""
    from mote_b200 import build_optimizer, fused_step
    from mote_b200.functional import AdamWItem, CapturedStep, MuonItem, optimizer_step
    m1, m2 = _tiny_model(dev), _tiny_model(dev)
    o1 = build_optimizer(m1, 1e-2, 0.1, [2.0, 1.0], optimizer="muon")
    o2 = build_optimizer(m2, 1e-2, 0.1, [2.0, 1.0], optimizer="muon")

    real_item = torch.Tensor.item

    def no_item(self):   # a CPU tensor's item() (AdamW's step count) does not wait on the GPU
        if self.is_cuda:
            raise AssertionError("host synchronisation: Tensor.item() called on a GPU tensor")
        return real_item(self)
    for step in range(3):
        _grads(m1, step)
        _grads(m2, step)
        total_n = torch.tensor(3 + step, device=dev)   # int64, as a token count
        monkeypatch.setattr(torch.Tensor, "item", no_item)
        n1 = fused_step(o1, max_norm=0.05, grad_divisor=total_n)
        monkeypatch.undo()
        n2 = fused_step(o2, max_norm=0.05, grad_divisor=float(3 + step))
        assert torch.equal(n1, n2)
    for p, q in zip(m1.parameters(), m2.parameters()):
        assert torch.equal(p, q)
    # captured: the divisor tensor is updated in place between replays
    gen = torch.Generator(device=dev)
    gen.manual_seed(9)
    ps = [torch.randn(s, generator=gen, device=dev) * 0.02 for s in [(64, 96), (96, 64)]]
    gs = [(torch.randn(p.shape, generator=gen, device=dev) * 1e-3).to(torch.bfloat16) for p in ps]
    a = torch.randn(300, generator=gen, device=dev) * 0.02
    ag = (torch.randn(300, generator=gen, device=dev) * 1e-3).to(torch.bfloat16)
    sets = [([p.clone() for p in ps], [torch.zeros_like(p) for p in ps], a.clone(), torch.zeros_like(a),
             torch.zeros_like(a)) for _ in range(2)]
    divs = [2.0, 5.0, 7.0, 3.0]
    mp, mb, ap, am, av = sets[0]
    for k, d in enumerate(divs):
        optimizer_step([MuonItem(p, g, b, 0.02, 0.002) for p, g, b in zip(mp, gs, mb)],
                       [AdamWItem(ap, ag, am, av, 3e-4, 0.1, k + 1)], betas=(0.9, 0.95), max_norm=0.01,
                       grad_divisor=d)
    mp2, mb2, ap2, am2, av2 = sets[1]
    div_t = torch.zeros((), device=dev)
    cs = CapturedStep([MuonItem(p, g, b, 0.02, 0.002) for p, g, b in zip(mp2, gs, mb2)],
                      [AdamWItem(ap2, ag, am2, av2, 3e-4, 0.1, 0)], betas=(0.9, 0.95), max_norm=0.01,
                      grad_divisor=div_t)
    for d in divs:
        div_t.fill_(d)
        cs()
    torch.cuda.synchronize()
    assert cs.graph is not None
    for x, y in zip(mp + mb + [ap, am, av], mp2 + mb2 + [ap2, am2, av2]):
        assert torch.equal(x, y)
