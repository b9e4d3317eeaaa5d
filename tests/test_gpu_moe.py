"""The lossfree MoE router's bias step on the GPU (mote/model/moe.py:147-159, called for every MoE layer after the
optimizer step at mote/train/train.py:948-949): every layer in one launch, bit for bit equal to the reference's own
outputs (tests/golden/moe_reference.npz, made by running MoESwiGLU.update_bias) and to the CPU oracle on the
cases the fixture does not hold (wide layers, more layers than one argument block, NaN loads)."""

import types

import numpy as np
import pytest
import torch

from oracle import moteopt_oracle as O
from tests.conftest import golden
from tests.golden.cases import MOE_CASES, MOE_GAMMA, MOE_STEPS, moe_bias0, moe_loads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().view(np.uint32)


def _module(dev, load, bias, gamma=MOE_GAMMA, router="lossfree"):
    """Stands in for mote.model.moe.MoESwiGLU: the four attributes update_bias reads."""
    return types.SimpleNamespace(router_kind=router, bias_gamma=gamma,
                                 _load_acc=torch.from_numpy(load.copy()).to(dev),
                                 expert_bias=torch.from_numpy(bias.copy()).to(dev))


def test_all_layers_in_one_call_match_the_reference(dev):
    from mote_b200 import moe_update_bias
    ref = golden("moe_reference")
    mods = [_module(dev, np.zeros(e, np.float32), moe_bias0(e, seed)) for _, e, _, seed in MOE_CASES]
    for step in range(MOE_STEPS):
        for m, (_, e, kind, seed) in zip(mods, MOE_CASES):
            m._load_acc.copy_(torch.from_numpy(moe_loads(e, kind, seed, step)))
        moe_update_bias(mods)
        for m, (name, *_rest) in zip(mods, MOE_CASES):
            assert np.array_equal(_bits(m.expert_bias), ref[f"{name}_bias{step}"].view(np.uint32)), (name, step)
            assert np.array_equal(_bits(m._load_acc), ref[f"{name}_load{step}"].view(np.uint32)), (name, step)


def test_skipped_layers_are_untouched(dev):
    """moe.py:151-152: a router that is not lossfree, or gamma <= 0, returns before touching bias or load."""
    from mote_b200 import moe_update_bias
    load = np.array([10.0, 2.0, 2.0, 2.0], np.float32)
    bias = np.zeros(4, np.float32)
    mods = [_module(dev, load, bias, router="aux"), _module(dev, load, bias, gamma=0.0),
            _module(dev, load, bias, gamma=-1e-3)]
    moe_update_bias(mods)
    for m in mods:
        assert np.array_equal(m._load_acc.cpu().numpy(), load) and np.array_equal(m.expert_bias.cpu().numpy(), bias)


def test_reference_case_moves_towards_balance(dev):
    """reference tests/test_moe.py:85-90: overloaded expert goes down, the others up, centred, load cleared."""
    from mote_b200 import moe_update_bias
    m = _module(dev, np.array([10.0, 2.0, 2.0, 2.0], np.float32), np.zeros(4, np.float32))
    moe_update_bias([m])
    b = m.expert_bias.cpu()
    assert b[0] < 0 and bool((b[1:] > 0).all()) and abs(float(b.sum())) < 1e-6
    assert float(m._load_acc.sum()) == 0.0


@pytest.mark.parametrize("experts,layers", [(1000, 3), (8, 600), (257, 2)])
def test_wide_and_many_layers_match_the_oracle(dev, experts, layers):
    """Layers wider than a block (1000, 257 experts) and more layers than one argument block (600 > 512)."""
    from mote_b200 import moe_update_bias
    rng = np.random.default_rng(experts * 7 + layers)
    loads = [rng.integers(0, 3000, size=experts).astype(np.float32) for _ in range(layers)]
    biases = [rng.uniform(-0.1, 0.1, size=experts).astype(np.float32) for _ in range(layers)]
    gammas = [float(g) for g in rng.uniform(1e-4, 1e-2, size=layers)]
    rows = [(torch.from_numpy(ld.copy()).to(dev), torch.from_numpy(b.copy()).to(dev), g)
            for ld, b, g in zip(loads, biases, gammas)]
    moe_update_bias(rows)
    for (ld_t, b_t, _), ld, b, g in zip(rows, loads, biases, gammas):
        O.moe_update_bias(ld, b, g)
        assert np.array_equal(_bits(b_t), b.view(np.uint32))
        assert np.array_equal(_bits(ld_t), ld.view(np.uint32))


def test_nan_and_zero_loads_follow_the_reference_rules(dev):
    """A NaN load makes the sum NaN: `load.sum() <= 0` is false, every sign is 0 (torch.sign(NaN) = 0), the bias is
    unchanged and the load cleared. An all-zero load returns early and keeps everything."""
    from mote_b200 import moe_update_bias
    nan = np.array([3.0, np.nan, 1.0, 5.0], np.float32)
    zero = np.zeros(6, np.float32)
    b4 = np.array([0.1, -0.2, 0.3, 0.0], np.float32)
    b6 = np.linspace(-0.1, 0.1, 6).astype(np.float32)
    rows = [(torch.from_numpy(nan.copy()).to(dev), torch.from_numpy(b4.copy()).to(dev), 1e-3),
            (torch.from_numpy(zero.copy()).to(dev), torch.from_numpy(b6.copy()).to(dev), 1e-3)]
    moe_update_bias(rows)
    for (ld_t, b_t, g), ld, b in zip(rows, (nan, zero), (b4, b6)):
        O.moe_update_bias(ld, b, g)
        assert np.array_equal(_bits(b_t), b.view(np.uint32))
        assert np.array_equal(_bits(ld_t), ld.view(np.uint32))


def test_captured_in_a_cuda_graph(dev):
    """No host round trip: the step records into a CUDA graph, and replays equal eager calls bit for bit."""
    from mote_b200 import moe_update_bias
    e = 64
    rng = np.random.default_rng(5)
    loads = [rng.integers(0, 4000, size=e).astype(np.float32) for _ in range(3)]
    eager_load = torch.zeros(e, device=dev)
    eager_bias = torch.zeros(e, device=dev)
    g_load = torch.zeros(e, device=dev)
    g_bias = torch.zeros(e, device=dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):   # warm the library up outside the capture
        moe_update_bias([(g_load, g_bias, 1e-3)])
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        moe_update_bias([(g_load, g_bias, 1e-3)])
    torch.cuda.synchronize(dev)
    g_bias.zero_()
    for ld in loads:
        eager_load.copy_(torch.from_numpy(ld))
        moe_update_bias([(eager_load, eager_bias, 1e-3)])
        g_load.copy_(torch.from_numpy(ld))
        graph.replay()
    torch.cuda.synchronize(dev)
    assert np.array_equal(_bits(g_bias), _bits(eager_bias))
    assert float(g_load.abs().sum()) == 0.0
    del graph


def test_fused_step_runs_the_bias_step_after_the_optimizer(dev):
    """fused_step(opt, ..., moe=layers) = the optimizer step, then every layer's update_bias (train.py:947-949)."""
    from mote_b200 import AdamW, fused_step
    p = torch.nn.Parameter(torch.randn(64, device=dev) * 0.02)
    p.grad = torch.randn(64, device=dev) * 1e-3
    opt = AdamW([p], lr=3e-4)
    loads = [np.array([10.0, 2.0, 2.0, 2.0], np.float32), np.arange(12, dtype=np.float32)]
    biases = [np.zeros(4, np.float32), np.linspace(-0.01, 0.01, 12).astype(np.float32)]
    mods = [_module(dev, ld, b) for ld, b in zip(loads, biases)] + [_module(dev, loads[0], biases[0], router="aux")]
    fused_step(opt, max_norm=1.0, moe=mods)
    for m, ld, b in zip(mods[:2], loads, biases):
        ld, b = ld.copy(), b.copy()
        O.moe_update_bias(ld, b, MOE_GAMMA)
        assert np.array_equal(_bits(m.expert_bias), b.view(np.uint32))
        assert np.array_equal(_bits(m._load_acc), ld.view(np.uint32))
    assert np.array_equal(mods[2]._load_acc.cpu().numpy(), loads[0])   # not lossfree: untouched
