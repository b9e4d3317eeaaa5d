"""The drop-in optimizer construction on the CPU (no kernel runs): mote_b200.split_muon_params, build_optimizer and
set_lr against the reference's own results on the same model (tests/golden/groups_reference.json, made by running
mote/train/muon.py:103-126 and mote/train/train.py:76-105, :177-179). A checkpoint written by the reference trainer
holds these param_groups, so a drop-in must build the same groups, in the same order, with the same keys and values,
for its load_state_dict to line the saved state up with the right parameters. Also: CPU tensors and a missing library
are refused with an error, never computed some other way."""

import json
import os
import subprocess
import sys

import pytest
import torch

from tests.conftest import GOLDEN, ROOT
from tests.golden.cases import (GROUP_KINDS, GROUP_LR, GROUP_MULTS, GROUP_SET_LR, GROUP_WD, describe_optimizer,
                                group_model, mixer_parts)


class Mamba3Mixer(torch.nn.Module):
    """Stands in for mote.model.mamba3.Mamba3Mixer: the split recognises the mixer by its class name."""

    def __init__(self):
        super().__init__()
        mixer_parts(self)


@pytest.fixture(scope="module")
def ref():
    return json.loads((GOLDEN / "groups_reference.json").read_text())


def _fused_as_here(d: dict, ref_cuda: bool) -> dict:
    """build_optimizer asks for fused=torch.cuda.is_available(): the fixture's value follows the generating machine."""
    if ref_cuda == torch.cuda.is_available():
        return d
    for o in d["opts"]:
        for g in o["groups"] + o["state_dict_groups"]:
            if "fused" in g:
                g["fused"] = torch.cuda.is_available()
    return d


def test_split_muon_params_matches_the_reference(ref):
    from mote_b200 import split_muon_params
    model = group_model(Mamba3Mixer)
    names = {id(p): n for n, p in model.named_parameters()}
    muon, other = split_muon_params(model)
    assert [names[id(p)] for p in muon] == ref["split"]["muon"]
    assert [names[id(p)] for p in other] == ref["split"]["other"]


@pytest.mark.parametrize("kind", GROUP_KINDS)
def test_build_optimizer_groups_match_the_reference(ref, kind):
    from mote_b200 import AdamW, Muon, MultiOpt, build_optimizer, set_lr
    model = group_model(Mamba3Mixer)
    opt = build_optimizer(model, GROUP_LR, GROUP_WD, GROUP_MULTS, optimizer=kind)
    assert isinstance(opt, MultiOpt) == (kind != "adamw")
    for o in (opt.opts if isinstance(opt, MultiOpt) else [opt]):
        assert isinstance(o, (AdamW, Muon))
    got = describe_optimizer(opt, model)
    want = _fused_as_here(json.loads(json.dumps(ref[kind])), ref["cuda"])
    want_lrs = want.pop("set_lr")
    assert got == want
    set_lr(opt, GROUP_SET_LR)
    assert [g["lr"] for g in opt.param_groups] == want_lrs


def test_a_reference_shaped_state_dict_loads_into_the_drop_in():
    """The param_groups of a checkpoint (train.py:385-399) load back: every saved key survives the round trip."""
    from mote_b200 import build_optimizer
    model = group_model(Mamba3Mixer)
    a = build_optimizer(model, GROUP_LR, GROUP_WD, GROUP_MULTS, optimizer="muonsw")
    sd = a.state_dict()
    b = build_optimizer(group_model(Mamba3Mixer), 1.0, 0.0, [1.0, 1.0, 1.0], optimizer="muonsw")
    b.load_state_dict(sd)
    assert b.state_dict()["multi"][0]["param_groups"] == sd["multi"][0]["param_groups"]
    assert b.state_dict()["multi"][1]["param_groups"] == sd["multi"][1]["param_groups"]


@pytest.mark.parametrize("call", ["muon", "adamw", "multi", "fused_step", "newton_schulz", "clip_grad_norm_"])
def test_cpu_tensors_are_refused_not_computed(call):
    """There is no CPU or PyTorch fallback: every entry point refuses CPU tensors with an error and leaves the
    parameters as they were."""
    from mote_b200 import AdamW, Muon, MultiOpt, clip_grad_norm_, fused_step, newton_schulz
    p = torch.nn.Parameter(torch.randn(8, 16))
    p.grad = torch.randn(8, 16)
    v = torch.nn.Parameter(torch.randn(16))
    v.grad = torch.randn(16)
    before = (p.detach().clone(), v.detach().clone())
    run = {"muon": lambda: Muon([p]).step(), "adamw": lambda: AdamW([p, v]).step(),
           "multi": lambda: MultiOpt([AdamW([v]), Muon([p])]).step(),
           "fused_step": lambda: fused_step(MultiOpt([AdamW([v]), Muon([p])]), max_norm=1.0, grad_divisor=2.0),
           "newton_schulz": lambda: newton_schulz(p.grad), "clip_grad_norm_": lambda: clip_grad_norm_([p, v], 1.0)}
    with pytest.raises(ValueError, match="GPU"):
        run[call]()
    assert torch.equal(p.detach(), before[0]) and torch.equal(v.detach(), before[1])


def test_a_missing_library_is_an_import_error():
    env = {**os.environ, "MOTEOPT_LIB": str(ROOT / "no_such_dir" / "libmoteopt.so")}
    r = subprocess.run([sys.executable, "-c", "import mote_b200._lib"], cwd=ROOT, capture_output=True, text=True,
                       env=env, timeout=300)
    assert r.returncode != 0 and "ImportError" in r.stderr and "no CPU or PyTorch fallback" in r.stderr
