"""The drop-in optimizer construction on the CPU (no kernel runs): mote_b200.split_muon_params, build_optimizer and
set_lr against the reference's own results on the same model (tests/golden/groups_reference.json, made by running
mote/train/muon.py:103-126 and mote/train/train.py:76-105, :177-179). A checkpoint written by the reference trainer
holds these param_groups, so a drop-in must build the same groups, in the same order, with the same keys and values,
for its load_state_dict to line the saved state up with the right parameters."""

import json

import pytest
import torch

from tests.conftest import GOLDEN
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
