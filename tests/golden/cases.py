"""Inputs of the golden fixtures, shared by the generator (make_golden.py) and the tests. No reference import."""

import numpy as np

from mote_b200 import configs

NS_CASES = [  # (name, shape, seed)
    ("sq40", (40, 40), 1),
    ("wide64x48", (48, 64), 2),
    ("tall64x48", (64, 48), 3),
    ("stack3x24x40", (3, 24, 40), 4),
    ("tall2x130x72", (2, 130, 72), 5),
    ("wide96x200", (96, 200), 6),
    ("sq128", (2, 128, 128), 7),
    ("wide128x512", (128, 512), 8),
    ("odd37x53", (37, 53), 10),
]
NS_STEPS = (1, 2, 5)

ADAM_SHAPES = [(271, 16), (24,), (5, 7), (1,), (3, 1000)]
ADAM_WDS = [0.1, 0.0, 0.1, 0.0, 0.1]

SAMPLES = 256
C0_DIVISOR = 4.0   # train.py:945 divides the grads by the token count; the fixtures use this fixed stand-in


def ns_input(shape, seed):
    """A Nesterov-like update u = g + 0.95 g of bf16 grads, the first-step input Muon hands to Newton-Schulz."""
    rng = np.random.default_rng(seed)
    g = configs._bf16_round(rng.standard_normal(size=shape, dtype=np.float32) * np.float32(1e-3))
    return (g + np.float32(0.95) * g).astype(np.float32)


def sample_index(numel: int, k: int = SAMPLES) -> np.ndarray:
    """Fixed element indices of one tensor that the c0 fixture stores."""
    rng = np.random.default_rng(numel)
    return np.sort(rng.choice(numel, size=min(k, numel), replace=False))


# the lossfree router's bias step (mote/model/moe.py:147-159): (name, experts, load kind, seed); gamma per case below
MOE_CASES = [
    ("zipf64", 64, "zipf", 21),
    ("balanced8", 8, "equal", 22),
    ("odd12", 12, "uniform", 23),
    ("idle16", 16, "zero", 24),
    ("onehot5", 5, "onehot", 25),
    ("ties4", 4, "ties", 26),
    ("wide256", 256, "uniform", 27),
    ("pair2", 2, "uniform", 28),
]
MOE_GAMMA = 1e-3
MOE_STEPS = 3


def moe_loads(experts: int, kind: str, seed: int, step: int) -> np.ndarray:
    """Token counts per expert for one step of a MOE_CASES case (integers stored as fp32, as the router's _load_acc)."""
    rng = np.random.default_rng(seed * 100 + step)
    if kind == "zipf":
        x = np.minimum(rng.zipf(1.3, size=experts), 50000)
    elif kind == "equal":
        x = np.full(experts, 4096)
    elif kind == "zero":
        x = np.zeros(experts)
    elif kind == "onehot":
        x = np.zeros(experts)
        x[step % experts] = 2048
    elif kind == "ties":
        x = np.array([1, 2, 3, 2][:experts]) * (step + 1)
    else:
        x = rng.integers(0, 5000, size=experts)
    return x.astype(np.float32)


def moe_bias0(experts: int, seed: int) -> np.ndarray:
    """The expert bias a case starts from."""
    return np.random.default_rng(seed).uniform(-0.05, 0.05, size=experts).astype(np.float32)


# optimizer construction (mote/train/train.py:76-105 build_optimizer, mote/train/muon.py:103-126 split_muon_params,
# train.py:177-179 set_lr): a model with one parameter of every kind the split distinguishes, in three stages
GROUP_LR = 3e-3
GROUP_WD = 0.1
GROUP_MULTS = [2.0, 1.0, 0.5]
GROUP_KINDS = ("adamw", "muon", "muonsw")
GROUP_SET_LR = 1.5e-3


def mixer_parts(mod) -> None:
    """The two projections of a Mamba-3 mixer that the split looks at: `in_proj` goes to AdamW, `out_proj` to Muon.
    Both the test's stand-in class and the generator's subclass of the reference's Mamba3Mixer call this."""
    import torch
    mod.in_proj = torch.nn.Linear(16, 40, bias=False)
    mod.out_proj = torch.nn.Linear(20, 16, bias=False)


def group_model(mixer_cls):
    """Embeddings with a tied head, a Mamba-3 mixer, a 3-D MoE expert stack (`_muon_stack`), a router
    (`_no_muon`), a 2-D `_no_weight_decay` gain, a 3-D conv kernel without the stack flag, vectors, a frozen matrix,
    and a stage with no matrix for Muon."""
    import torch

    class GroupModel(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.embeddings = torch.nn.Embedding(50, 16)
            self.lm_head = torch.nn.Linear(16, 50, bias=False)
            self.lm_head.weight = self.embeddings.weight
            self.norm0 = torch.nn.Parameter(torch.ones(16))
            self.mixer = mixer_cls()
            self.conv = torch.nn.Parameter(torch.zeros(4, 1, 8))
            self.gain = torch.nn.Parameter(torch.ones(1, 16))
            self.gain._no_weight_decay = True
            self.w1 = torch.nn.Linear(16, 32)
            self.w2 = torch.nn.Linear(32, 16, bias=False)
            self.experts = torch.nn.Parameter(torch.zeros(4, 16, 24))
            self.experts._muon_stack = True
            self.router = torch.nn.Parameter(torch.zeros(4, 16))
            self.router._no_muon = True
            self.frozen = torch.nn.Parameter(torch.zeros(8, 8), requires_grad=False)
            self.head_norm = torch.nn.Parameter(torch.ones(16))
            self.scale = torch.nn.Parameter(torch.ones(()))

        def stage_param_groups(self):
            return {0: [self.embeddings.weight, self.norm0, self.mixer.in_proj.weight, self.mixer.out_proj.weight,
                        self.conv, self.gain],
                    1: [self.w1.weight, self.w1.bias, self.w2.weight, self.experts, self.router, self.frozen],
                    2: [self.head_norm, self.scale]}

    torch.manual_seed(0)
    return GroupModel()


def _jsonable(v):
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    if isinstance(v, dict):
        return {k: _jsonable(x) for k, x in v.items()}
    if hasattr(v, "item"):   # a 0-dim tensor (lr, betas given as tensors)
        return float(v.item())
    return v


def describe_optimizer(opt, model) -> dict:
    """What a drop-in must reproduce of a freshly built optimizer: whether it is a MultiOpt, and per optimizer its kind,
    every param group (parameter names in order and every other key) and the param_groups of its state_dict (what a
    checkpoint stores)."""
    names = {id(p): n for n, p in model.named_parameters()}
    opts = opt.opts if hasattr(opt, "opts") else [opt]
    out = {"multi": hasattr(opt, "opts"), "opts": []}
    for o in opts:
        groups = [{"params": [names[id(p)] for p in g["params"]],
                   **{k: _jsonable(v) for k, v in sorted(g.items()) if k != "params"}} for g in o.param_groups]
        sd = o.state_dict()
        out["opts"].append({"kind": "muon" if "ns_steps" in o.defaults else "adamw", "groups": groups,
                            "state_dict_groups": _jsonable(sd["param_groups"]), "state": len(sd["state"])})
    return out
