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
