"""Benchmark / parity workloads of the optimizer step, as seeded synthetic inputs.

The shapes follow the reference's Mote presets (noahsabaj/mote mote/config.py:193-237) as the benchmark
configurations describe them: c0 is Mote-1M-shaped and CPU-sized, c1 is Mote-96M-shaped, c2 is a batched Muon
stress test, c3 an MoE expert stack, c4 an AdamW-only bandwidth sweep. The reference publishes no dataset for the
optimizer step, so every tensor is drawn from a seeded numpy generator (PCG64, identical on every machine):
params ~ N(0, 0.02^2) fp32, grads ~ N(0, 1e-3^2) rounded to bf16.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np

Shape = Tuple[int, ...]


@dataclass
class Workload:
    name: str
    muon_shapes: List[Shape]
    adam_decay_shapes: List[Shape]       # >= 2-D AdamW params (decayed; train.py:87-90)
    adam_nodecay_shapes: List[Shape]     # vectors / scalars (weight_decay 0; train.py:87-88)
    muon_lr: float = 0.02
    muon_momentum: float = 0.95
    muon_wd: float = 0.1
    ns_steps: int = 5
    adam_lr: float = 3e-4
    betas: Tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-8
    adam_wd: float = 0.1
    clip: Optional[float] = 1.0
    grad_scale: Optional[List[float]] = None   # per-Muon-param grad multipliers (c3's Zipf factors)
    notes: str = ""

    @property
    def adam_shapes(self) -> List[Shape]:
        return list(self.adam_decay_shapes) + list(self.adam_nodecay_shapes)

    def numel(self):
        m = sum(int(np.prod(s)) for s in self.muon_shapes)
        a = sum(int(np.prod(s)) for s in self.adam_shapes)
        return m, a

    def ns_flops(self) -> float:
        """Algorithmic Newton-Schulz FLOPs per step: sum over matrices of steps * (4 s^2 l + 2 s^3)."""
        tot = 0.0
        for s in self.muon_shapes:
            batch = int(np.prod(s[:-2])) if len(s) > 2 else 1
            a, b = min(s[-2], s[-1]), max(s[-2], s[-1])
            tot += batch * self.ns_steps * (4.0 * a * a * b + 2.0 * a ** 3)
        return tot

    def ns_flops_gram(self) -> float:
        """Algorithmic Newton-Schulz FLOPs per step with the opt-in Gram variant (moteopt_muon_config::ns_variant 1):
        matrices whose long side is at least twice the short one take 4 s^2 l + (4 steps - 3) 2 s^3, the others the
        reference iteration's steps (4 s^2 l + 2 s^3)."""
        tot = 0.0
        for s in self.muon_shapes:
            batch = int(np.prod(s[:-2])) if len(s) > 2 else 1
            a, b = min(s[-2], s[-1]), max(s[-2], s[-1])
            if b >= 2 * a:
                tot += batch * (4.0 * a * a * b + (4.0 * self.ns_steps - 3.0) * 2.0 * a ** 3)
            else:
                tot += batch * self.ns_steps * (4.0 * a * a * b + 2.0 * a ** 3)
        return tot

    def ns_flops_issued(self, tile: int = 256) -> float:
        """Newton-Schulz FLOPs the tensor cores perform per step: the Gram (X X^T) and polynomial (A A) products are
        symmetric, so only their output blocks on and above the diagonal (tile x tile, clipped at the edge) are
        computed; the update product B X is computed whole."""
        tot = 0.0
        for s in self.muon_shapes:
            batch = int(np.prod(s[:-2])) if len(s) > 2 else 1
            a, b = min(s[-2], s[-1]), max(s[-2], s[-1])
            edges = [min(tile, a - i) for i in range(0, a, tile)]
            upper = sum(edges[i] * edges[j] for i in range(len(edges)) for j in range(i, len(edges)))
            tot += batch * self.ns_steps * (2.0 * upper * b + 2.0 * upper * a + 2.0 * a * a * b)
        return tot

    def ns_tiles_per_iter(self, tile: int = 256) -> int:
        """256 x 256 output tiles of one Newton-Schulz iteration (upper-triangle Gram and A A blocks, full B X)."""
        tot = 0
        for s in self.muon_shapes:
            batch = int(np.prod(s[:-2])) if len(s) > 2 else 1
            a, b = min(s[-2], s[-1]), max(s[-2], s[-1])
            t, u = -(-a // tile), -(-b // tile)
            tot += batch * (t * (t + 1) + t * u)
        return tot

    def state_bytes(self) -> float:
        """Algorithmic HBM bytes per step: Muon 20 B/element (bf16 grad read twice, fp32 momentum and param read
        and written), AdamW 28 B/element (bf16 grad twice, fp32 param, exp_avg, exp_avg_sq read and written)."""
        m, a = self.numel()
        return 20.0 * m + 28.0 * a


def c0() -> Workload:
    layer = [(128, 128)] * 4 + [(128, 512), (512, 128)]
    return Workload("c0_mote1m_shaped", layer * 4, [(271, 128)], [(128,)] * 24,
                    notes="Mote-1M-shaped step (CPU-sized), 10 steps")


def c1() -> Workload:
    layer = [(768, 768)] * 4 + [(768, 3072), (3072, 768)]
    return Workload("c1_mote96m_shaped", layer * 12 + [(512, 2048)] * 8, [(271, 768)], [(768,)] * 200,
                    notes="Mote-96M-shaped single step on 1 B200")


def c2() -> Workload:
    return Workload("c2_batched_muon_stress", [(1024, 1024)] * 256 + [(1024, 4096)] * 64, [], [], clip=None,
                    notes="batched Muon stress, no AdamW")


def c3() -> Workload:
    # 64 experts; per-expert token-count factor ~ Zipf(1.1) (rank r -> r^-1.1), normalised to mean 1
    r = np.arange(1, 65, dtype=np.float64) ** -1.1
    f = (r / r.mean()).tolist()
    return Workload("c3_moe_expert_stack", [(64, 768, 2048), (64, 2048, 768)], [(768, 64)], [(64,)] * 2,
                    grad_scale=f, notes="3-D expert stacks; grads scaled per expert by a Zipf(1.1) factor")


def c4(numel: int = 100_000_000) -> Workload:
    return Workload(f"c4_adamw_flat_{numel}", [], [(numel,)], [], notes="AdamW-only bandwidth sweep")


CONFIGS = {"c0": c0, "c1": c1, "c2": c2, "c3": c3, "c4": c4}


# ----------------------------------------------------------------------------------------------------------------
def _bf16_round(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32).reshape(np.shape(x))


@dataclass
class Inputs:
    muon_params: List[np.ndarray] = field(default_factory=list)
    adam_params: List[np.ndarray] = field(default_factory=list)


def make_params(w: Workload, seed: int = 0) -> Inputs:
    """fp32 params ~ N(0, 0.02^2): AdamW tensors first, then Muon tensors, in declaration order."""
    rng = np.random.default_rng(seed)
    out = Inputs()
    for s in w.adam_shapes:
        out.adam_params.append((rng.standard_normal(size=s, dtype=np.float32) * np.float32(0.02)).astype(np.float32))
    for s in w.muon_shapes:
        out.muon_params.append((rng.standard_normal(size=s, dtype=np.float32) * np.float32(0.02)).astype(np.float32))
    return out


def make_grads(w: Workload, seed: int = 0, step: int = 0):
    """bf16-valued grads ~ N(0, 1e-3^2) for one step (returned as fp32 arrays holding bf16 values):
    (adam_grads, muon_grads). c3's per-expert factors scale each expert slice before rounding."""
    rng = np.random.default_rng([seed, 1_000_003 + step])
    ag, mg = [], []
    for s in w.adam_shapes:
        ag.append(_bf16_round(rng.standard_normal(size=s, dtype=np.float32) * np.float32(1e-3)))
    for s in w.muon_shapes:
        g = rng.standard_normal(size=s, dtype=np.float32) * np.float32(1e-3)
        if w.grad_scale is not None and len(s) == 3:
            g = g * np.asarray(w.grad_scale, np.float32)[: s[0], None, None]
        mg.append(_bf16_round(g))
    return ag, mg
