"""CPU oracle for the Mote optimizer step -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of the reference optimizer step so that the CUDA product can be
checked against it. Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import it; the
product path (`mote_b200`) never does, and fails loudly if its CUDA library is missing.

What it restates (paths relative to the reference project noahsabaj/mote):

* `newton_schulz`            -- mote/train/muon.py:26-43 (quintic Newton-Schulz, bf16 per op)
* `muon_step`                -- mote/train/muon.py:52-100 (Nesterov momentum, shape batching, scale, decay, apply)
* `adamw_step`               -- torch.optim.AdamW as constructed at mote/train/train.py:98; torch is a third-party
                                dependency pinned only as ``torch>=2.6.0`` (pyproject.toml:10). Restated from torch's
                                documented single-tensor update (the path torch takes for CPU tensors), which is
                                the published decoupled-weight-decay Adam of Loshchilov & Hutter.
* `clip_grad_norm`           -- torch.nn.utils.clip_grad_norm_ as called at mote/train/train.py:946
* `moe_update_bias`          -- mote/model/moe.py:147-159 (the lossfree router's bias step, train.py:948-949)
* `ema_lerp`, `frob_norm32`  -- train.py:950-953 (the weights' EMA) and elr.py:85-87 (the ELR tracker's norms)
* `optimizer_step`           -- mote/train/train.py:944-947 followed by MultiOpt.step (train.py:64-66: AdamW, then Muon)
* `gram_newton_schulz`       -- NOT in the reference's code: the Gram Newton-Schulz variant its research notes propose
                                (docs/research/efficiency-campaign-2026-08-23.md:903-911), the specification of an
                                opt-in variant; checked by its exact-arithmetic identity with the reference iteration
                                and against the reference's own Newton-Schulz outputs (tests/test_oracle_gram_ns.py)

Rounding model. Each elementwise op rounds to the tensor's dtype exactly where the reference's tensor op does.
Where torch's CPU kernels fuse a multiply-add (``add(alpha=)``, ``lerp_``, ``addcmul_``) the oracle fuses too; this
was established by running the reference in the build container and is pinned by `tests/golden/`. bf16 matmuls are
computed with fp32 accumulation and rounded once to bf16, which is what the reference's CPU matmul does (checked
element-wise: >99.98 % of outputs identical, the rest one bf16 ulp apart).

Parity pin: `tests/golden/make_golden.py` runs the reference itself (imported from a checkout of noahsabaj/mote)
and stores its outputs; `tests/test_oracle_golden.py` checks this module against them.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

# mote/train/muon.py:31 -- quintic coefficients (a, b, c)
NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315
# mote/train/muon.py:23 -- the stack cap. It only bounds memory; the numerics do not depend on it (tested in the
# reference at tests/test_muon_batched.py:45), so the oracle orthogonalises every matrix on its own.
MAX_STACK_BYTES = 32 << 20

f32 = np.float32


# ----------------------------------------------------------------------------------------------------------------
# rounding helpers
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); returns fp32 holding bf16-representable values."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).reshape(a.shape)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.float32("nan")
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of bf16-representable fp32 values (for compact fixtures)."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def fma32(a, b, c) -> np.ndarray:
    """fp32 fused multiply-add a*b + c, rounded once (the product of two fp32 values is exact in fp64)."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(np.float32)


def _mm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """bf16 x bf16 matmul with fp32 accumulation, rounded to bf16 (torch's bf16 `@`)."""
    return bf16_round(np.matmul(a, b))


# ----------------------------------------------------------------------------------------------------------------
# Newton-Schulz
def frob_norm(x: np.ndarray) -> np.ndarray:
    """Per-matrix Frobenius norm over the last two dims, accumulated in fp64 and rounded to fp32."""
    x64 = np.asarray(x, np.float64)
    return np.sqrt((x64 * x64).sum(axis=(-2, -1), keepdims=True)).astype(np.float32)


def ns_normalize(G: np.ndarray, eps: float = 1e-7) -> np.ndarray:
    """mote/train/muon.py:32-33: X = bf16(G_fp32 / (||G||_F + eps)) per matrix."""
    X = np.asarray(G, dtype=np.float32)
    return bf16_round(X / (frob_norm(X) + f32(eps)))


def ns_iterate(X: np.ndarray, steps: int) -> np.ndarray:
    """mote/train/muon.py:34-42 on an already-normalised bf16 X (given in the caller's orientation)."""
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    a, b, c = f32(NS_A), f32(NS_B), f32(NS_C)
    for _ in range(steps):
        A = _mm(X, np.swapaxes(X, -1, -2))                                   # A = X X^T
        B = bf16_round(bf16_round(b * A) + bf16_round(c * _mm(A, A)))        # B = b*A + c*(A@A)
        X = bf16_round(bf16_round(a * X) + _mm(B, X))                        # X = a*X + B@X
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    return X


def newton_schulz(G: np.ndarray, steps: int = 5, eps: float = 1e-7) -> np.ndarray:
    """mote/train/muon.py:26-43. G: [..., m, n] (any float dtype). Returns fp32 holding bf16 values."""
    return ns_iterate(ns_normalize(G, eps), steps)


def newton_schulz_f64(G: np.ndarray, steps: int = 5, eps: float = 1e-7) -> np.ndarray:
    """The same iteration in fp64 with no rounding: the yardstick both bf16 iterations are measured against."""
    X = np.asarray(G, np.float64)
    X = X / (np.sqrt((X * X).sum(axis=(-2, -1), keepdims=True)) + eps)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = np.swapaxes(X, -1, -2)
    for _ in range(steps):
        A = X @ np.swapaxes(X, -1, -2)
        B = NS_B * A + NS_C * (A @ A)
        X = NS_A * X + B @ X
    if transposed:
        X = np.swapaxes(X, -1, -2)
    return X


# ----------------------------------------------------------------------------------------------------------------
# Gram Newton-Schulz: an opt-in variant, NOT the reference's iteration (no product kernel implements it yet)
#
# The reference's research notes (docs/research/efficiency-campaign-2026-08-23.md:903-911) propose it as a drop-in
# for muon.py's newton_schulz: since polar(X) = (X X^T)^(-1/2) X, iterate on the small m x m Gram matrix and touch
# the rectangular X only twice. Every iterate of the quintic iteration is X_k = Q_k X_0 with Q_k a polynomial in
# R_0 = X_0 X_0^T, so all of Q_k, R_k = X_k X_k^T and P_k = aI + bR_k + cR_k^2 commute and
#     X_{k+1} = P_k X_k  ->  Q_{k+1} = P_k Q_k,   R_{k+1} = P_k R_k P_k = P_k (P_k R_k).
# The schedule below (steps >= 1): R_0 = X X^T; per iteration B_k = bR_k + cR_k^2 (the polynomial phase),
# Q_1 = aI + B_0, Q_{k+1} = aQ_k + B_k Q_k, and, while another iteration follows, T = aR_k + B_k R_k,
# R_{k+1} = aT + B_k T with its upper triangle mirrored (R is symmetric); finally X = Q_steps X_0. Each product is
# one of the three kinds the Newton-Schulz kernel already runs (Gram, polynomial, a*Y + B Y), on m x m operands.

def gram_ns_eligible(m: int, n: int) -> bool:
    """Shapes the variant is for: the long side at least twice the short one. Square matrices gain no FLOPs (the
    m x m iterate costs more products than X does) and lose accuracy in bf16 (R squares X's condition number)."""
    s, l = min(m, n), max(m, n)
    return l >= 2 * s


def gram_ns_flops(m: int, n: int, steps: int = 5) -> float:
    """Algorithmic FLOPs of the schedule above: two rectangular products (4 s^2 l) and 4*steps - 3 square ones
    (steps polynomial, steps - 1 Q updates, 2 (steps - 1) R updates), 2 s^3 each."""
    s, l = min(m, n), max(m, n)
    return 4.0 * s * s * l + (4.0 * steps - 3.0) * 2.0 * s ** 3


def _fused_round(x: np.ndarray) -> np.ndarray:
    return bf16_round(np.asarray(x, np.float32))


def gram_newton_schulz(G: np.ndarray, steps: int = 5, eps: float = 1e-7) -> np.ndarray:
    """The schedule above in bf16 with fused epilogues: every product accumulates in fp32 and its output, including
    the a*Y / b*R terms added in fp32, is rounded once to bf16, as a GEMM epilogue writes it. (With the reference's
    rounding of every elementwise op the variant lands farther from the exact polar factor than the reference's own
    iteration; with one rounding per product it lands closer.) G: [..., m, n]; returns fp32 holding bf16 values."""
    if steps < 1:
        raise ValueError("steps must be >= 1")
    X = ns_normalize(G, eps)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    a, b, c = f32(NS_A), f32(NS_B), f32(NS_C)
    m = X.shape[-2]
    eye = np.eye(m, dtype=np.float32)
    R = _fused_round(np.matmul(X, np.swapaxes(X, -1, -2)))
    Q = None
    for k in range(steps):
        B = _fused_round(b * R + c * np.matmul(R, R))
        Q = _fused_round(a * eye + B) if Q is None else _fused_round(a * Q + np.matmul(B, Q))
        if k < steps - 1:
            T = _fused_round(a * R + np.matmul(B, R))
            R = _fused_round(a * T + np.matmul(B, T))
            R = np.triu(R) + np.swapaxes(np.triu(R, 1), -1, -2)
    X = _fused_round(np.matmul(Q, X))
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    return X


def block_symmetric(M: np.ndarray, block: int = 256) -> np.ndarray:
    """The matrix a kernel sees when it stores only the block x block tiles on and above the diagonal of M (m x m)
    and reads a tile below the diagonal as the transpose of its mirror tile: tiles (i, j) with i > j replaced by
    (j, i)^T; diagonal tiles as stored."""
    out = np.array(M, copy=True)
    m = M.shape[-1]
    for i0 in range(block, m, block):
        for j0 in range(0, i0, block):
            out[..., i0:i0 + block, j0:j0 + block] = np.swapaxes(M[..., j0:j0 + block, i0:i0 + block], -1, -2)
    return out


def symmetric_upper(M: np.ndarray) -> np.ndarray:
    """M with every element below the main diagonal replaced by its mirror above it (exactly symmetric)."""
    return np.triu(M) + np.swapaxes(np.triu(M, 1), -1, -2)


def gram_newton_schulz_blocked(G: np.ndarray, steps: int = 5, eps: float = 1e-7, block: int = 256) -> np.ndarray:
    """gram_newton_schulz with the storage of the library's GPU kernel (per-phase tcgen05 launches, 256 x 256 output
    tiles): R is kept exactly symmetric (its upper triangle mirrored, after X X^T and after every R update), T and Q
    are stored whole, B is computed on its upper tiles only and read through their mirrors below the diagonal, and
    the final Q X0 reads Q through its upper tiles. Every product accumulates in fp32 and rounds once to bf16 with
    its a*Y / b*R term."""
    if steps < 1:
        raise ValueError("steps must be >= 1")
    X = ns_normalize(G, eps)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    a, b, c = f32(NS_A), f32(NS_B), f32(NS_C)
    m = X.shape[-2]
    eye = np.eye(m, dtype=np.float32)
    R = symmetric_upper(_fused_round(np.matmul(X, np.swapaxes(X, -1, -2))))
    Q = None
    for k in range(steps):
        B = block_symmetric(_fused_round(b * R + c * np.matmul(R, R)), block)
        Q = _fused_round(a * eye + B) if Q is None else _fused_round(a * Q + np.matmul(B, Q))
        if k < steps - 1:
            T = _fused_round(a * R + np.matmul(B, R))
            R = symmetric_upper(_fused_round(a * T + np.matmul(B, T)))
    X = _fused_round(np.matmul(block_symmetric(Q, block), X))
    if transposed:
        X = np.ascontiguousarray(np.swapaxes(X, -1, -2))
    return X


def gram_newton_schulz_f64(G: np.ndarray, steps: int = 5, eps: float = 1e-7) -> np.ndarray:
    """The same schedule in fp64 with no rounding; in exact arithmetic it equals newton_schulz_f64."""
    if steps < 1:
        raise ValueError("steps must be >= 1")
    X = np.asarray(G, np.float64)
    X = X / (np.sqrt((X * X).sum(axis=(-2, -1), keepdims=True)) + eps)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = np.swapaxes(X, -1, -2)
    eye = np.eye(X.shape[-2])
    R = X @ np.swapaxes(X, -1, -2)
    Q = None
    for k in range(steps):
        B = NS_B * R + NS_C * (R @ R)
        Q = NS_A * eye + B if Q is None else NS_A * Q + B @ Q
        if k < steps - 1:
            T = NS_A * R + B @ R
            R = NS_A * T + B @ T
    X = Q @ X
    if transposed:
        X = np.swapaxes(X, -1, -2)
    return X


# ----------------------------------------------------------------------------------------------------------------
# Muon
@dataclass
class MuonGroup:
    """One Muon param group (mote/train/muon.py:47-48 defaults; `param_lr` per mote/train/elr.py:283-286)."""
    lr: float = 1e-3
    momentum: float = 0.95
    nesterov: bool = True
    weight_decay: float = 0.0
    ns_steps: int = 5
    rms_scale: float = 0.2
    sw_decay: bool = False
    lr_max: float = 1.0
    param_lr: Optional[Dict[int, float]] = None   # keyed by position in the group's param list


def muon_momentum(buf: np.ndarray, g: np.ndarray, mom: float, nesterov: bool) -> np.ndarray:
    """mote/train/muon.py:69-70. Updates `buf` in place, returns the update u."""
    buf[...] = np.asarray(buf * f32(mom), np.float32) + g                    # buf.mul_(mom).add_(g)
    if nesterov:
        return fma32(f32(mom), buf, g)                                        # g.add(buf, alpha=mom)
    return buf.copy()


def muon_lr_decay(group: MuonGroup, index: int):
    """mote/train/muon.py:75-79: (lr, decay) for one parameter."""
    lr, wd = group.lr, group.weight_decay
    e = lr if group.param_lr is None else group.param_lr.get(index, lr)
    d = (e * e / group.lr_max if group.sw_decay else e) * wd if wd else 0.0
    return e, d


def muon_apply(p: np.ndarray, o: np.ndarray, scale: float, lr: float, decay: float) -> None:
    """mote/train/muon.py:97-99: p *= 1-decay; p += -lr * (O.to(fp32) * scale)."""
    if decay:
        p[...] = np.asarray(p * f32(1.0 - decay), np.float32)
    t = np.asarray(o.astype(np.float32) * f32(scale), np.float32)
    p[...] = fma32(f32(-lr), t, p)


def muon_step(params: Sequence[np.ndarray], grads: Sequence[Optional[np.ndarray]], bufs: List[Optional[np.ndarray]],
              group: MuonGroup, return_updates: bool = False):
    """mote/train/muon.py:52-100 for one group. `params` are updated in place, `bufs[i]` is created on first use
    (zeros, muon.py:66-67). Parameters whose grad is None are skipped (muon.py:61-62)."""
    outs = []
    for i, (p, g) in enumerate(zip(params, grads)):
        if g is None:
            continue
        assert p.ndim in (2, 3), "Muon is for 2-D matrices (or 3-D stacks of them)"
        g = np.asarray(g, np.float32)
        if bufs[i] is None:
            bufs[i] = np.zeros_like(g, dtype=np.float32)
        u = muon_momentum(bufs[i], g, group.momentum, group.nesterov)
        m, n = p.shape[-2], p.shape[-1]
        o = newton_schulz(u.reshape(-1, m, n), steps=group.ns_steps).reshape(p.shape)
        scale = group.rms_scale * max(m, n) ** 0.5
        lr, decay = muon_lr_decay(group, i)
        muon_apply(p, o, scale, lr, decay)
        outs.append(o)
    return outs if return_updates else None


# ----------------------------------------------------------------------------------------------------------------
# AdamW (torch.optim.AdamW, single-tensor path, amsgrad=False, maximize=False)
@dataclass
class AdamWGroup:
    lr: float = 1e-3
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 1e-2


def adamw_scalars(lr: float, beta1: float, beta2: float, wd: float, step: int):
    """The per-step host scalars of torch's single-tensor AdamW, in fp64 as torch computes them:
    (1 - lr*wd, step_size, sqrt(bias_correction2))."""
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    return 1 - lr * wd, lr / bc1, bc2 ** 0.5


def adamw_update(p, g, m, v, lr, beta1, beta2, eps, wd, step) -> None:
    """One tensor's AdamW update, in place on p, m, v (all fp32). `step` is the already-incremented count."""
    g = np.asarray(g, np.float32)
    decay_mul, step_size, bc2s = adamw_scalars(lr, beta1, beta2, wd, step)
    if wd != 0:
        p[...] = np.asarray(p * f32(decay_mul), np.float32)                  # param.mul_(1 - lr*wd)
    m[...] = fma32(f32(1 - beta1), (g - m).astype(np.float32), m)           # exp_avg.lerp_(grad, 1-beta1)
    v[...] = np.asarray(v * f32(beta2), np.float32)                          # exp_avg_sq.mul_(beta2)
    v[...] = fma32(np.asarray(f32(1 - beta2) * g, np.float32), g, v)        # .addcmul_(g, g, value=1-beta2)
    denom = (np.sqrt(v) / f32(bc2s)).astype(np.float32) + f32(eps)          # (v.sqrt()/bc2_sqrt).add_(eps)
    p[...] = p + np.asarray(np.asarray(f32(-step_size) * m, np.float32) / denom, np.float32)   # addcdiv_


def adamw_step(params, grads, exp_avgs, exp_avg_sqs, steps: List[int], group: AdamWGroup) -> None:
    """torch.optim.AdamW.step for one group (train.py:98 constructs it). State tensors are created as zeros on
    first use; `steps[i]` is the per-parameter step count (torch keeps it as an fp32 scalar tensor)."""
    b1, b2 = group.betas
    for i, (p, g) in enumerate(zip(params, grads)):
        if g is None:
            continue
        if exp_avgs[i] is None:
            exp_avgs[i] = np.zeros_like(p, dtype=np.float32)
            exp_avg_sqs[i] = np.zeros_like(p, dtype=np.float32)
        steps[i] += 1
        adamw_update(p, g, exp_avgs[i], exp_avg_sqs[i], group.lr, b1, b2, group.eps, group.weight_decay, steps[i])


# ----------------------------------------------------------------------------------------------------------------
# gradient normalisation and clipping
def grad_total_norm(grads: Sequence[np.ndarray]) -> np.float32:
    """torch.nn.utils.get_total_norm (2-norm): the norm of the per-tensor norms."""
    norms = [np.float32(np.sqrt(np.sum(np.square(np.asarray(g, np.float64))))) for g in grads]
    if not norms:
        return np.float32(0.0)
    return np.float32(np.sqrt(np.sum(np.square(np.asarray(norms, np.float64)))))


def clip_coef(total_norm: np.float32, max_norm: float) -> np.float32:
    """torch clip coefficient: clamp(max_norm / (total + 1e-6), max=1), in fp32 tensor arithmetic. torch evaluates
    the Python-float-over-tensor quotient as Tensor.__rdiv__, reciprocal(total + 1e-6) * max_norm: two roundings."""
    r = np.float32(np.float32(1.0) / np.float32(np.float32(total_norm) + np.float32(1e-6)))
    c = np.float32(r * np.float32(max_norm))
    return np.float32(min(c, np.float32(1.0))) if not np.isnan(c) else c


def clip_grad_norm(grads: List[np.ndarray], max_norm: float) -> np.float32:
    """train.py:946 -> torch.nn.utils.clip_grad_norm_: scales `grads` in place and returns the total norm."""
    total = grad_total_norm(grads)
    coef = clip_coef(total, max_norm)
    for g in grads:
        g[...] = np.asarray(g * coef, np.float32)
    return total


# ----------------------------------------------------------------------------------------------------------------
# the weights' EMA and the ELR tracker's norms after the optimizer step
def ema_lerp(ema: np.ndarray, p: np.ndarray, weight: float) -> None:
    """mote/train/train.py:950-953, torch._foreach_lerp_(ema, params, weight), in place: torch's fp32 lerp,
    e + w*(p - e) for |w| < 0.5 and p - (p - e)*(1 - w) otherwise, each one fused multiply-add."""
    w = np.float32(weight)
    d = (np.asarray(p, np.float32) - ema).astype(np.float32)
    if abs(w) < np.float32(0.5):
        ema[...] = fma32(w, d, ema)
    else:
        ema[...] = fma32(-(np.float32(1.0) - w), d, p)


def frob_norm32(p: np.ndarray) -> np.float32:
    """mote/train/elr.py:85-87 (NormTracker.sample: p.detach().float().norm()) as an fp32 value from an fp64 sum."""
    return np.float32(np.sqrt(np.sum(np.asarray(p, np.float64) ** 2)))


# ----------------------------------------------------------------------------------------------------------------
# the MoE router's bias step after the optimizer step
def moe_update_bias(load: np.ndarray, bias: np.ndarray, gamma: float) -> None:
    """mote/model/moe.py:147-159 (MoESwiGLU.update_bias, called at mote/train/train.py:948-949), in place, for a
    "lossfree" router with gamma > 0 (the other cases return before touching anything, moe.py:151-152).

    fp32 tensor ops as the reference: mean = sum/E; e = (mean - load) / clamp_min(mean, 1e-9); sgn = sign(e) (0 for
    NaN); bias += fp32(gamma) * (sgn - sgn.mean()); load = 0. Nothing happens when load.sum() <= 0 (moe.py:154-155).
    The loads are token counts (integers), so their fp32 sum is exact in any order; it is formed in fp64 here."""
    E = load.size
    total = np.float32(np.sum(load.astype(np.float64)))
    if E == 0 or total <= 0:
        return
    mean = np.float32(total / np.float32(E))
    den = mean if not mean < np.float32(1e-9) else np.float32(1e-9)
    with np.errstate(invalid="ignore", divide="ignore"):
        e = ((mean - load.astype(np.float32)).astype(np.float32) / den).astype(np.float32)
    sgn = (e > 0).astype(np.float32) - (e < 0).astype(np.float32)
    sgn_mean = np.float32(np.float32(np.sum(sgn, dtype=np.float64)) / np.float32(E))
    t = (sgn - sgn_mean).astype(np.float32)
    bias[...] = (bias + (np.float32(gamma) * t).astype(np.float32)).astype(np.float32)
    load[...] = 0


# ----------------------------------------------------------------------------------------------------------------
# the trainer's whole optimizer step
@dataclass
class StepState:
    muon_bufs: List[Optional[np.ndarray]] = field(default_factory=list)
    exp_avgs: List[Optional[np.ndarray]] = field(default_factory=list)
    exp_avg_sqs: List[Optional[np.ndarray]] = field(default_factory=list)
    adam_steps: List[int] = field(default_factory=list)


def optimizer_step(muon_params, muon_grads, adam_params, adam_grads, state: StepState, muon: MuonGroup,
                   adam: AdamWGroup, max_norm: Optional[float] = 1.0, grad_divisor: Optional[float] = None):
    """mote/train/train.py:944-947: grads /= total_n; clip_grad_norm_(all params, clip); MultiOpt.step()
    (AdamW first, then Muon: train.py:64-66). Grads may be bf16-valued fp32 (the build's inputs) or fp32.
    Returns the total grad norm (before clipping), as clip_grad_norm_ does."""
    if not state.muon_bufs:
        state.muon_bufs = [None] * len(muon_params)
        state.exp_avgs = [None] * len(adam_params)
        state.exp_avg_sqs = [None] * len(adam_params)
        state.adam_steps = [0] * len(adam_params)
    mg = [np.array(g, np.float32) for g in muon_grads]
    ag = [np.array(g, np.float32) for g in adam_grads]
    allg = ag + mg   # the order does not matter for the norm's value beyond fp rounding of the final sum
    if grad_divisor is not None:
        for g in allg:
            g[...] = np.asarray(g / f32(grad_divisor), np.float32)
    total = np.float32(float("nan"))
    if max_norm is not None:
        total = clip_grad_norm(allg, max_norm)
    adamw_step(adam_params, ag, state.exp_avgs, state.exp_avg_sqs, state.adam_steps, adam)
    muon_step(muon_params, mg, state.muon_bufs, muon)
    return total


# ----------------------------------------------------------------------------------------------------------------
# synthetic inputs of the benchmark configurations (seeded; identical on every machine)
def make_rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def normal(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def bf16_normal(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    """bf16 gradients ~N(0, std^2), returned as fp32 holding bf16 values."""
    return bf16_round(normal(rng, shape, std))


def ns_flops(m: int, n: int, steps: int = 5) -> float:
    """Algorithmic Newton-Schulz FLOPs of one m x n matrix: steps * (4 s^2 l + 2 s^3), s = min, l = max."""
    s, l = min(m, n), max(m, n)
    return float(steps) * (4.0 * s * s * l + 2.0 * s ** 3)


def rel_frob(a: np.ndarray, b: np.ndarray) -> float:
    a64, b64 = np.asarray(a, np.float64), np.asarray(b, np.float64)
    den = float(np.linalg.norm(b64.ravel()))
    num = float(np.linalg.norm((a64 - b64).ravel()))
    return num / den if den else num

