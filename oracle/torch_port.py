"""The reference optimizer step run by torch on the host CPU -- TEST AND BASELINE INFRASTRUCTURE ONLY.

`bench.py --impl reference` times the reference's own CPU implementation of the optimizer step. The reference
(noahsabaj/mote) is Python on top of torch and is not installed on the GPU host, so this module performs its step
with the same torch CPU operations, in the same order and on the same dtypes:

* `newton_schulz`  -- mote/train/muon.py:26-43: per-matrix Frobenius normalisation in fp32, then the quintic
                      iteration in bf16 on the side with fewer rows
* `muon_update`    -- mote/train/muon.py:52-99 for one param group: momentum and Nesterov look-ahead in place,
                      Newton-Schulz batched per matrix shape in stacks of at most MAX_STACK_BYTES (muon.py:23,
                      :81-90), decoupled decay and the scaled apply
* `optimizer_step` -- mote/train/train.py:944-947: grads divided by the token count, torch.nn.utils.clip_grad_norm_,
                      then the AdamW step (torch.optim.AdamW itself, the third-party class train.py:98 builds) and
                      the Muon step

Because the operations are torch's own, its results equal the reference's bit for bit on the same host
(tests/test_oracle_torch_port.py checks them against the fixtures made by running the reference). The numpy oracle
(moteopt_oracle.py) remains the parity checker of the CUDA path: it spells out every rounding point. Only `tests/`
and `bench.py`'s reference arm import this module.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .moteopt_oracle import MAX_STACK_BYTES, NS_A, NS_B, NS_C


@torch.no_grad()
def newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7, exact_norm: bool = False) -> torch.Tensor:
    """mote/train/muon.py:26-43 on a tensor G [..., m, n] (CPU or CUDA); returns bf16. `exact_norm` replaces torch's
    fp32 reduction for ||G||_F by the correctly rounded norm (an fp64 sum of the exactly squared fp32 entries, its
    square root rounded to fp32): the one place where two faithful runs of muon.py:33 can differ in the last bit."""
    g32 = G.to(torch.float32)
    if exact_norm:
        nrm = g32.double().square().sum(dim=(-2, -1), keepdim=True).sqrt().to(torch.float32)
    else:
        nrm = g32.norm(dim=(-2, -1), keepdim=True)
    X = (g32 / (nrm + eps)).to(torch.bfloat16)
    wide_side = X.shape[-2] > X.shape[-1]
    if wide_side:
        X = X.transpose(-2, -1)
    for _ in range(steps):
        A = X @ X.transpose(-2, -1)
        B = NS_B * A + NS_C * (A @ A)
        X = NS_A * X + B @ X
    return X.transpose(-2, -1) if wide_side else X


def stacks(shapes: Sequence[Tuple[int, ...]], elem_bytes: int = 4) -> List[Tuple[Tuple[int, int], List[int]]]:
    """The Newton-Schulz launches of one Muon step, in order: per matrix shape (m, n) (first-seen order), the indices
    of the params stacked into each launch, at most MAX_STACK_BYTES // (m n elem_bytes) params per launch; a 3-D
    param counts as one item however many slices it holds (muon.py:81-90)."""
    by_shape: Dict[Tuple[int, int], List[int]] = {}
    for i, s in enumerate(shapes):
        by_shape.setdefault((s[-2], s[-1]), []).append(i)
    out = []
    for (m, n), idx in by_shape.items():
        per = max(1, MAX_STACK_BYTES // max(m * n * elem_bytes, 1))
        for k in range(0, len(idx), per):
            out.append(((m, n), idx[k:k + per]))
    return out


@torch.no_grad()
def muon_update(params: Sequence[torch.Tensor], bufs: List[Optional[torch.Tensor]], *, lr: float,
                momentum: float = 0.95, nesterov: bool = True, weight_decay: float = 0.0, ns_steps: int = 5,
                rms_scale: float = 0.2, sw_decay: bool = False, lr_max: float = 1.0, exact_norm: bool = False) -> None:
    """mote/train/muon.py:52-99 for one param group without `param_lr`: `params` carry `.grad`; `bufs[i]` is the
    momentum buffer of params[i], created on first use (zeros like the grad). The decay is lr * wd, or
    lr^2 / lr_max * wd under Muon-SW (muon.py:76-79). `exact_norm` as for newton_schulz."""
    upd: Dict[int, torch.Tensor] = {}
    live = []
    for i, p in enumerate(params):
        g = p.grad
        if g is None:
            continue
        if bufs[i] is None:
            bufs[i] = torch.zeros_like(g)
        bufs[i].mul_(momentum).add_(g)
        u = g.add(bufs[i], alpha=momentum) if nesterov else bufs[i]
        upd[i] = u.reshape(-1, p.shape[-2], p.shape[-1])
        live.append(i)
    decay = ((lr * lr / lr_max) if sw_decay else lr) * weight_decay if weight_decay else 0.0
    elem = upd[live[0]].element_size() if live else 4
    for (m, n), idx in stacks([tuple(params[i].shape) for i in live], elem):
        members = [live[j] for j in idx]
        batch = torch.cat([upd[i] for i in members], dim=0) if len(members) > 1 else upd[members[0]]
        orth = newton_schulz(batch, steps=ns_steps, exact_norm=exact_norm)
        scale = rms_scale * max(m, n) ** 0.5
        row = 0
        for i in members:
            p = params[i]
            k = upd[i].shape[0]
            o = orth[row:row + k].reshape(p.shape)
            row += k
            if decay:
                p.mul_(1.0 - decay)
            p.add_(o.to(p.dtype) * scale, alpha=-lr)


@torch.no_grad()
def clip_grad_norm_exact_(params: Sequence[torch.Tensor], max_norm: float) -> torch.Tensor:
    """torch.nn.utils.clip_grad_norm_ (torch's get_total_norm + _clip_grads_with_norm_, line for line) with each
    fp32 reduction replaced by the correctly rounded norm: per-tensor norms and the norm of those norms from fp64 sums
    of exact squares, rounded to fp32. The coefficient is torch's own expression, max_norm / (total + 1e-6), which
    Tensor.__rdiv__ evaluates as reciprocal(total + 1e-6) * max_norm, clamped to 1, then one _foreach_mul_."""
    grads = [p.grad for p in params if p.grad is not None]
    norms = [g.double().square().sum().sqrt().to(torch.float32) for g in grads]
    total = torch.stack(norms).double().square().sum().sqrt().to(torch.float32)
    clip_coef = max_norm / (total + 1e-6)
    torch._foreach_mul_(grads, torch.clamp(clip_coef, max=1.0))
    return total


@torch.no_grad()
def optimizer_step(adam: Optional[torch.optim.Optimizer], muon_params: Sequence[torch.Tensor],
                   muon_bufs: List[Optional[torch.Tensor]], all_params: Sequence[torch.Tensor], *, divisor,
                   max_norm: Optional[float], muon_kw: dict, exact_norm: bool = False) -> Optional[torch.Tensor]:
    """mote/train/train.py:944-947: grads /= divisor, clip_grad_norm_(all params), AdamW step, Muon step. Returns the
    pre-clip total norm. A workload without AdamW params passes adam=None; max_norm=None skips the clip. `exact_norm`
    takes every norm of the step correctly rounded: the clip's (clip_grad_norm_exact_) and, through muon_kw, the
    Newton-Schulz normalisation's."""
    grads = [p.grad for p in all_params if p.grad is not None]
    torch._foreach_div_(grads, divisor)
    if max_norm is None:
        total = None
    elif exact_norm:
        total = clip_grad_norm_exact_(all_params, max_norm)
    else:
        total = torch.nn.utils.clip_grad_norm_(all_params, max_norm)
    if adam is not None:
        adam.step()
    muon_update(muon_params, muon_bufs, **muon_kw)
    return total
