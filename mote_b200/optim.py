"""Drop-in optimizer classes for the Mote trainer, running on the B200 kernels of libmoteopt.so.

Reference interfaces mirrored (noahsabaj/mote):
  Muon               -- mote/train/muon.py:46-100 (same constructor, param-group keys, `param_lr`, state layout)
  split_muon_params  -- mote/train/muon.py:103-126
  AdamW              -- torch.optim.AdamW as constructed at mote/train/train.py:98 (a subclass: same defaults and
                        state_dict keys; the update runs in the library instead of ATen)
  MultiOpt           -- mote/train/train.py:50-73
  build_optimizer    -- mote/train/train.py:76-105
  set_lr             -- mote/train/train.py:177-179
  fused_step         -- mote/train/train.py:944-947 (grads /= n; clip_grad_norm_; opt.step()) in one call

`Muon` subclasses the reference's `mote.train.muon.Muon` when that module is importable, so the reference's
`isinstance(o, Muon)` checks (elr.py:50-51, :283-284) keep recognising it. All parameters must be fp32 CUDA
tensors; there is no CPU fallback.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import functional as F
from .functional import AdamWItem, MuonItem

try:  # the reference trainer's own class, when it is on the path
    from mote.train.muon import Muon as _ReferenceMuon  # type: ignore
    _MuonBase = _ReferenceMuon
except Exception:  # noqa: BLE001
    _MuonBase = torch.optim.Optimizer


def _lr(v) -> float:
    return float(v.item()) if isinstance(v, torch.Tensor) else float(v)


# -----------------------------------------------------------------------------------------------------------------
class Muon(_MuonBase):
    """Nesterov momentum + batched Newton-Schulz orthogonalisation + RMS-matched scale + decoupled (or Muon-SW)
    weight decay, with per-parameter `param_lr` overrides (mote/train/muon.py:46-100). Every matrix of every group
    is orthogonalised in one batched tcgen05 launch sequence; the decay and the scaled update are then applied in
    one memory-bound pass over every parameter (muon.py:93-99). State: `momentum_buffer` (fp32, the parameter's
    shape) per parameter.

    `gram_ns=True` (keyword only, not in the reference's signature and not a param-group key, so checkpoints keep
    the reference's layout) opts into the Gram Newton-Schulz variant of the reference's research notes
    (docs/research/efficiency-campaign-2026-08-23.md:903-911) on matrices whose long side is at least twice the
    short one: fewer FLOPs, not the reference's iteration."""

    def __init__(self, params, lr: float = 1e-3, momentum: float = 0.95, nesterov: bool = True,
                 weight_decay: float = 0.0, ns_steps: int = 5, rms_scale: float = 0.2, sw_decay: bool = False,
                 lr_max: float = 1.0, *, gram_ns: bool = False):
        defaults = dict(lr=lr, momentum=momentum, nesterov=nesterov, weight_decay=weight_decay, ns_steps=ns_steps,
                        rms_scale=rms_scale, sw_decay=sw_decay, lr_max=lr_max)
        torch.optim.Optimizer.__init__(self, params, defaults)
        self.ns_variant = 1 if gram_ns else 0

    def _items(self) -> Dict[Tuple[int, float], List[MuonItem]]:
        """Per (ns_steps, rms_scale): the step's MuonItems (muon.py:55-79)."""
        out: Dict[Tuple[int, float], List[MuonItem]] = defaultdict(list)
        for group in self.param_groups:
            lr, mom, wd = _lr(group["lr"]), group["momentum"], group["weight_decay"]
            param_lr = group.get("param_lr")
            for p in group["params"]:
                if p.grad is None:
                    continue
                assert p.ndim in (2, 3), "Muon is for 2-D matrices (or 3-D stacks of them)"
                g = p.grad
                if g.dtype not in (torch.float32, torch.bfloat16):
                    g = g.float()
                if not g.is_contiguous():
                    g = g.contiguous()
                state = self.state[p]
                if "momentum_buffer" not in state:
                    state["momentum_buffer"] = torch.zeros_like(p, dtype=torch.float32)
                e = lr if param_lr is None else _lr(param_lr.get(id(p), lr))
                d = (e * e / group["lr_max"] if group["sw_decay"] else e) * wd if wd else 0.0
                out[(int(group["ns_steps"]), float(group["rms_scale"]))].append(
                    MuonItem(p.data, g, state["momentum_buffer"], e, d, mom, bool(group["nesterov"])))
        return out

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for (ns, rms), items in self._items().items():
            F.muon_step(items, ns_steps=ns, rms_scale=rms, ns_variant=getattr(self, "ns_variant", 0))
        return loss


# -----------------------------------------------------------------------------------------------------------------
class AdamW(torch.optim.AdamW):
    """torch.optim.AdamW with its update run by libmoteopt (one multi-tensor kernel for every group): the same
    constructor, defaults, param-group keys and state ({step: fp32 0-dim tensor, exp_avg, exp_avg_sq}). `step` is
    kept on the CPU, as torch keeps it for a non-capturable optimizer. amsgrad, maximize and differentiable are not
    supported (the reference does not use them)."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, amsgrad=False, *,
                 maximize=False, foreach=None, capturable=False, differentiable=False, fused=None):
        if amsgrad or maximize or differentiable or capturable:
            raise NotImplementedError("moteopt AdamW: amsgrad, maximize, capturable and differentiable are not supported")
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=False,
                         maximize=False, foreach=foreach, capturable=False, differentiable=False, fused=fused)
        self._step_cache: Dict[int, Tuple[torch.Tensor, int]] = {}

    def _step_count(self, p, st) -> int:
        t = st["step"]
        hit = self._step_cache.get(id(p))
        if hit is not None and hit[0] is t:
            return hit[1]
        v = int(t.item())
        self._step_cache[id(p)] = (t, v)
        return v

    def _items(self) -> Tuple[List[AdamWItem], Tuple[float, float], float, List[Tuple[torch.Tensor, torch.Tensor]]]:
        items: List[AdamWItem] = []
        betas = eps = None
        bumped = []
        for group in self.param_groups:
            b, e = tuple(float(x) for x in group["betas"]), float(group["eps"])
            if betas is None:
                betas, eps = b, e
            elif (b, e) != (betas, eps):
                raise NotImplementedError("moteopt AdamW: every param group must share betas and eps")
            lr, wd = _lr(group["lr"]), float(group["weight_decay"])
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("AdamW does not support sparse gradients")
                g = p.grad
                if g.dtype not in (torch.float32, torch.bfloat16):
                    g = g.float()
                if not g.is_contiguous():
                    g = g.contiguous()
                st = self.state[p]
                if len(st) == 0:
                    st["step"] = torch.tensor(0.0, dtype=torch.float32)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                n = self._step_count(p, st) + 1
                items.append(AdamWItem(p.data, g, st["exp_avg"], st["exp_avg_sq"], lr, wd, n))
                bumped.append((p, st["step"]))
        return items, betas or (0.9, 0.999), eps or 1e-8, bumped

    def _bump(self, bumped) -> None:
        steps = [t for _, t in bumped]
        if steps:
            torch._foreach_add_(steps, 1.0)
        for p, t in bumped:
            hit = self._step_cache.get(id(p))
            if hit is not None and hit[0] is t:
                self._step_cache[id(p)] = (t, hit[1] + 1)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        items, betas, eps, bumped = self._items()
        F.adamw_step(items, betas=betas, eps=eps)
        self._bump(bumped)
        return loss


# -----------------------------------------------------------------------------------------------------------------
class MultiOpt:
    """Several optimizers driven as one (Muon for hidden matrices + AdamW for the rest); mote/train/train.py:50-73."""

    def __init__(self, opts):
        self.opts = opts

    @property
    def param_groups(self):
        return [g for o in self.opts for g in o.param_groups]

    def zero_grad(self, set_to_none=True):
        for o in self.opts:
            o.zero_grad(set_to_none=set_to_none)

    def step(self):
        """train.py:64-66 (AdamW.step(), then Muon.step()). When every optimizer is this module's AdamW or Muon and
        their groups can share one launch sequence (one ns_steps / rms_scale over the Muon groups, one betas / eps
        over the AdamW groups), both run as ONE library call (fused_step without a clip or divisor), which gives
        the same bits as the two separate steps; otherwise each optimizer steps in turn."""
        if _fusable(self.opts):
            fused_step(self)
            return
        for o in self.opts:
            o.step()

    def state_dict(self):
        return {"multi": [o.state_dict() for o in self.opts]}

    def load_state_dict(self, sd):
        for o, s in zip(self.opts, sd["multi"]):
            o.load_state_dict(s)


def _fusable(opts) -> bool:
    """Whether fused_step can run these optimizers as one library call."""
    muon_keys, adam_keys = set(), set()
    for o in opts:
        if isinstance(o, Muon):
            muon_keys.update((int(g["ns_steps"]), float(g["rms_scale"]), getattr(o, "ns_variant", 0))
                             for g in o.param_groups)
        elif isinstance(o, AdamW):
            adam_keys.update((tuple(float(b) for b in g["betas"]), float(g["eps"])) for g in o.param_groups)
        else:
            return False
    return len(muon_keys) <= 1 and len(adam_keys) <= 1


def set_lr(opt, lr: float):
    """mote/train/train.py:177-179."""
    for g in opt.param_groups:
        g["lr"] = lr * g["lr_mult"]


# -----------------------------------------------------------------------------------------------------------------
@torch.no_grad()
def fused_step(opt, max_norm: Optional[float] = None, grad_divisor=None, ema: Optional[dict] = None,
               ema_decay: float = 0.0, moe: Optional[Sequence] = None) -> Optional[torch.Tensor]:
    """mote/train/train.py:944-947 in one library call:

        torch._foreach_div_(grads, total_n); gnorm = clip_grad_norm_(model.parameters(), clip); opt.step()

    `opt` is a MultiOpt of this module's AdamW and Muon (or one of them). The division and the clip are folded into
    the update kernels: the grads are read once for the norm and once for the update and never rewritten. Returns
    the pre-clip total grad norm (0-dim fp32 CUDA tensor) when max_norm is given. Only the parameters the optimizers
    own enter the norm; the reference passes model.parameters(), which is the same set when every trainable
    parameter is in the optimizer (train.py:82-83 skips requires_grad=False ones, which have no grad).

    `ema` ({param: fp32 EMA buffer}) with `ema_decay` folds train.py:950-953 (_foreach_lerp_(ema, params,
    1 - ema_decay)) into the same step for the stepped params; the caller lerps any other params itself.

    `moe` (the trainer's MoE layers) runs their routers' bias step after the optimizer step, as train.py:948-949
    (`for m in self._moe: m.update_bias()`), in one launch (functional.moe_update_bias)."""
    opts = getattr(opt, "opts", [opt])
    variants = {getattr(o, "ns_variant", 0) for o in opts if isinstance(o, Muon)}
    if len(variants) > 1:
        raise NotImplementedError("fused_step: every Muon optimizer must use the same Newton-Schulz variant")
    ns_variant = variants.pop() if variants else 0
    muon_sets: Dict[Tuple[int, float], List[MuonItem]] = {}
    adam_items: List[AdamWItem] = []
    betas, eps = (0.9, 0.999), 1e-8
    bumps = []
    for o in opts:
        if isinstance(o, Muon):
            for k, v in o._items().items():
                muon_sets.setdefault(k, []).extend(v)
        elif isinstance(o, AdamW):
            items, betas, eps, bumped = o._items()
            adam_items.extend(items)
            bumps.append((o, bumped))
        else:
            raise TypeError(f"fused_step handles mote_b200 Muon and AdamW, got {type(o).__name__}")
    if len(muon_sets) > 1:
        raise NotImplementedError("fused_step: all Muon groups must share ns_steps and rms_scale")
    (ns, rms), muon_items = next(iter(muon_sets.items())) if muon_sets else ((5, 0.2), [])
    div = None   # a tensor (the trainer's total_n) stays on the device: the kernels read it there, no host sync
    if grad_divisor is not None:
        div = grad_divisor if isinstance(grad_divisor, torch.Tensor) else float(grad_divisor)
    bufs = None
    if ema is not None:
        bufs = [ema.get(it.param) for it in adam_items] + [ema.get(it.param) for it in muon_items]
    norm = F.optimizer_step(muon_items, adam_items, ns_steps=ns, rms_scale=rms, betas=betas, eps=eps,
                            max_norm=max_norm, grad_divisor=div, ema=bufs, ema_weight=1.0 - float(ema_decay),
                            ns_variant=ns_variant)
    for o, bumped in bumps:
        o._bump(bumped)
    if moe:
        F.moe_update_bias(moe)
    return norm


# -----------------------------------------------------------------------------------------------------------------
def split_muon_params(model) -> Tuple[list, list]:
    """(muon_params, other_params), mote/train/muon.py:103-126: hidden 2-D matrices and `_muon_stack` 3-D expert
    stacks go to Muon; embeddings / tied head, every other shape, Mamba-3's `in_proj` and `_no_muon` params go to
    AdamW."""
    skip = set()
    for name in ("embeddings", "lm_head"):
        mod = getattr(model, name, None)
        if mod is not None and getattr(mod, "weight", None) is not None:
            skip.add(id(mod.weight))
    for m in model.modules():
        if type(m).__name__ == "Mamba3Mixer" and getattr(m, "in_proj", None) is not None:
            skip.add(id(m.in_proj.weight))
    muon, other = [], []
    seen = set()
    for p in model.parameters():
        if id(p) in seen:
            continue
        seen.add(id(p))
        stack = p.ndim == 3 and getattr(p, "_muon_stack", False)
        if (p.ndim == 2 or stack) and id(p) not in skip and not getattr(p, "_no_muon", False):
            muon.append(p)
        else:
            other.append(p)
    return muon, other


def build_optimizer(model, lr: float, weight_decay: float, stage_lr_mult, betas=(0.9, 0.95), optimizer: str = "adamw"):
    """mote/train/train.py:76-105 with this module's AdamW and Muon."""
    groups = model.stage_param_groups()
    muon_ids = {id(p) for p in split_muon_params(model)[0]} if optimizer in ("muon", "muonsw") else set()
    adam_groups, muon_groups = [], []
    for stage, params in groups.items():
        decay, no_decay, muon = [], [], []
        for p in params:
            if not p.requires_grad:
                continue
            if id(p) in muon_ids:
                muon.append(p)
            elif p.ndim < 2 or getattr(p, "_no_weight_decay", False):
                no_decay.append(p)
            else:
                decay.append(p)
        mult = stage_lr_mult[stage]
        if decay:
            adam_groups.append({"params": decay, "weight_decay": weight_decay, "lr_mult": mult, "stage": stage})
        if no_decay:
            adam_groups.append({"params": no_decay, "weight_decay": 0.0, "lr_mult": mult, "stage": stage})
        if muon:
            muon_groups.append({"params": muon, "weight_decay": weight_decay, "lr_mult": mult, "stage": stage})
    adam = AdamW(adam_groups, lr=lr, betas=betas, eps=1e-8, fused=torch.cuda.is_available())
    if not muon_groups:
        return adam
    for g in muon_groups:
        g["lr_max"] = lr * g["lr_mult"]
    return MultiOpt([adam, Muon(muon_groups, lr=lr, momentum=0.95, nesterov=True, weight_decay=weight_decay,
                                sw_decay=(optimizer == "muonsw"))])
