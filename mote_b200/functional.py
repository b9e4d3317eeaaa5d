"""Functional form of the optimizer step over plain tensors: the one place that packs tensors into the C ABI's
descriptor arrays. The optimizer classes (optim.py), the tests and bench.py all go through here.

    optimizer_step(muon=[MuonItem...], adamw=[AdamWItem...], ...)   # mote/train/train.py:944-947
    muon_step(...)                                                  # mote/train/muon.py:52-100
    adamw_step(...)                                                 # torch.optim.AdamW.step (train.py:98)
    moe_update_bias(moe_layers)                                     # mote/model/moe.py:147-159 (train.py:948-949)
    ema_lerp(emas, params, 1 - decay)                               # train.py:950-953
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from . import _lib as L
from .ops import grad_dtype_code, stream_handle, workspace


@dataclass
class MuonItem:
    """One Muon parameter for one step (mote/train/muon.py:60-79): `lr` is already the effective rate (param_lr
    override resolved) and `decay` the decoupled decay of muon.py:78 (0 for none). For a step whose lr is read on
    the device (`optimizer_step(lr_device=...)`, `CapturedStep(dynamic_lr=True)`), `wd` and `lr_max` give the decay
    rule instead: decay = lr * wd, or (lr * lr / lr_max) * wd with Muon-SW (lr_max > 0); `wd` None derives it from
    decay / lr."""
    param: torch.Tensor
    grad: torch.Tensor
    momentum_buffer: torch.Tensor
    lr: float
    decay: float = 0.0
    momentum: float = 0.95
    nesterov: bool = True
    wd: Optional[float] = None
    lr_max: float = 0.0


@dataclass
class AdamWItem:
    """One AdamW tensor for one step; `step` counts this update (1 on the first)."""
    param: torch.Tensor
    grad: torch.Tensor
    exp_avg: torch.Tensor
    exp_avg_sq: torch.Tensor
    lr: float
    weight_decay: float
    step: int


def _check_param(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{what} must be on a CUDA device: the optimizer runs only on the GPU")
    if t.dtype != torch.float32:
        raise TypeError(f"{what} must be fp32 (the master-parameter dtype), got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous")


def muon_array(items: Sequence[MuonItem]):
    arr = (L.MuonParam * max(1, len(items)))()
    for i, it in enumerate(items):
        p, g, b = it.param, it.grad, it.momentum_buffer
        _check_param(p, "Muon param")
        _check_param(b, "Muon momentum buffer")
        if g.shape != p.shape or b.shape != p.shape:
            raise ValueError(f"Muon param {i}: grad/momentum shape {tuple(g.shape)}/{tuple(b.shape)} != {tuple(p.shape)}")
        if not g.is_contiguous():
            raise ValueError(f"Muon param {i}: grad must be contiguous")
        if p.ndim not in (2, 3):
            raise AssertionError("Muon is for 2-D matrices (or 3-D stacks of them)")
        batch = p.shape[0] if p.ndim == 3 else 1
        e = arr[i]
        e.param, e.grad, e.momentum_buffer = p.data_ptr(), g.data_ptr(), b.data_ptr()
        e.batch, e.rows, e.cols = batch, p.shape[-2], p.shape[-1]
        e.lr, e.decay, e.momentum = float(it.lr), float(it.decay), float(it.momentum)
        e.nesterov, e.grad_dtype = int(bool(it.nesterov)), grad_dtype_code(g)
    return arr


def adamw_array(items: Sequence[AdamWItem]):
    arr = (L.AdamWTensor * max(1, len(items)))()
    for i, it in enumerate(items):
        for t, w in ((it.param, "param"), (it.exp_avg, "exp_avg"), (it.exp_avg_sq, "exp_avg_sq")):
            _check_param(t, f"AdamW {w}")
            if t.shape != it.param.shape:
                raise ValueError(f"AdamW tensor {i}: {w} shape mismatch")
        if it.grad.shape != it.param.shape or not it.grad.is_contiguous():
            raise ValueError(f"AdamW tensor {i}: grad must be contiguous with the param's shape")
        e = arr[i]
        e.param, e.grad, e.exp_avg, e.exp_avg_sq = (it.param.data_ptr(), it.grad.data_ptr(), it.exp_avg.data_ptr(),
                                                    it.exp_avg_sq.data_ptr())
        e.numel, e.lr, e.weight_decay, e.step = it.param.numel(), float(it.lr), float(it.weight_decay), int(it.step)
        e.grad_dtype = grad_dtype_code(it.grad)
    return arr


def _device_divisor(grad_divisor, dev: torch.device) -> Optional[torch.Tensor]:
    """A tensor divisor (the trainer's total_n, train.py:945) as the fp32 device scalar the kernels read: the tensor
    itself when it already is one (so a captured step reads its value at every replay), else an fp32 copy on the
    device, made on the current stream (no host round trip). A number gives None (passed by value)."""
    if not isinstance(grad_divisor, torch.Tensor):
        return None
    if grad_divisor.numel() != 1:
        raise ValueError("grad_divisor must be a number or a one-element tensor")
    if grad_divisor.device == dev and grad_divisor.dtype == torch.float32:
        return grad_divisor
    return grad_divisor.detach().to(device=dev, dtype=torch.float32)


def _device(muon: Sequence[MuonItem], adamw: Sequence[AdamWItem]) -> torch.device:
    for it in list(muon) + list(adamw):
        return it.param.device
    return torch.device("cuda", torch.cuda.current_device())


@torch.no_grad()
def optimizer_step(muon: Sequence[MuonItem] = (), adamw: Sequence[AdamWItem] = (), *, ns_steps: int = 5,
                   rms_scale: float = 0.2, ns_eps: float = 1e-7, betas=(0.9, 0.95), eps: float = 1e-8,
                   max_norm: Optional[float] = None, grad_divisor: Optional[float] = None,
                   out_norm: Optional[torch.Tensor] = None,
                   device_step: Optional[torch.Tensor] = None,
                   ema: Optional[Sequence[Optional[torch.Tensor]]] = None, ema_weight: float = 0.0,
                   muon_norms: Optional[torch.Tensor] = None,
                   lr_device: Optional[torch.Tensor] = None, ns_variant: int = 0) -> Optional[torch.Tensor]:
    """mote/train/train.py:944-947 in one call: grads /= grad_divisor; clip_grad_norm_(every grad, max_norm);
    AdamW; Muon. The grads are read, never written. Returns the pre-clip total norm (0-dim device tensor) when
    max_norm is given. With `device_step` (a 0-dim fp32 CUDA tensor) AdamW's step count is that counter, which the
    call increments on the device (the AdamItems' `step` is then ignored). `grad_divisor` is a number or a
    one-element tensor (the trainer's total_n): a tensor is read by the kernels on the device, with no host
    synchronisation.

    Fused extras (the work train.py:950-953 and elr.py:85-87 do in separate passes after the step):
    `ns_variant` 1 runs the opt-in Gram Newton-Schulz variant on the Muon matrices whose long side is at least twice
    the short one (not the reference's iteration; include/moteopt.h, moteopt_muon_config::ns_variant).

    `ema` - one fp32 buffer (or None) per AdamW item, then per Muon item, updated as
    torch._foreach_lerp_(ema, params, ema_weight) in the pass that writes the params; `muon_norms` - an fp32 CUDA
    tensor of len(muon) that receives ||p||_F of every Muon param after the update; `lr_device` - an fp64 CUDA tensor
    of len(adamw) + len(muon) lrs (AdamW items, then Muon items) read by the kernels at run time instead of the items'
    `lr` (a schedule under graph capture; see MuonItem for the decay rule)."""
    dev = _device(muon, adamw)
    m_arr, a_arr = muon_array(muon), adamw_array(adamw)
    cfg = L.MuonConfig(int(ns_steps), float(rms_scale), float(ns_eps), int(ns_variant))
    nbytes = L.lib.moteopt_optimizer_step_workspace_size_cfg(m_arr, len(muon), C.byref(cfg), a_arr, len(adamw))
    if nbytes == 0:
        raise L.MoteoptError("optimizer_step: invalid shapes or ns_variant")
    ws = workspace(dev, nbytes)
    hp = L.AdamWHparams(float(betas[0]), float(betas[1]), float(eps),
                        device_step.data_ptr() if device_step is not None else None)
    div_t = _device_divisor(grad_divisor, dev)
    gc = L.GradConfig(int(max_norm is not None), float(max_norm or 0.0),
                      0.0 if div_t is not None else float(grad_divisor or 0.0),
                      div_t.data_ptr() if div_t is not None else None)
    if max_norm is not None and out_norm is None:
        out_norm = torch.empty((), dtype=torch.float32, device=dev)
    onorm = C.c_void_p(out_norm.data_ptr() if out_norm is not None else 0)
    stream = C.c_void_p(stream_handle(dev))
    if ema is None and muon_norms is None and lr_device is None:
        L.check(L.lib.moteopt_optimizer_step(m_arr, len(muon), C.byref(cfg), a_arr, len(adamw), C.byref(hp),
                                             C.byref(gc), onorm, C.c_void_p(ws.data_ptr()), ws.numel(), stream),
                "moteopt_optimizer_step")
        return out_norm
    ex = L.StepExtras(None, float(ema_weight), None)
    if ema is not None:
        items = list(adamw) + list(muon)
        if len(ema) != len(items):
            raise ValueError(f"ema: {len(ema)} buffers for {len(items)} tensors (AdamW items, then Muon items)")
        for e, it in zip(ema, items):
            if e is not None:
                _check_param(e, "EMA buffer")
                if e.shape != it.param.shape:
                    raise ValueError("EMA buffer shape mismatch")
        ex.ema = L.array(C.c_void_p, [e.data_ptr() if e is not None else None for e in ema])
    if muon_norms is not None:
        if not (muon_norms.is_cuda and muon_norms.dtype == torch.float32 and muon_norms.numel() >= len(muon)):
            raise ValueError("muon_norms must be an fp32 CUDA tensor with one element per Muon item")
        ex.muon_norms = muon_norms.data_ptr()
    keep = []
    if lr_device is not None:
        if not (lr_device.is_cuda and lr_device.dtype == torch.float64 and lr_device.is_contiguous()
                and lr_device.numel() >= len(adamw) + len(muon)):
            raise ValueError("lr_device must be a contiguous fp64 CUDA tensor with one lr per AdamW and Muon item")
        ex.lr = lr_device.data_ptr()
        wds = [it.wd if it.wd is not None else (it.decay / it.lr if it.lr else 0.0) for it in muon]
        keep = [L.array(C.c_double, wds or [0.0]), L.array(C.c_double, [float(it.lr_max) for it in muon] or [0.0])]
        ex.muon_wd, ex.muon_lr_max = keep
    L.check(L.lib.moteopt_optimizer_step_ex(m_arr, len(muon), C.byref(cfg), a_arr, len(adamw), C.byref(hp),
                                            C.byref(gc), C.byref(ex), onorm, C.c_void_p(ws.data_ptr()), ws.numel(),
                                            stream), "moteopt_optimizer_step_ex")
    return out_norm


@torch.no_grad()
def muon_step(muon: Sequence[MuonItem], *, ns_steps: int = 5, rms_scale: float = 0.2, ns_eps: float = 1e-7,
              grad_scale: Optional[torch.Tensor] = None, ns_variant: int = 0) -> None:
    """mote/train/muon.py:52-100 for a list of parameters (any mix of groups and shapes). ns_variant 1 runs the
    opt-in Gram Newton-Schulz variant on matrices whose long side is at least twice the short one (include/moteopt.h,
    moteopt_muon_config::ns_variant); 0, the default, is the reference's iteration."""
    if not muon:
        return
    dev = _device(muon, ())
    arr = muon_array(muon)
    cfg = L.MuonConfig(int(ns_steps), float(rms_scale), float(ns_eps), int(ns_variant))
    nbytes = L.lib.moteopt_muon_step_workspace_size_cfg(arr, len(muon), C.byref(cfg))
    if nbytes == 0:
        raise L.MoteoptError("muon_step: invalid shapes or ns_variant")
    ws = workspace(dev, nbytes)
    L.check(L.lib.moteopt_muon_step(arr, len(muon), C.byref(cfg),
                                    C.c_void_p(grad_scale.data_ptr() if grad_scale is not None else 0),
                                    C.c_void_p(ws.data_ptr()), ws.numel(), C.c_void_p(stream_handle(dev))),
            "moteopt_muon_step")


@torch.no_grad()
def adamw_step(adamw: Sequence[AdamWItem], *, betas=(0.9, 0.999), eps: float = 1e-8,
               grad_scale: Optional[torch.Tensor] = None) -> None:
    """torch.optim.AdamW.step (single-tensor arithmetic, amsgrad=False) for a list of tensors."""
    if not adamw:
        return
    dev = _device((), adamw)
    arr = adamw_array(adamw)
    hp = L.AdamWHparams(float(betas[0]), float(betas[1]), float(eps), None)
    L.check(L.lib.moteopt_adamw_step(arr, len(adamw), C.byref(hp),
                                     C.c_void_p(grad_scale.data_ptr() if grad_scale is not None else 0),
                                     C.c_void_p(stream_handle(dev))), "moteopt_adamw_step")


def ema_lerp(emas: Sequence[torch.Tensor], params: Sequence[torch.Tensor], weight: float) -> None:
    """torch._foreach_lerp_(emas, params, weight) (the EMA update of mote/train/train.py:950-953, weight = 1 -
    ema_decay) in one library launch, bit for bit torch's lerp. For params that no fused pass writes; the optimizer
    step itself takes `ema=` for the params it updates."""
    if len(emas) != len(params):
        raise ValueError("ema_lerp: one EMA buffer per param")
    if not emas:
        return
    for e, p in zip(emas, params):
        if not (e.is_cuda and p.is_cuda and e.dtype == torch.float32 and p.dtype == torch.float32
                and e.is_contiguous() and p.is_contiguous() and e.numel() == p.numel() and e.device == p.device):
            raise TypeError("ema_lerp: EMA buffers and params must be contiguous fp32 CUDA tensors of equal size")
    dev = emas[0].device
    n = len(emas)
    L.check(L.lib.moteopt_ema_lerp(L.array(C.c_void_p, [e.data_ptr() for e in emas]),
                                   L.array(C.c_void_p, [p.data_ptr() for p in params]),
                                   L.array(C.c_int64, [p.numel() for p in params]), n, float(weight),
                                   C.c_void_p(stream_handle(dev))), "moteopt_ema_lerp")


def moe_update_bias(layers: Sequence) -> None:
    """MoESwiGLU.update_bias (mote/model/moe.py:147-159) of every given MoE layer in one launch, as the trainer calls
    it after the optimizer step (mote/train/train.py:948-949). `layers` holds MoE modules (anything with the
    reference module's `router_kind`, `bias_gamma`, `_load_acc` and `expert_bias`) or (load_acc, expert_bias, gamma)
    tuples. Layers whose router is not "lossfree" or whose gamma is <= 0 are skipped, as moe.py:151-152 does. No
    host synchronisation, so the call can sit inside a captured CUDA graph."""
    rows = []
    for m in layers:
        if isinstance(m, tuple):
            load, bias, gamma = m
        else:
            if getattr(m, "router_kind", None) != "lossfree" or float(m.bias_gamma) <= 0:
                continue
            load, bias, gamma = m._load_acc, m.expert_bias, float(m.bias_gamma)
        if float(gamma) <= 0:
            continue
        for t, what in ((load, "load_acc"), (bias, "expert_bias")):
            if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
                raise TypeError(f"moe_update_bias: {what} must be a contiguous fp32 CUDA tensor")
        if load.numel() != bias.numel() or load.device != bias.device:
            raise ValueError("moe_update_bias: load_acc and expert_bias must match in size and device")
        rows.append((load, bias, float(gamma)))
    if not rows:
        return
    dev = rows[0][0].device
    if any(r[0].device != dev for r in rows):
        raise ValueError("moe_update_bias: all layers must be on one device")
    arr = (L.MoeBias * len(rows))(*[L.MoeBias(ld.data_ptr(), b.data_ptr(), ld.numel(), g) for ld, b, g in rows])
    L.check(L.lib.moteopt_moe_update_bias(arr, len(rows), C.c_void_p(stream_handle(dev))), "moteopt_moe_update_bias")


class CapturedStep:
    """optimizer_step over a fixed set of tensors, captured once into a CUDA graph and then replayed, so a step
    costs one graph launch on the host instead of ~20 kernel launches and their argument packing.

    The tensors (params, grads, state) must stay the same objects at the same addresses; the hyperparameters (lr,
    decay, betas, clip, divisor) are the ones given here, fixed at capture (build a new CapturedStep to change
    them). AdamW's step count is a device counter starting at `start_step`. The first call runs the step eagerly
    (it also warms the library up), the second captures it and replays it, every later call replays. Returns the
    pre-clip grad norm tensor (overwritten by every call).

    The trainer's after-step work can ride in the same graph (train.py:948-953, elr.py:85-87): `ema` (one fp32 EMA
    buffer or None per AdamW item, then per Muon item) with `ema_weight` = 1 - ema_decay, `muon_norms` (fp32, one
    per Muon item, receives each param's norm) and `moe` (MoE layers, as moe_update_bias takes them)."""

    def __init__(self, muon: Sequence[MuonItem] = (), adamw: Sequence[AdamWItem] = (), *, ns_steps: int = 5,
                 rms_scale: float = 0.2, ns_eps: float = 1e-7, betas=(0.9, 0.95), eps: float = 1e-8,
                 max_norm: Optional[float] = None, grad_divisor: Optional[float] = None, start_step: int = 0,
                 dynamic_lr: bool = False, ema: Optional[Sequence[Optional[torch.Tensor]]] = None,
                 ema_weight: float = 0.0, muon_norms: Optional[torch.Tensor] = None, moe: Optional[Sequence] = None,
                 ns_variant: int = 0):
        self.dev = _device(muon, adamw)
        if isinstance(grad_divisor, torch.Tensor) and _device_divisor(grad_divisor, self.dev) is not grad_divisor:
            raise ValueError("CapturedStep: a tensor grad_divisor must be a one-element fp32 tensor on the step's "
                             "device (the graph reads it in place at every replay)")
        self.kw = dict(ns_steps=ns_steps, rms_scale=rms_scale, ns_eps=ns_eps, betas=betas, eps=eps,
                       max_norm=max_norm, grad_divisor=grad_divisor, ema=ema, ema_weight=ema_weight,
                       muon_norms=muon_norms, ns_variant=ns_variant)
        self.moe = list(moe) if moe else []
        self.muon, self.adamw = list(muon), list(adamw)
        self.device_step = torch.full((), float(start_step), dtype=torch.float32, device=self.dev)
        self.out_norm = torch.zeros((), dtype=torch.float32, device=self.dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.calls = 0
        self.launches_per_step = 0
        self.lr_device: Optional[torch.Tensor] = None
        if dynamic_lr:   # the kernels read every tensor's lr here at replay time (set_lrs)
            self.lr_device = torch.tensor([it.lr for it in self.adamw] + [it.lr for it in self.muon],
                                          dtype=torch.float64, device=self.dev)

    def set_lrs(self, adamw_lrs: Sequence[float], muon_lrs: Sequence[float]) -> None:
        """This step's lrs (dynamic_lr=True): one per AdamW item and one per Muon item, as set_lr / param_lr give them
        (train.py:177-179); the decay follows each item's rule. A synchronous host-to-device copy of a few bytes, so
        it is safe to call between replays."""
        if self.lr_device is None:
            raise RuntimeError("CapturedStep was built without dynamic_lr")
        vals = [float(x) for x in adamw_lrs] + [float(x) for x in muon_lrs]
        if len(vals) != self.lr_device.numel():
            raise ValueError(f"set_lrs: {len(vals)} lrs for {self.lr_device.numel()} tensors")
        self.lr_device.copy_(torch.tensor(vals, dtype=torch.float64))

    def _run(self):
        optimizer_step(self.muon, self.adamw, out_norm=self.out_norm, device_step=self.device_step,
                       lr_device=self.lr_device, **self.kw)
        if self.moe:
            moe_update_bias(self.moe)

    @torch.no_grad()
    def __call__(self) -> torch.Tensor:
        if self.graph is not None:
            self.graph.replay()
        elif self.calls == 0:
            self._run()
        else:
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            n0 = L.lib.moteopt_launch_count()
            with torch.cuda.graph(g):
                self._run()
            self.launches_per_step = int(L.lib.moteopt_launch_count() - n0)
            self.graph = g
            g.replay()
        self.calls += 1
        return self.out_norm


def items_from_lists(params: List[torch.Tensor], grads: List[torch.Tensor], bufs: List[torch.Tensor], lr: float,
                     decay: float, momentum: float = 0.95, nesterov: bool = True) -> List[MuonItem]:
    return [MuonItem(p, g, b, lr, decay, momentum, nesterov) for p, g, b in zip(params, grads, bufs)]
