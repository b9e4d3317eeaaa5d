"""The optimizer step across the GPUs of one node (the reference has no multi-GPU code; this is the build's own).

Layout. Two flat buffers per tensor kind (params, grads): a Muon region and an AdamW region.
  * Muon region: rank r's segment holds the Muon parameters it owns, whole, in declaration order, padded to the
    longest segment. Ownership is greedy longest-processing-time over each matrix's estimated cost (Newton-Schulz
    FLOPs at the tensor rate plus optimizer bytes at HBM rate), so ranks finish together.
  * AdamW region: every AdamW parameter concatenated in declaration order; rank r owns the r-th of N equal slices
    (ZeRO-1: exp_avg / exp_avg_sq exist only for the owned slice).
Every parameter is a contiguous view of its region, so a model's parameters can live there.

Step (grads: each rank's local, unreduced grads in the grad regions):
  1. reduce-scatter (sum) of both grad regions: rank r receives the reduced grads of its own segments;
  2. rank r's sum of (g / divisor)^2 per grad tensor over what it owns, all-gathered; per tensor the ranks' sums
     added in rank order -> the per-tensor norms -> their norm (torch's get_total_norm, as the single-GPU step forms
     it) and the clip coefficient, bitwise identical on every rank;
  3. rank r runs AdamW on its slice and, for its matrices, Muon's momentum and Newton-Schulz, writing the
     orthogonalised updates O (bf16) into its segment of an update region laid out like the Muon param region;
  4. all-gather of the update region (bf16) and of the AdamW param region (fp32);
  5. every rank applies every O to its copy of the Muon params (the same arithmetic on identical inputs, so all
     ranks hold the same bits). The bf16 O is exactly what the reference applies (muon.py:99 casts it to fp32), and
     gathering it moves half the bytes of gathering the fp32 params.
With peer updates enabled (`enable_peer_updates`, NCCL only), steps 4-5 for the Muon region become one pass: every
rank maps the other ranks' update regions (CUDA IPC, once), a one-element all-reduce orders the owners' writes
before the reads, and the apply kernel reads each owner's O straight over NVLink while it updates the local params,
so no gathered copy of O is ever written. Mappings of the grad regions (by default on 2 ranks, where this measured
faster than NCCL's reduce-scatter) turn steps 1-2 into one pass: after a
one-element all-reduce (every rank's grads complete), each rank reads its segments from every rank's grads over
NVLink, sums them in rank order, stores the reduced grads and forms the per-tensor sums of squares in the same pass
(moteopt_peer_reduce_sumsq); the later all-reduce before the O reads orders every rank's grad reads before any rank
can overwrite its grads.
Collectives go through torch.distributed (NCCL on GPUs; gloo works for the host-side tests). The compute steps are
injected (`Compute`), so the same choreography runs with the CUDA library or with a CPU stand-in.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

ALIGN = 64   # elements: every segment and every parameter starts 256-byte aligned in fp32


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


def muon_cost(shape: Sequence[int], ns_steps: int = 5, tflops: float = 1000.0, hbm_gbs: float = 6000.0) -> float:
    """Estimated seconds of one Muon parameter's update on one B200: Newton-Schulz FLOPs + 28 B/element."""
    batch = 1
    for d in shape[:-2]:
        batch *= int(d)
    m, n = sorted((int(shape[-2]), int(shape[-1])))
    flops = batch * ns_steps * (4.0 * m * m * n + 2.0 * m ** 3)
    return flops / (tflops * 1e12) + batch * m * n * 28.0 / (hbm_gbs * 1e9)


@dataclass
class ShardPlan:
    world: int
    muon_shapes: List[Tuple[int, ...]]
    adam_shapes: List[Tuple[int, ...]]
    owner: List[int] = field(default_factory=list)             # rank owning each Muon param
    muon_off: List[int] = field(default_factory=list)          # element offset of each Muon param in its region
    m_seg: int = 0                                              # Muon segment length per rank (elements)
    m_used: List[int] = field(default_factory=list)            # elements of rank r's segment that hold params
    adam_off: List[int] = field(default_factory=list)          # element offset of each AdamW param
    a_total: int = 0
    a_seg: int = 0

    @property
    def muon_len(self) -> int:
        return self.world * self.m_seg

    @property
    def adam_len(self) -> int:
        return self.world * self.a_seg

    def owned_muon(self, rank: int) -> List[int]:
        return [i for i, o in enumerate(self.owner) if o == rank]

    def adam_pieces(self, rank: int) -> List[Tuple[int, int, int]]:
        """(param index, first element inside the param, length) of the AdamW elements rank owns."""
        lo, hi = rank * self.a_seg, min((rank + 1) * self.a_seg, self.a_total)
        out = []
        for i, s in enumerate(self.adam_shapes):
            n = _numel(s)
            a, b = max(lo, self.adam_off[i]), min(hi, self.adam_off[i] + n)
            if a < b:
                out.append((i, a - self.adam_off[i], b - a))
        return out


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def make_plan(muon_shapes, adam_shapes, world: int, ns_steps: int = 5) -> ShardPlan:
    plan = ShardPlan(world, [tuple(s) for s in muon_shapes], [tuple(s) for s in adam_shapes])
    load = [0.0] * world
    plan.owner = [-1] * len(muon_shapes)
    order = sorted(range(len(muon_shapes)), key=lambda i: (-muon_cost(muon_shapes[i], ns_steps), i))
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        plan.owner[i] = r
        load[r] += muon_cost(muon_shapes[i], ns_steps)
    used = [0] * world
    plan.muon_off = [0] * len(muon_shapes)
    for i, s in enumerate(muon_shapes):        # declaration order inside each segment
        r = plan.owner[i]
        plan.muon_off[i] = used[r]             # relative to the segment; made absolute below
        used[r] += _round_up(_numel(s), ALIGN)
    plan.m_seg = _round_up(max(used) if used else 0, ALIGN)
    plan.m_used = used
    for i in range(len(muon_shapes)):
        plan.muon_off[i] += plan.owner[i] * plan.m_seg
    off = 0
    for s in adam_shapes:
        plan.adam_off.append(off)
        off += _numel(s)
    plan.a_total = off
    plan.a_seg = _round_up(-(-off // world), ALIGN) if off else 0
    return plan


# -----------------------------------------------------------------------------------------------------------------
@dataclass
class Compute:
    """The step's compute, injected: `sumsq(views, tensors, n_tensors, divisor) -> fp64 tensor [n_tensors]` (per grad
    tensor index, the sum of (g/divisor)^2 over the views that belong to it; 0 for the others), `coef(sums, n_tensors,
    max_norm) -> 2-element fp32 tensor [norm, coef]` from every rank's sums ([world * n_tensors], rank-major: per
    tensor the ranks' sums added in rank order, the fp32 norm of each tensor, then the norm of those norms),
    `update(muon_items, adam_items, coef,
    divisor, muon_out)` with items as in mote_b200.functional (AdamW applied; Muon's update O written to the bf16
    tensors `muon_out`, one per Muon item), and `apply(muon_items, updates, ema=None, ema_weight=0.0, norms=None)`:
    p = p*(1-decay); p += -lr*(O*scale) for every item (grad and momentum buffer unused), then, when given,
    ema[k] = lerp(ema[k], p, ema_weight) and norms[k] = ||p||_F in the same pass. `ema(emas, params, weight)` lerps
    tensors that no pass writes (the all-gathered AdamW region). `peer_reduce(pieces, world, n_tensors, divisor) ->
    fp64 [n_tensors]`, when given, reduces the grads straight from every rank's memory: each piece is (reduced view,
    the piece's address in every rank's grad region, tensor index); it stores the reduced grads and returns `sumsq`'s
    result for them."""
    sumsq: Callable
    coef: Callable
    update: Callable
    apply: Callable
    set_step: Optional[Callable] = None   # set_step(device, n): AdamW's step count, when the compute keeps one
    ema: Optional[Callable] = None
    peer_reduce: Optional[Callable] = None


def _reduce_scatter(out: torch.Tensor, flat: torch.Tensor, seg: int, rank: int, group=None) -> None:
    """out (seg elements) = this rank's segment of the sum of every rank's `flat`; `flat` is left as it was."""
    if seg == 0:
        return
    if dist.get_backend(group) == "nccl":
        dist.reduce_scatter_tensor(out, flat, op=dist.ReduceOp.SUM, group=group)
    else:   # gloo has no reduce-scatter of a flat tensor: an all-reduce of a copy gives the same sums
        tmp = flat.clone()
        dist.all_reduce(tmp, op=dist.ReduceOp.SUM, group=group)
        out.copy_(tmp[rank * seg:(rank + 1) * seg])


def _all_gather_inplace(flat: torch.Tensor, seg: int, rank: int, group=None) -> None:
    if seg == 0:
        return
    dist.all_gather_into_tensor(flat, flat[rank * seg:(rank + 1) * seg].clone() if dist.get_backend(group) != "nccl"
                                else flat[rank * seg:(rank + 1) * seg], group=group)


class PeerPieces(list):
    """The grad pieces a rank reduces from every rank's memory: (reduced view, the piece's address in every rank's
    grad region, grad tensor index); `packed` caches the compute's own encoding of the list."""
    packed = None


class ShardedStep:
    """Rank-local state and the step of the module docstring. `params_m`/`params_a` are the fp32 param regions,
    `grads_m`/`grads_a` the local grad regions (fp32 or bf16), of length plan.muon_len / plan.adam_len. The grad
    regions are only read: the reduced grads of the rank's own segments land in rank-local buffers."""

    def __init__(self, plan: ShardPlan, rank: int, params_m: torch.Tensor, params_a: torch.Tensor,
                 grads_m: torch.Tensor, grads_a: torch.Tensor, compute: Compute, *, muon_lr: float,
                 muon_wd: float, momentum: float = 0.95, nesterov: bool = True, adam_lr: float, adam_wd: Sequence[float],
                 group=None):
        self.plan, self.rank, self.group = plan, rank, group
        self.pm, self.pa, self.gm, self.ga = params_m, params_a, grads_m, grads_a
        self.compute = compute
        self.muon_lr, self.muon_wd, self.momentum, self.nesterov = muon_lr, muon_wd, momentum, nesterov
        self.adam_lr, self.adam_wd = adam_lr, list(adam_wd)
        self.mine = plan.owned_muon(rank)
        self.bufs = {i: torch.zeros(plan.muon_shapes[i], dtype=torch.float32, device=params_m.device) for i in self.mine}
        self.pieces = plan.adam_pieces(rank)
        self.gm_seg = torch.zeros(plan.m_seg, dtype=grads_m.dtype, device=grads_m.device)
        self.om = torch.zeros(plan.muon_len, dtype=torch.bfloat16, device=params_m.device)   # Muon updates O
        self.ga_seg = torch.zeros(plan.a_seg, dtype=grads_a.dtype, device=grads_a.device)
        self.m_state = torch.zeros(plan.a_seg, dtype=torch.float32, device=params_a.device)
        self.v_state = torch.zeros(plan.a_seg, dtype=torch.float32, device=params_a.device)
        self.steps = 0
        self.graph = None
        self.peer_ptrs: Optional[List[int]] = None   # update region of every rank, mapped into this process
        self._peer_bases: List[int] = []
        self._flag = None
        self._peer_pieces: Optional[list] = None     # the grad pieces this rank reduces from every rank's memory
        self._gflag = None
        self.n_tensors = len(plan.adam_shapes) + len(plan.muon_shapes)   # AdamW grads first, as the 1-GPU clip
        self.ema_decay: Optional[float] = None
        self.em: Optional[torch.Tensor] = None   # EMA of the Muon and AdamW param regions (every rank, replicated)
        self.ea: Optional[torch.Tensor] = None

    def enable_ema(self, decay: float, zero_init: bool = True) -> None:
        """Keep the weights' EMA of train.py:950-953 (ema = lerp(ema, p, 1 - decay) after every step). It starts at
        zero, as train.py:716-721 keeps it (a reader divides by 1 - decay^steps, hnet.ema_scale), or from the params
        as they are now with `zero_init=False` (the average of checkpoints written before that change); a resumed
        average is copied into `step.em` / `step.ea` after this call. Every rank holds the whole EMA: the Muon
        region's is lerped in the apply pass that writes the params, the AdamW region's in one pass after its
        all-gather, so each is a pure function of the replicated params and stays identical across ranks. The EMA of
        param i is `muon_view(step.em, i)` / `adam_view(step.ea, i)`."""
        if self.compute.ema is None:
            raise ValueError("enable_ema: the step's Compute has no `ema` pass")
        self.ema_decay = float(decay)
        self.em = torch.zeros_like(self.pm) if zero_init else self.pm.detach().clone()
        self.ea = torch.zeros_like(self.pa) if zero_init else self.pa.detach().clone()

    def enable_peer_updates(self, peer_grads: Optional[bool] = None) -> None:
        """Map every rank's update region into this process (CUDA IPC through libmoteopt); collective, eager, once.
        With `peer_grads` (and a Compute that has `peer_reduce`) the grad regions are mapped too, and the step reduces
        the grads by reading them from every rank's memory instead of an NCCL reduce-scatter. By default it does so on
        2 ranks only: on B200s with c1's 187 MB of bf16 grads the peer reduction (all-reduce barrier included) took
        0.17 ms against NCCL's 0.25 ms at 2 ranks, tied at 4 (0.28 ms) and lost at 8 (0.36 against 0.29 ms, where
        NCCL reduces inside the NVSwitch)."""
        if peer_grads is None:
            peer_grads = self.plan.world == 2
        import ctypes as C

        from . import _lib as L
        opened = {}   # (rank, handle) -> base: tensors of one allocation share one mapping

        def mapped(t: torch.Tensor) -> List[int]:
            handle = (C.c_ubyte * 64)()
            off = C.c_uint64(0)
            L.check(L.lib.moteopt_ipc_export(C.c_void_p(t.data_ptr()), handle, C.byref(off)), "moteopt_ipc_export")
            allh: List[Tuple[bytes, int]] = [None] * self.plan.world   # type: ignore[list-item]
            dist.all_gather_object(allh, (bytes(handle), int(off.value)), group=self.group)
            ptrs = []
            for r, (h, o) in enumerate(allh):
                if r == self.rank:
                    ptrs.append(t.data_ptr())
                    continue
                if (r, h) not in opened:
                    base = C.c_void_p(0)
                    L.check(L.lib.moteopt_ipc_import(bytes(h), C.byref(base)), "moteopt_ipc_import")
                    opened[(r, h)] = int(base.value)
                    self._peer_bases.append(int(base.value))
                ptrs.append(opened[(r, h)] + o)
            return ptrs
        self.peer_ptrs = mapped(self.om)
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.om.device)
        if peer_grads and self.compute.peer_reduce is not None:
            gm = mapped(self.gm) if self.plan.muon_len else []
            ga = mapped(self.ga) if self.plan.adam_len else []
            pieces = []
            na = len(self.plan.adam_shapes)
            for i in self.mine:
                nb = self.gm.element_size() * self.plan.muon_off[i]
                pieces.append((self.reduced_muon_grad(i).reshape(-1), [b + nb for b in gm], na + i))
            for i, start, n in self.pieces:
                nb = self.ga.element_size() * (self.plan.adam_off[i] + start)
                pieces.append((self.reduced_adam_grad(i, start, n), [b + nb for b in ga], i))
            self._peer_pieces = PeerPieces(pieces)
            self._gflag = torch.zeros(1, dtype=torch.float32, device=self.om.device)
        torch.cuda.synchronize(self.om.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the peers' update regions (collective: no rank frees its region while another still maps it)."""
        import ctypes as C

        from . import _lib as L
        if self.peer_ptrs is None:
            return
        torch.cuda.synchronize(self.om.device)
        for b in self._peer_bases:
            L.check(L.lib.moteopt_ipc_close(C.c_void_p(b)), "moteopt_ipc_close")
        self._peer_bases, self.peer_ptrs, self._peer_pieces = [], None, None
        dist.barrier(group=self.group)

    @torch.no_grad()
    def state_dict(self) -> dict:
        """The optimizer state in the trainer's checkpoint layout, {"multi": [adamw_sd, muon_sd]} (train.py:68-73;
        each in torch.optim's state_dict form, AdamW state {step, exp_avg, exp_avg_sq}, Muon {momentum_buffer},
        params numbered in plan order). Assembled on the devices with collectives: the ZeRO-1 slices of exp_avg /
        exp_avg_sq are all-gathered, the momentum buffers go from their owners through an all-gather of an fp32
        copy of the Muon region. Collective; every rank gets the whole dict, its tensors views of device buffers."""
        plan, r = self.plan, self.rank
        dev = self.pa.device
        m_full = torch.zeros(plan.adam_len, dtype=torch.float32, device=dev)
        v_full = torch.zeros(plan.adam_len, dtype=torch.float32, device=dev)
        m_full[r * plan.a_seg:(r + 1) * plan.a_seg].copy_(self.m_state)
        v_full[r * plan.a_seg:(r + 1) * plan.a_seg].copy_(self.v_state)
        _all_gather_inplace(m_full, plan.a_seg, r, self.group)
        _all_gather_inplace(v_full, plan.a_seg, r, self.group)
        mb = torch.zeros(plan.muon_len, dtype=torch.float32, device=self.pm.device)
        for i in self.mine:
            self.muon_view(mb, i).copy_(self.bufs[i])
        _all_gather_inplace(mb, plan.m_seg, r, self.group)
        groups, order = {}, []
        for i, wd in enumerate(self.adam_wd):
            if wd not in groups:
                groups[wd] = []
                order.append(wd)
            groups[wd].append(i)
        adam_groups, idx, adam_state = [], 0, {}
        for wd in order:   # torch numbers a state_dict's params in group order
            ids = []
            for i in groups[wd]:
                adam_state[idx] = {"step": torch.tensor(float(self.steps)), "exp_avg": self.adam_view(m_full, i),
                                   "exp_avg_sq": self.adam_view(v_full, i)}
                ids.append(idx)
                idx += 1
            adam_groups.append({"lr": self.adam_lr, "weight_decay": wd, "params": ids, "plan_index": groups[wd]})
        muon_state = {i: {"momentum_buffer": self.muon_view(mb, i)} for i in range(len(plan.muon_shapes))}
        muon_groups = [{"lr": self.muon_lr, "momentum": self.momentum, "nesterov": self.nesterov,
                        "weight_decay": self.muon_wd, "params": list(range(len(plan.muon_shapes)))}]
        return {"multi": [{"state": adam_state, "param_groups": adam_groups},
                          {"state": muon_state, "param_groups": muon_groups}]}

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        """Resume from state_dict()'s layout (on any device or the CPU): each rank takes its ZeRO-1 slices and the
        momentum buffers of the matrices it owns. Local, no collectives."""
        adam_sd, muon_sd = sd["multi"]
        plan = self.plan
        by_plan = {}
        for g in adam_sd["param_groups"]:
            for k, i in zip(g["params"], g.get("plan_index", g["params"])):
                by_plan[i] = adam_sd["state"][k]
        base = self.rank * plan.a_seg
        steps = None
        for i, start, n in self.pieces:
            st = by_plan[i]
            o = plan.adam_off[i] + start - base
            self.m_state[o:o + n].copy_(st["exp_avg"].reshape(-1)[start:start + n])
            self.v_state[o:o + n].copy_(st["exp_avg_sq"].reshape(-1)[start:start + n])
            steps = int(float(st["step"]))
        if steps is None and by_plan:
            steps = int(float(next(iter(by_plan.values()))["step"]))
        self.steps = steps or 0
        for i in self.mine:
            self.bufs[i].copy_(muon_sd["state"][i]["momentum_buffer"].reshape(self.bufs[i].shape))
        if self.compute.set_step is not None:
            self.compute.set_step(self.pa.device, self.steps)

    def muon_view(self, flat: torch.Tensor, i: int) -> torch.Tensor:
        o, s = self.plan.muon_off[i], self.plan.muon_shapes[i]
        return flat[o:o + _numel(s)].view(s)

    def adam_view(self, flat: torch.Tensor, i: int) -> torch.Tensor:
        o, s = self.plan.adam_off[i], self.plan.adam_shapes[i]
        return flat[o:o + _numel(s)].view(s)

    def reduced_muon_grad(self, i: int) -> torch.Tensor:
        o = self.plan.muon_off[i] - self.rank * self.plan.m_seg
        s = self.plan.muon_shapes[i]
        return self.gm_seg[o:o + _numel(s)].view(s)

    def reduced_adam_grad(self, i: int, start: int, n: int) -> torch.Tensor:
        o = self.plan.adam_off[i] + start - self.rank * self.plan.a_seg
        return self.ga_seg[o:o + n]

    def owned_grad_views(self) -> List[torch.Tensor]:
        views = [self.reduced_muon_grad(i).reshape(-1) for i in self.mine]
        views += [self.reduced_adam_grad(i, start, n) for i, start, n in self.pieces]
        return views

    def owned_tensor_ids(self) -> List[int]:
        """The grad tensor index of each of owned_grad_views(): AdamW param i is i, Muon param i is n_adam + i."""
        na = len(self.plan.adam_shapes)
        return [na + i for i in self.mine] + [i for i, _, _ in self.pieces]

    @torch.no_grad()
    def step(self, max_norm: Optional[float] = 1.0, grad_divisor: Optional[float] = None,
             marks: Optional[list] = None, norms: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One sharded step. `norms` (fp32, one per Muon param, on the device) receives ||p||_F of every Muon param
        after the update (the ELR tracker's NormTracker.sample, elr.py:85-87), computed in the apply pass. `marks`
        (eager use only): a list that receives (phase name, CUDA event) pairs recorded on the current stream after
        each phase, for a per-phase time breakdown."""
        from .functional import AdamWItem, MuonItem
        plan, r = self.plan, self.rank

        def mark(name):
            if marks is not None:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                marks.append((name, e))
        mark("start")
        nt = self.n_tensors
        if self._peer_pieces is not None:   # reduced from every rank's memory, the clip's sums in the same pass
            dist.all_reduce(self._gflag, group=self.group)   # every rank's grads are complete before any is read
            mine = self.compute.peer_reduce(self._peer_pieces, plan.world, nt, grad_divisor)
            mark("reduce_scatter")
        else:
            _reduce_scatter(self.gm_seg, self.gm, plan.m_seg, r, self.group)
            _reduce_scatter(self.ga_seg, self.ga, plan.a_seg, r, self.group)
            mark("reduce_scatter")
            mine = self.compute.sumsq(self.owned_grad_views(), self.owned_tensor_ids(), nt, grad_divisor)
        sums = torch.empty(plan.world * nt, dtype=torch.float64, device=mine.device)
        dist.all_gather_into_tensor(sums, mine.reshape(nt), group=self.group)
        norm_coef = self.compute.coef(sums, nt, max_norm)
        mark("grad_norm")
        self.steps += 1
        muon = [MuonItem(self.muon_view(self.pm, i), self.reduced_muon_grad(i), self.bufs[i], self.muon_lr,
                         self.muon_lr * self.muon_wd if self.muon_wd else 0.0, self.momentum, self.nesterov)
                for i in self.mine]
        adam = []
        base = r * plan.a_seg
        for i, start, n in self.pieces:
            o = plan.adam_off[i] + start
            adam.append(AdamWItem(self.pa[o:o + n], self.reduced_adam_grad(i, start, n), self.m_state[o - base:o - base + n],
                                  self.v_state[o - base:o - base + n], self.adam_lr, self.adam_wd[i], self.steps))
        self.compute.update(muon, adam, norm_coef[1:2] if max_norm is not None else None, grad_divisor,
                            [self.muon_view(self.om, i) for i in self.mine])
        mark("owned_update")
        every = range(len(plan.muon_shapes))
        if self.peer_ptrs is not None:   # the owners' O, read in place over NVLink once every owner has written it
            dist.all_reduce(self._flag, group=self.group)
            updates = [self.peer_ptrs[plan.owner[i]] + 2 * plan.muon_off[i] for i in every]   # bf16 elements
        else:
            _all_gather_inplace(self.om, plan.m_seg, r, self.group)
            updates = [self.muon_view(self.om, i) for i in every]
        _all_gather_inplace(self.pa, plan.a_seg, r, self.group)
        mark("exchange")
        extras = {}   # passed only when asked for, so a Compute without them keeps working
        if self.em is not None:
            extras.update(ema=[self.muon_view(self.em, i) for i in every], ema_weight=1.0 - self.ema_decay)
        if norms is not None:
            extras["norms"] = norms
        self.compute.apply([MuonItem(self.muon_view(self.pm, i), None, None, self.muon_lr,
                                     self.muon_lr * self.muon_wd if self.muon_wd else 0.0, self.momentum, self.nesterov)
                            for i in every], updates, **extras)
        if self.ea is not None:
            self.compute.ema([self.ea], [self.pa], 1.0 - self.ema_decay)
        mark("apply_all")
        return norm_coef[0]


def capture(step: ShardedStep, max_norm: Optional[float] = 1.0, grad_divisor: Optional[float] = None):
    """Record one ShardedStep.step (its NCCL collectives and kernels) in a CUDA graph on every rank. The compute must
    keep AdamW's step count on the device (cuda_compute does). Returns (graph, norm tensor); replaying the graph is
    one step. Capture on every rank together, after at least one eager step; drop the graph before
    destroy_process_group."""
    torch.cuda.synchronize()
    dist.barrier(group=step.group)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        norm = step.step(max_norm=max_norm, grad_divisor=grad_divisor)
    return g, norm


def cuda_compute(ns_steps: int = 5, betas=(0.9, 0.95), eps: float = 1e-8, rms_scale: float = 0.2,
                 ns_variant: int = 0) -> Compute:
    """The step's compute on the CUDA library (libmoteopt.so). AdamW's step count is a device counter (so that a
    captured step stays correct when replayed). ns_variant as moteopt_muon_config::ns_variant (0: the reference's
    iteration)."""
    import ctypes as C

    from . import _lib as L
    from .functional import adamw_array, muon_array
    from .ops import grad_dtype_code, stream_handle, workspace

    def sumsq(views, tensors, n_tensors, divisor):
        if not views:
            return torch.zeros(n_tensors, dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
        dev = views[0].device
        out = torch.empty(n_tensors, dtype=torch.float64, device=dev)   # every entry written by the library
        n = len(views)
        ptrs = L.array(C.c_void_p, [v.data_ptr() for v in views])
        numels = L.array(C.c_int64, [v.numel() for v in views])
        dts = L.array(C.c_int, [grad_dtype_code(v) for v in views])
        ids = L.array(C.c_int, list(tensors))
        ws = workspace(dev, L.lib.moteopt_grad_sumsq_workspace_size(numels, n))
        L.check(L.lib.moteopt_grad_sumsq_tensors(ptrs, numels, dts, ids, n, n_tensors, float(divisor or 0.0),
                                                 C.c_void_p(out.data_ptr()), C.c_void_p(ws.data_ptr()), ws.numel(),
                                                 C.c_void_p(stream_handle(dev))), "moteopt_grad_sumsq_tensors")
        return out

    def coef(sums, n_tensors, max_norm):
        out = torch.empty(2, dtype=torch.float32, device=sums.device)
        L.check(L.lib.moteopt_clip_coef_from_tensor_sums(
            C.c_void_p(sums.data_ptr()), sums.numel() // n_tensors, n_tensors, int(max_norm is not None),
            float(max_norm or 0.0), C.c_void_p(out.data_ptr()), C.c_void_p(stream_handle(sums.device))),
            "moteopt_clip_coef_from_tensor_sums")
        return out

    def peer_reduce(pieces, world, n_tensors, divisor):
        if not pieces:
            return torch.zeros(n_tensors, dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
        dev = pieces[0][0].device
        out = torch.empty(n_tensors, dtype=torch.float64, device=dev)   # every entry written by the library
        arr = getattr(pieces, "packed", None)   # the ctypes array, built once and kept with its piece list
        if arr is None:
            arr = (L.PeerPiece * len(pieces))()
            for k, (dst, srcs, t) in enumerate(pieces):
                e = arr[k]
                e.dst = dst.data_ptr()
                for q, a in enumerate(srcs):
                    e.src[q] = a
                e.numel, e.dtype, e.tensor = dst.numel(), grad_dtype_code(dst), int(t)
            if isinstance(pieces, PeerPieces):
                pieces.packed = arr
        ws = workspace(dev, L.lib.moteopt_peer_reduce_workspace_size(arr, len(pieces)))
        L.check(L.lib.moteopt_peer_reduce_sumsq(arr, len(pieces), int(world), n_tensors, float(divisor or 0.0),
                                                C.c_void_p(out.data_ptr()), C.c_void_p(ws.data_ptr()), ws.numel(),
                                                C.c_void_p(stream_handle(dev))), "moteopt_peer_reduce_sumsq")
        return out

    counter = {}

    def update(muon, adam, coef_t, divisor, muon_out):
        dev = (muon[0].param if muon else adam[0].param).device if (muon or adam) else None
        if dev is None:
            return
        if dev not in counter:
            counter[dev] = torch.zeros((), dtype=torch.float32, device=dev)
        m_arr, a_arr = muon_array(muon), adamw_array(adam)
        cfg = L.MuonConfig(int(ns_steps), float(rms_scale), 1e-7, int(ns_variant))
        nbytes = L.lib.moteopt_optimizer_step_workspace_size_cfg(m_arr, len(muon), C.byref(cfg), a_arr, len(adam))
        ws = workspace(dev, nbytes)
        hp = L.AdamWHparams(float(betas[0]), float(betas[1]), float(eps), counter[dev].data_ptr())
        outs = L.array(C.c_void_p, [o.data_ptr() for o in muon_out])
        L.check(L.lib.moteopt_optimizer_step_with_coef_out(
            m_arr, len(muon), C.byref(cfg), a_arr, len(adam), C.byref(hp), float(divisor or 0.0),
            C.c_void_p(coef_t.data_ptr() if coef_t is not None else 0), outs, C.c_void_p(ws.data_ptr()),
            ws.numel(), C.c_void_p(stream_handle(dev))), "moteopt_optimizer_step_with_coef_out")

    def apply(muon, updates, ema=None, ema_weight=0.0, norms=None):
        if not muon:
            return
        dev = muon[0].param.device
        arr = (L.MuonParam * len(muon))()
        for k, (it, o) in enumerate(zip(muon, updates)):
            p = it.param
            if not isinstance(o, int) and (o.dtype != torch.bfloat16 or o.shape != p.shape or not o.is_contiguous()):
                raise ValueError("Muon updates must be contiguous bf16 tensors shaped like their params")
            e = arr[k]
            e.param = p.data_ptr()
            e.batch, e.rows, e.cols = (p.shape[0] if p.ndim == 3 else 1), p.shape[-2], p.shape[-1]
            e.lr, e.decay, e.momentum = float(it.lr), float(it.decay), float(it.momentum)
        cfg = L.MuonConfig(int(ns_steps), float(rms_scale), 1e-7, int(ns_variant))
        ptrs = L.array(C.c_void_p, [o if isinstance(o, int) else o.data_ptr() for o in updates])
        emas = L.array(C.c_void_p, [e.data_ptr() for e in ema]) if ema is not None else None
        if norms is not None and (norms.dtype != torch.float32 or norms.numel() < len(muon) or not norms.is_cuda):
            raise ValueError("norms must be an fp32 CUDA tensor with one entry per Muon param")
        ws = None
        if norms is not None:
            ws = workspace(dev, L.lib.moteopt_muon_apply_workspace_size(arr, len(muon)))
        L.check(L.lib.moteopt_muon_apply_ex(arr, len(muon), C.byref(cfg), ptrs, emas, float(ema_weight),
                                            C.c_void_p(norms.data_ptr() if norms is not None else 0),
                                            C.c_void_p(ws.data_ptr() if ws is not None else 0),
                                            ws.numel() if ws is not None else 0, C.c_void_p(stream_handle(dev))),
                "moteopt_muon_apply_ex")

    def ema(emas, params, weight):
        from .functional import ema_lerp
        ema_lerp([e.reshape(-1) for e in emas], [p.reshape(-1) for p in params], weight)

    def set_step(dev, n):
        if dev not in counter:
            counter[dev] = torch.zeros((), dtype=torch.float32, device=dev)
        counter[dev].fill_(float(n))

    return Compute(sumsq, coef, update, apply, set_step, ema, peer_reduce)
