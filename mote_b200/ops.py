"""Torch-facing wrappers of the C ABI (include/moteopt.h). Device tensors in; the library's kernels run on the
current CUDA stream. PyTorch provides device memory and streams only.

Reference functions mirrored (noahsabaj/mote):
  newton_schulz    -- mote/train/muon.py:26-43
  clip_grad_norm_  -- torch.nn.utils.clip_grad_norm_ as called at mote/train/train.py:946
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, Iterable, Union

import torch

from . import _lib as L

_workspaces: Dict[int, torch.Tensor] = {}


def grad_dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.DTYPE_F32
    if t.dtype == torch.bfloat16:
        return L.DTYPE_BF16
    raise TypeError(f"moteopt handles fp32 and bf16 gradients, got {t.dtype}")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


HEADER_BYTES = 256   # the workspace header of include/moteopt.h


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A grow-only scratch buffer per device (allocated through PyTorch's caching allocator, 512-byte aligned).
    Calls on one device share it, so they must be issued on one stream at a time. Its first 256 bytes are the
    library's header (the last call's status word, norm and clip coefficient): zeroed when first allocated and
    copied when the buffer grows, so read_status still returns the last call's header after a growth."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        new = torch.empty(max(int(nbytes), 1024), dtype=torch.uint8, device=torch.device("cuda", idx))
        if ws is None:
            new[:HEADER_BYTES].zero_()
        else:
            new[:HEADER_BYTES].copy_(ws[:HEADER_BYTES])
        ws = new
        _workspaces[idx] = ws
    return ws


def read_status(device: torch.device, clear: bool = True):
    """(status bits, [total norm, clip coefficient]) of the last call on `device`; synchronises its stream."""
    ws = workspace(device, 1024)
    st = C.c_int(0)
    nc = (C.c_float * 2)()
    L.check(L.lib.moteopt_read_status(C.c_void_p(ws.data_ptr()), C.byref(st), nc, int(clear),
                                      C.c_void_p(stream_handle(device))), "moteopt_read_status")
    return st.value, (nc[0], nc[1])


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor (the optimizer runs only on the GPU)")


@torch.no_grad()
def newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7, variant: int = 0) -> torch.Tensor:
    """mote/train/muon.py:26-43: the quintic Newton-Schulz orthogonal factor of every matrix of G ([..., m, n]),
    computed on tcgen05 tensor cores; returns bf16 of G's shape. variant 1: the opt-in Gram Newton-Schulz variant
    (not the reference's iteration) when the long side is at least twice the short one."""
    _require_cuda(G, "G")
    if G.ndim < 2:
        raise ValueError("newton_schulz needs a matrix or a batch of matrices")
    if G.dtype not in (torch.float32, torch.bfloat16):
        G = G.float()
    G = G.contiguous()
    m, n = G.shape[-2], G.shape[-1]
    batch = G.numel() // max(m * n, 1)
    out = torch.empty(G.shape, dtype=torch.bfloat16, device=G.device)
    if G.numel() == 0:
        return out
    nbytes = L.lib.moteopt_newton_schulz_workspace_size_variant(batch, m, n, int(variant))
    if nbytes == 0:
        raise L.MoteoptError(f"newton_schulz: unsupported shape {tuple(G.shape)} or variant {variant}")
    ws = workspace(G.device, nbytes)
    L.check(L.lib.moteopt_newton_schulz_variant(C.c_void_p(G.data_ptr()), grad_dtype_code(G),
                                                C.c_void_p(out.data_ptr()), batch, m, n, int(steps), float(eps),
                                                int(variant), C.c_void_p(ws.data_ptr()), ws.numel(),
                                                C.c_void_p(stream_handle(G.device))), "moteopt_newton_schulz_variant")
    return out


@torch.no_grad()
def clip_grad_norm_(parameters: Union[torch.Tensor, Iterable[torch.Tensor]], max_norm: float) -> torch.Tensor:
    """torch.nn.utils.clip_grad_norm_ (2-norm) on the GPU: returns the total norm (a 0-dim fp32 tensor) and scales
    every grad in place by min(1, max_norm / (norm + 1e-6)). The reduction order is fixed, so the result is
    bitwise reproducible."""
    if isinstance(parameters, torch.Tensor):
        parameters = [parameters]
    grads = [p.grad for p in parameters if p.grad is not None]
    if not grads:
        return torch.tensor(0.0)
    dev = grads[0].device
    for g in grads:
        _require_cuda(g, "grad")
        if not g.is_contiguous():
            raise ValueError("clip_grad_norm_: grads must be contiguous")
    n = len(grads)
    ptrs = L.array(C.c_void_p, [g.data_ptr() for g in grads])
    numels = L.array(C.c_int64, [g.numel() for g in grads])
    dts = L.array(C.c_int, [grad_dtype_code(g) for g in grads])
    nbytes = L.lib.moteopt_clip_grad_norm_workspace_size(numels, n)
    ws = workspace(dev, nbytes)
    out = torch.empty((), dtype=torch.float32, device=dev)
    L.check(L.lib.moteopt_clip_grad_norm(ptrs, numels, dts, n, float(max_norm), C.c_void_p(out.data_ptr()),
                                         C.c_void_p(ws.data_ptr()), ws.numel(), C.c_void_p(stream_handle(dev))),
            "moteopt_clip_grad_norm")
    return out
