"""ctypes binding of libmoteopt.so (the C ABI declared in include/moteopt.h).

The library is the product: there is no Python or PyTorch fallback. Importing this module without the built
library, or calling into it without a B200-class GPU, raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("MOTEOPT_LIB", Path(__file__).resolve().parent / "libmoteopt.so"))

DTYPE_F32 = 0
DTYPE_BF16 = 1
STATUS_WAIT_TIMEOUT = 1
STATUS_ABORTED = 2
STATUS_NONFINITE = 4

# every exported symbol of include/moteopt.h
EXPORTS = (
    "moteopt_version", "moteopt_last_error", "moteopt_read_status", "moteopt_launch_count", "moteopt_check_count",
    "moteopt_profile_ns_events", "moteopt_ns_set_persistent", "moteopt_ns_set_tall",
    "moteopt_optimizer_step_workspace_size", "moteopt_optimizer_step", "moteopt_optimizer_step_ex",
    "moteopt_optimizer_step_with_coef",
    "moteopt_optimizer_step_with_coef_out", "moteopt_muon_apply", "moteopt_muon_apply_workspace_size",
    "moteopt_muon_apply_ex", "moteopt_ema_lerp",
    "moteopt_ipc_export", "moteopt_ipc_import", "moteopt_ipc_close",
    "moteopt_grad_sumsq_workspace_size", "moteopt_grad_sumsq", "moteopt_clip_coef_from_sums",
    "moteopt_muon_step_workspace_size", "moteopt_muon_step",
    "moteopt_adamw_step",
    "moteopt_clip_grad_norm_workspace_size", "moteopt_clip_grad_norm", "moteopt_clip_grad_norm_noalloc",
    "moteopt_newton_schulz_workspace_size", "moteopt_newton_schulz",
    "moteopt_moe_update_bias",
    "moteopt_selftest_divide", "moteopt_selftest_wait_timeout",
    "moteopt_optimizer_step_workspace_size_cfg", "moteopt_muon_step_workspace_size_cfg",
    "moteopt_newton_schulz_workspace_size_variant", "moteopt_newton_schulz_variant",
    "moteopt_grad_sumsq_tensors", "moteopt_peer_reduce_workspace_size", "moteopt_peer_reduce_sumsq",
    "moteopt_clip_coef_from_tensor_sums", "moteopt_selftest_grad_divide",
)
MAX_PEERS = 8


class MuonParam(C.Structure):
    _fields_ = [("param", C.c_void_p), ("grad", C.c_void_p), ("momentum_buffer", C.c_void_p),
                ("batch", C.c_int64), ("rows", C.c_int64), ("cols", C.c_int64),
                ("lr", C.c_double), ("decay", C.c_double), ("momentum", C.c_double),
                ("nesterov", C.c_int), ("grad_dtype", C.c_int)]


class MuonConfig(C.Structure):
    _fields_ = [("ns_steps", C.c_int), ("rms_scale", C.c_double), ("ns_eps", C.c_double), ("ns_variant", C.c_int)]


class AdamWTensor(C.Structure):
    _fields_ = [("param", C.c_void_p), ("grad", C.c_void_p), ("exp_avg", C.c_void_p), ("exp_avg_sq", C.c_void_p),
                ("numel", C.c_int64), ("lr", C.c_double), ("weight_decay", C.c_double), ("step", C.c_int64),
                ("grad_dtype", C.c_int)]


class AdamWHparams(C.Structure):
    _fields_ = [("beta1", C.c_double), ("beta2", C.c_double), ("eps", C.c_double), ("device_step", C.c_void_p)]


class GradConfig(C.Structure):
    _fields_ = [("clip", C.c_int), ("max_norm", C.c_double), ("grad_divisor", C.c_double),
                ("grad_divisor_device", C.c_void_p)]


class StepExtras(C.Structure):
    _fields_ = [("ema", C.POINTER(C.c_void_p)), ("ema_weight", C.c_double), ("muon_norms", C.c_void_p),
                ("lr", C.c_void_p), ("muon_wd", C.POINTER(C.c_double)), ("muon_lr_max", C.POINTER(C.c_double))]


class MoeBias(C.Structure):
    _fields_ = [("load_acc", C.c_void_p), ("expert_bias", C.c_void_p), ("n_experts", C.c_int), ("gamma", C.c_float)]


class PeerPiece(C.Structure):
    _fields_ = [("dst", C.c_void_p), ("src", C.c_void_p * MAX_PEERS), ("numel", C.c_int64), ("dtype", C.c_int),
                ("tensor", C.c_int)]


class MoteoptError(RuntimeError):
    pass


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"libmoteopt.so not found at {LIB_PATH}: build it with `python -m mote_b200.build` "
                          "(the optimizer has no CPU or PyTorch fallback)")
    lib = C.CDLL(str(LIB_PATH))
    vp, i32, i64, sz, dbl, f32p = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_double, C.POINTER(C.c_float)
    sig = {
        "moteopt_version": (i32, []),
        "moteopt_last_error": (C.c_char_p, []),
        "moteopt_launch_count": (C.c_ulonglong, []),
        "moteopt_check_count": (C.c_longlong, [i32]),
        "moteopt_profile_ns_events": (i32, [vp, vp]),
        "moteopt_ns_set_persistent": (i32, [i32]),
        "moteopt_ns_set_tall": (i32, [i32]),
        "moteopt_read_status": (i32, [vp, C.POINTER(C.c_int), f32p, i32, vp]),
        "moteopt_optimizer_step_workspace_size": (sz, [C.POINTER(MuonParam), i32, i32, C.POINTER(AdamWTensor), i32]),
        "moteopt_optimizer_step": (i32, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig), C.POINTER(AdamWTensor), i32,
                                         C.POINTER(AdamWHparams), C.POINTER(GradConfig), vp, vp, sz, vp]),
        "moteopt_optimizer_step_with_coef": (i32, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig),
                                                   C.POINTER(AdamWTensor), i32, C.POINTER(AdamWHparams), dbl, vp, vp, sz,
                                                   vp]),
        "moteopt_optimizer_step_ex": (i32, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig), C.POINTER(AdamWTensor), i32,
                                            C.POINTER(AdamWHparams), C.POINTER(GradConfig), C.POINTER(StepExtras), vp,
                                            vp, sz, vp]),
        "moteopt_optimizer_step_with_coef_out": (i32, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig),
                                                       C.POINTER(AdamWTensor), i32, C.POINTER(AdamWHparams), dbl, vp,
                                                       C.POINTER(vp), vp, sz, vp]),
        "moteopt_muon_apply": (i32, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig), C.POINTER(vp), vp]),
        "moteopt_muon_apply_workspace_size": (sz, [C.POINTER(MuonParam), i32]),
        "moteopt_muon_apply_ex": (i32, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig), C.POINTER(vp), C.POINTER(vp),
                                        dbl, vp, vp, sz, vp]),
        "moteopt_ema_lerp": (i32, [C.POINTER(vp), C.POINTER(vp), C.POINTER(C.c_int64), i32, dbl, vp]),
        "moteopt_ipc_export": (i32, [vp, vp, C.POINTER(C.c_uint64)]),
        "moteopt_ipc_import": (i32, [vp, C.POINTER(vp)]),
        "moteopt_ipc_close": (i32, [vp]),
        "moteopt_grad_sumsq_workspace_size": (sz, [C.POINTER(C.c_int64), i32]),
        "moteopt_grad_sumsq": (i32, [C.POINTER(vp), C.POINTER(C.c_int64), C.POINTER(C.c_int), i32, dbl, vp, vp, sz, vp]),
        "moteopt_clip_coef_from_sums": (i32, [vp, i32, i32, dbl, vp, vp]),
        "moteopt_muon_step_workspace_size": (sz, [C.POINTER(MuonParam), i32, i32]),
        "moteopt_muon_step": (i32, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig), vp, vp, sz, vp]),
        "moteopt_adamw_step": (i32, [C.POINTER(AdamWTensor), i32, C.POINTER(AdamWHparams), vp, vp]),
        "moteopt_clip_grad_norm_workspace_size": (sz, [C.POINTER(C.c_int64), i32]),
        "moteopt_clip_grad_norm": (i32, [C.POINTER(vp), C.POINTER(C.c_int64), C.POINTER(C.c_int), i32, dbl, vp, vp, sz, vp]),
        "moteopt_clip_grad_norm_noalloc": (i32, [C.POINTER(vp), C.POINTER(C.c_int64), C.POINTER(C.c_int), i32, dbl, vp, vp]),
        "moteopt_newton_schulz_workspace_size": (sz, [i64, i64, i64]),
        "moteopt_newton_schulz": (i32, [vp, i32, vp, i64, i64, i64, i32, dbl, vp, sz, vp]),
        "moteopt_moe_update_bias": (i32, [C.POINTER(MoeBias), i32, vp]),
        "moteopt_selftest_divide": (i32, [vp, vp, vp, i64, vp]),
        "moteopt_selftest_wait_timeout": (i32, [i32, dbl, vp, vp, vp, vp]),
        "moteopt_selftest_grad_divide": (i32, [vp, C.c_float, vp, i64, vp]),
        "moteopt_optimizer_step_workspace_size_cfg": (sz, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig),
                                                           C.POINTER(AdamWTensor), i32]),
        "moteopt_muon_step_workspace_size_cfg": (sz, [C.POINTER(MuonParam), i32, C.POINTER(MuonConfig)]),
        "moteopt_newton_schulz_workspace_size_variant": (sz, [i64, i64, i64, i32]),
        "moteopt_newton_schulz_variant": (i32, [vp, i32, vp, i64, i64, i64, i32, dbl, i32, vp, sz, vp]),
        "moteopt_grad_sumsq_tensors": (i32, [C.POINTER(vp), C.POINTER(C.c_int64), C.POINTER(C.c_int),
                                             C.POINTER(C.c_int), i32, i32, dbl, vp, vp, sz, vp]),
        "moteopt_peer_reduce_workspace_size": (sz, [C.POINTER(PeerPiece), i32]),
        "moteopt_peer_reduce_sumsq": (i32, [C.POINTER(PeerPiece), i32, i32, i32, dbl, vp, vp, sz, vp]),
        "moteopt_clip_coef_from_tensor_sums": (i32, [vp, i32, i32, i32, dbl, vp, vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


lib = _load()


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib.moteopt_last_error().decode(errors="replace")
        raise MoteoptError(f"{what} failed ({rc}): {msg}")


def array(ctype, items):
    arr = (ctype * max(1, len(items)))()
    for i, x in enumerate(items):
        arr[i] = x
    return arr
