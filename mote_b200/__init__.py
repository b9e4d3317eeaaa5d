"""B200-native optimizer step for the Mote trainer (noahsabaj/mote): Muon + AdamW + global grad-norm clip.

The public names load the CUDA library (libmoteopt.so) on first use; `mote_b200.configs` and
`mote_b200.build` work without it.

    from mote_b200 import Muon, AdamW, MultiOpt, build_optimizer, split_muon_params, clip_grad_norm_, newton_schulz
"""

_LAZY = {
    "Muon": "optim", "AdamW": "optim", "MultiOpt": "optim", "build_optimizer": "optim",
    "split_muon_params": "optim", "fused_step": "optim", "set_lr": "optim",
    "clip_grad_norm_": "ops", "newton_schulz": "ops",
    "optimizer_step": "functional", "MuonItem": "functional", "AdamWItem": "functional",
    "CapturedStep": "functional", "moe_update_bias": "functional",
}


def __getattr__(name):
    mod = _LAZY.get(name)
    if mod is None:
        raise AttributeError(name)
    import importlib
    return getattr(importlib.import_module(f"{__name__}.{mod}"), name)


__all__ = sorted(_LAZY)
