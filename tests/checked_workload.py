"""A workload that reaches every kernel of the library, for the checked-build test (tests/test_gpu_checked.py).

Run as `python tests/checked_workload.py OUT.npz` with MOTEOPT_LIB naming the library to load; writes every output
tensor to OUT.npz and prints the library's index-check count (moteopt_check_count) on its last line. Not a test
module itself (no test_ prefix): the test runs it in subprocesses, once per library.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402


def main(out_path: str) -> None:
    from mote_b200 import _lib as L
    from mote_b200 import ops
    from mote_b200.distributed import cuda_compute
    from mote_b200.functional import (AdamWItem, MuonItem, ema_lerp, moe_update_bias, muon_step,
                                      optimizer_step)
    dev = torch.device("cuda", 0)
    L.lib.moteopt_check_count(1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    out = {}

    def rnd(shape, std, dtype=torch.float32):
        return (torch.randn(shape, generator=gen, device=dev) * std).to(dtype)

    # the whole step (clip, divisor, AdamW, Muon) on odd, padded, transposed and stacked shapes, both NS launch modes
    mshapes = [(37, 53), (130, 72), (2, 24, 40), (64, 64), (8, 3000), (300, 256), (96, 160)]
    ashapes = [(271, 16), (24,), (5, 7), (1,)]
    for mode in (1, 0):
        L.lib.moteopt_ns_set_persistent(mode)
        mp = [rnd(s, 0.02) for s in mshapes]
        ap = [rnd(s, 0.02) for s in ashapes]
        mb = [torch.zeros_like(p) for p in mp]
        am, av = [torch.zeros_like(p) for p in ap], [torch.zeros_like(p) for p in ap]
        ema = [p.clone() for p in ap + mp]
        norms = torch.zeros(len(mp), device=dev)
        for step in range(3):
            muon = [MuonItem(p, rnd(p.shape, 1e-3, torch.bfloat16), b, 0.02, 0.002) for p, b in zip(mp, mb)]
            adam = [AdamWItem(p, rnd(p.shape, 1e-3), m, v, 3e-4, 0.1, step + 1) for p, m, v in zip(ap, am, av)]
            out[f"norm{mode}_{step}"] = optimizer_step(muon, adam, ns_steps=5, betas=(0.9, 0.95), max_norm=0.5,
                                                       grad_divisor=3.0, ema=ema, ema_weight=0.1,
                                                       muon_norms=norms).cpu().numpy()
        for i, t in enumerate(mp + ap + ema + mb):
            out[f"s{mode}_{i}"] = t.cpu().numpy()
        out[f"norms{mode}"] = norms.cpu().numpy()
    L.lib.moteopt_ns_set_persistent(-1)
    # standalone Newton-Schulz and Muon-only steps (direct mode, fp32 grads)
    for i, s in enumerate([(3, 40, 72), (200, 96), (1, 256, 256)]):
        out[f"ns{i}"] = ops.newton_schulz(rnd(s, 1.0), steps=3).float().cpu().numpy()
    p = rnd((512, 2048), 0.02)
    muon_step([MuonItem(p, rnd(p.shape, 1e-3), torch.zeros_like(p), 0.02, 0.0)], ns_steps=2)
    out["muon_only"] = p.cpu().numpy()
    # AdamW launches in both work units (2K and 16K elements)
    for n in (3000, 10_500_000):
        p, m, v = rnd(n, 0.02), torch.zeros(n, device=dev), torch.zeros(n, device=dev)
        optimizer_step((), [AdamWItem(p, rnd(n, 1e-3, torch.bfloat16), m, v, 3e-4, 0.1, 1)], betas=(0.9, 0.95))
        out[f"adam{n}"] = p[:4096].cpu().numpy()
    # the clip on its own, the standalone EMA lerp, the sharded step's apply with its extras, the MoE bias step
    cps = [torch.nn.Parameter(rnd(s, 0.02)) for s in [(1000,), (33, 17)]]
    for q in cps:
        q.grad = rnd(q.shape, 1e-3)
    ops.clip_grad_norm_(cps, 1e-4)
    out["clip"] = np.concatenate([q.grad.cpu().numpy().ravel() for q in cps])
    es, ps = [rnd(n, 1.0) for n in (5, 16384 * 2 + 3)], [rnd(n, 1.0) for n in (5, 16384 * 2 + 3)]
    ema_lerp(es, ps, 0.3)
    out["lerp"] = np.concatenate([e.cpu().numpy() for e in es])
    comp = cuda_compute()
    pa = [rnd(s, 0.02) for s in [(96, 160), (160, 96)]]
    ea = [p.clone() for p in pa]
    na = torch.zeros(2, device=dev)
    comp.apply([MuonItem(p, None, None, 0.02, 0.002) for p in pa], [rnd(p.shape, 0.05, torch.bfloat16) for p in pa],
               ema=ea, ema_weight=0.7, norms=na)
    out["apply"] = np.concatenate([t.cpu().numpy().ravel() for t in pa + ea] + [na.cpu().numpy()])
    load, bias = torch.arange(64, device=dev, dtype=torch.float32), torch.zeros(64, device=dev)
    moe_update_bias([(load, bias, 1e-3)])
    out["moe"] = bias.cpu().numpy()
    torch.cuda.synchronize()
    np.savez(out_path, **out)
    st, _ = ops.read_status(dev)
    print("status", st)
    print("checks", L.lib.moteopt_check_count(1))


if __name__ == "__main__":
    main(sys.argv[1])
