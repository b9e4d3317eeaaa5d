"""The C ABI without a GPU: the library loads, exports every function include/moteopt.h declares, the ctypes
mirrors of the header's structs have the C layout, and the workspace-size functions (pure host code) agree with the
layout rules."""

import re
import subprocess
import tempfile
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "moteopt.h"


def declared():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"MOTEOPT_API\s+[\w\s\*]+?\b(moteopt_\w+)\s*\(", txt)))


def test_header_declares_the_bound_entry_points():
    from mote_b200 import _lib
    assert declared() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    from mote_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    syms = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    for name in declared():
        assert name in syms, name
        assert hasattr(_lib.lib, name)


def test_checked_library_exports_the_same_symbols_and_release_counts_nothing():
    """libmoteopt_checked.so (the -DMOTE_OPT_CHECKS build) has the release library's ABI; the release library's
    moteopt_check_count compiles no check and returns 0 without touching a device."""
    from mote_b200 import _lib
    checked = ROOT / "mote_b200" / "libmoteopt_checked.so"
    if not checked.exists():
        pytest.skip("libmoteopt_checked.so not built (python -m mote_b200.build --checked)")
    out = subprocess.run(["nm", "-D", "--defined-only", str(checked)], capture_output=True, text=True,
                         check=True).stdout
    syms = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared()) <= syms
    assert _lib.lib.moteopt_check_count(0) == 0


def test_ctypes_structs_match_the_c_layout():
    import ctypes as C
    from mote_b200 import _lib
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "moteopt.h"
#define P(T) printf(#T " %zu\n", sizeof(T));
#define O(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  P(moteopt_muon_param) P(moteopt_muon_config) P(moteopt_adamw_tensor) P(moteopt_adamw_hparams) P(moteopt_grad_config)
  P(moteopt_moe_bias) O(moteopt_moe_bias, expert_bias) O(moteopt_moe_bias, n_experts) O(moteopt_moe_bias, gamma)
  O(moteopt_muon_param, lr) O(moteopt_muon_param, nesterov) O(moteopt_muon_param, grad_dtype)
  O(moteopt_adamw_tensor, numel) O(moteopt_adamw_tensor, step) O(moteopt_adamw_tensor, grad_dtype)
  O(moteopt_muon_config, rms_scale) O(moteopt_muon_config, ns_variant) O(moteopt_grad_config, max_norm)
  O(moteopt_grad_config, grad_divisor_device)
  O(moteopt_adamw_hparams, device_step)
  P(moteopt_peer_piece) O(moteopt_peer_piece, src) O(moteopt_peer_piece, numel) O(moteopt_peer_piece, dtype)
  O(moteopt_peer_piece, tensor)
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = Path(d) / "p.c"
        c.write_text(src)
        exe = Path(d) / "p"
        subprocess.run(["gcc", "-I", str(ROOT / "include"), str(c), "-o", str(exe)], check=True)
        got = dict(ln.rsplit(" ", 1) for ln in subprocess.run([str(exe)], capture_output=True, text=True,
                                                                check=True).stdout.splitlines())
    m = {"moteopt_muon_param": _lib.MuonParam, "moteopt_muon_config": _lib.MuonConfig,
         "moteopt_adamw_tensor": _lib.AdamWTensor, "moteopt_adamw_hparams": _lib.AdamWHparams,
         "moteopt_grad_config": _lib.GradConfig, "moteopt_moe_bias": _lib.MoeBias,
         "moteopt_peer_piece": _lib.PeerPiece}
    for k, v in got.items():
        if "." in k:
            t, f = k.split(".")
            assert getattr(m[t], f).offset == int(v), k
        else:
            assert C.sizeof(m[k]) == int(v), k


def test_workspace_sizes_follow_the_layout():
    from mote_b200 import _lib
    lib = _lib.lib
    # 48 x 768^2: header, partials, denominators, then X0, X1, A, B at 1024-byte alignment
    n = lib.moteopt_newton_schulz_workspace_size(48, 768, 768)
    per = 48 * 768 * 768 * 2
    assert n >= 4 * per and n < 4 * per + 64 * 1024
    # a transposed shape needs the same iteration buffers as its transpose; only the apply pass's norm partials
    # differ (one fp64 sum per 16K-element chunk when iterated as stored, one per 64 x 64 tile when transposed)
    a = lib.moteopt_newton_schulz_workspace_size(2, 3072, 768)
    b = lib.moteopt_newton_schulz_workspace_size(2, 768, 3072)
    assert abs(a - b) <= 8 * 2 * (3072 // 64) * (768 // 64) + 1024
    # invalid shapes report 0
    assert lib.moteopt_newton_schulz_workspace_size(0, 8, 8) == 0
    assert lib.moteopt_newton_schulz_workspace_size(1, -1, 8) == 0


def test_entry_points_reject_bad_arguments_without_touching_a_device():
    import ctypes as C
    from mote_b200 import _lib
    lib = _lib.lib
    rc = lib.moteopt_newton_schulz(None, 0, None, 1, 8, 8, 5, 1e-7, None, 0, None)
    assert rc == -1 and b"null" in lib.moteopt_last_error()
    rc = lib.moteopt_profile_ns_events(C.c_void_p(1), None)
    assert rc == -1
    # the after-step entry points check their lists before any device call
    assert lib.moteopt_moe_update_bias(None, -1, None) == -1
    assert lib.moteopt_moe_update_bias(None, 2, None) == -1 and b"MoE" in lib.moteopt_last_error()
    bad = (_lib.MoeBias * 1)(_lib.MoeBias(None, None, 4, 1e-3))
    assert lib.moteopt_moe_update_bias(bad, 1, None) == -1 and b"null" in lib.moteopt_last_error()
    assert lib.moteopt_ema_lerp(None, None, None, 1, 0.1, None) == -1
    numel = (C.c_int64 * 1)(-5)
    ptrs = (C.c_void_p * 1)(1)
    assert lib.moteopt_ema_lerp(ptrs, ptrs, numel, 1, 0.1, None) == -1 and b"bad tensor" in lib.moteopt_last_error()
    assert lib.moteopt_muon_apply_ex(None, 1, None, None, None, 0.0, None, None, 0, None) == -1
    assert lib.moteopt_muon_apply_workspace_size(None, 3) == 0
    # the sharded step's per-tensor sums and peer reduction check their pieces first
    out = C.c_void_p(8)
    piece = _lib.PeerPiece()
    piece.dst, piece.numel, piece.dtype, piece.tensor = 8, 16, _lib.DTYPE_BF16, 0
    one = (_lib.PeerPiece * 1)(piece)
    assert lib.moteopt_peer_reduce_sumsq(one, 1, 9, 1, 0.0, out, None, 0, None) == -3   # more ranks than 8
    assert lib.moteopt_peer_reduce_sumsq(one, 1, 2, 1, 0.0, out, None, 0, None) == -1   # null source
    assert b"source" in lib.moteopt_last_error()
    piece.src[0], piece.src[1], piece.tensor = 8, 8, 3
    one = (_lib.PeerPiece * 1)(piece)
    assert lib.moteopt_peer_reduce_sumsq(one, 1, 2, 2, 0.0, out, None, 0, None) == -1   # tensor index past n_tensors
    assert b"tensor index" in lib.moteopt_last_error()
    two = (_lib.PeerPiece * 2)(piece, piece)
    assert lib.moteopt_peer_reduce_sumsq(two, 2, 2, 4, 0.0, out, None, 0, None) == -1   # one tensor twice
    assert lib.moteopt_peer_reduce_workspace_size(None, 2) == 0
    ids = (C.c_int * 1)(0)
    assert lib.moteopt_grad_sumsq_tensors(ptrs, numel, ids, ids, 1, 1, 0.0, out, None, 0, None) == -1
    assert lib.moteopt_clip_coef_from_tensor_sums(out, 2, 0, 1, 1.0, out, None) == -3


C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "moteopt.h"

/* A non-Python host: the c1 workload's optimizer-step workspace, sized and checked without a device. */
int main(void) {
  moteopt_muon_param m[2];
  moteopt_adamw_tensor a[1];
  memset(m, 0, sizeof m);
  memset(a, 0, sizeof a);
  m[0].batch = 4; m[0].rows = 768; m[0].cols = 768; m[0].grad_dtype = MOTEOPT_DTYPE_BF16;
  m[1].batch = 1; m[1].rows = 3072; m[1].cols = 768; m[1].grad_dtype = MOTEOPT_DTYPE_BF16;
  a[0].numel = 271 * 768; a[0].grad_dtype = MOTEOPT_DTYPE_F32;
  size_t ws = moteopt_optimizer_step_workspace_size(m, 2, 5, a, 1);
  size_t ns = moteopt_newton_schulz_workspace_size(4, 768, 768);
  moteopt_muon_config mc = {5, 0.2, 1e-7, 0};
  moteopt_adamw_hparams hp = {0.9, 0.95, 1e-8, NULL};
  moteopt_grad_config gc = {1, 1.0, 0.0, NULL};
  int rc = moteopt_optimizer_step(m, 2, &mc, a, 1, &hp, &gc, NULL, NULL, 0, NULL);   /* null pointers: refused */
  printf("%d %zu %zu %d %s\n", moteopt_version(), ws, ns, rc, rc == MOTEOPT_ERR_INVALID ? "refused" : "?");
  printf("%s\n", moteopt_last_error());
  return (ws > 0 && ns > 0 && rc == MOTEOPT_ERR_INVALID) ? 0 : 1;
}
"""


def test_a_c_host_compiles_links_and_calls_the_library(tmp_path):
    """include/moteopt.h is plain C (C11, -Wall -Werror): a C program builds against it, links libmoteopt.so and
    calls it; the host-only entry points answer without a device and a bad call returns its error code."""
    from mote_b200 import _lib
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    exe = tmp_path / "host"
    lib_dir = Path(_lib.LIB_PATH).parent
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"), str(src),
                    "-L", str(lib_dir), "-l:" + Path(_lib.LIB_PATH).name, "-Wl,-rpath," + str(lib_dir), "-o",
                    str(exe)], check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    version, ws, ns, rc, word = r.stdout.splitlines()[0].split()
    assert int(version) == _lib.lib.moteopt_version() and int(ws) > int(ns) > 0
    assert int(rc) == -1 and word == "refused"


def _kernel_resources():
    """{kernel: (registers, spilled bytes: the larger of the spill stores and loads)} from ptxas's report of the
    release build (mote_b200/_build/)."""
    from mote_b200 import build
    if not build.RESOURCES.exists():
        pytest.skip("no ptxas report: rebuild with python -m mote_b200.build")
    if build.RESOURCES.stat().st_mtime < build.LIB.stat().st_mtime - 5:
        pytest.skip("the ptxas report is older than the library")
    out, name, props = {}, None, None
    for line in build.RESOURCES.read_text().splitlines():
        m = re.search(r"Compiling entry function '(\w+)'", line)
        if m:
            name = m.group(1)
            continue
        m = re.search(r"Function properties for (\w+)", line)
        if m:   # a kernel's own properties, or those of a device function it calls (not the kernel's)
            props = m.group(1)
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and name and props == name:
            out.setdefault(name, [0, 0])[1] = max(int(m.group(1)), int(m.group(2)))
        m = re.search(r"Used (\d+) registers", line)
        if m and name:
            out.setdefault(name, [0, 0])[0] = int(m.group(1))
    return {k: tuple(v) for k, v in out.items()}


def test_kernel_register_budgets():
    """Registers and spills of every kernel, against the budgets their launch shapes were tuned for: the
    Newton-Schulz kernel's 320 threads at one CTA per SM with 96 registers (104 for the Gram variant's
    instantiation); no spills anywhere except the
    20-byte one of the division-free momentum pass (its fp64 sum of squares included), whose register cap (four
    blocks per SM) was measured to run at the copy bandwidth with it."""
    res = _kernel_resources()
    assert len(res) >= 20, sorted(res)
    ns = {k: v for k, v in res.items() if "ns_gemm_kernel" in k}
    ref = [v for k, v in ns.items() if "ns_gemm_kernelILb0E" in k]   # the reference iteration's instantiation
    assert ref and ref[0][0] <= 96, ns
    assert all(regs <= 104 and spill == 0 for regs, spill in ns.values()), ns   # 320 threads, one CTA per SM
    for k, (regs, spill) in res.items():
        allowed = 20 if "muon_momentum_kernelILb0E" in k else 0
        assert spill <= allowed, (k, regs, spill)
        assert regs <= 255, k
