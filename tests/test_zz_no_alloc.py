"""moteopt_clip_grad_norm_noalloc: the grad-norm clip for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc (or any allocating routine) when they clip: a host runtime that owns all device
memory through its own pool, a region where a new allocation would break stream ordering, a plain C caller with no
allocator of its own. This entry point keeps its scratch in a fixed array inside the library, so the caller passes
only the grads and the output. The test drives it through the C ABI and checks it against the workspace-based
moteopt_clip_grad_norm on the same grads, on two calls in a row (the shared scratch must not carry anything from one
call to the next). This file is collected last, so a run that stops at its first failure has run every other test.
"""

import ctypes as C

import numpy as np
import pytest
import torch


def _grads(dev, seed, dt):
    rng = np.random.default_rng(seed)
    shapes = [(1000, 3), (17,), (4, 4, 4), (70000,), (3, 64, 96)]
    return [torch.from_numpy(rng.standard_normal(s).astype(np.float32) * np.float32(0.3)).to(dev).to(dt) for s in shapes]


def _call(lib, fn, grads, max_norm, out, ws=None):
    n = len(grads)
    ptrs = (C.c_void_p * n)(*[g.data_ptr() for g in grads])
    numels = (C.c_int64 * n)(*[g.numel() for g in grads])
    dts = (C.c_int * n)(*[0 if g.dtype == torch.float32 else 1 for g in grads])
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if fn == "noalloc":
        return lib.moteopt_clip_grad_norm_noalloc(ptrs, numels, dts, n, max_norm, C.c_void_p(out.data_ptr()), stream)
    return lib.moteopt_clip_grad_norm(ptrs, numels, dts, n, max_norm, C.c_void_p(out.data_ptr()),
                                      C.c_void_p(ws.data_ptr()), ws.numel(), stream)


@pytest.mark.gpu
def test_noalloc_clip_matches_the_workspace_entry_point_twice_in_a_row():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mote_b200 import _lib
    lib = _lib.lib
    dev = torch.device("cuda", 0)
    for call, (seed, dt, max_norm) in enumerate([(1, torch.float32, 1.0), (2, torch.bfloat16, 0.5)]):
        a = _grads(dev, seed, dt)
        b = [g.clone() for g in a]
        n = len(a)
        numels = (C.c_int64 * n)(*[g.numel() for g in a])
        ws = torch.empty(lib.moteopt_clip_grad_norm_workspace_size(numels, n), dtype=torch.uint8, device=dev)
        out_a = torch.full((), -1.0, device=dev)
        out_b = torch.full((), -2.0, device=dev)
        assert _call(lib, "noalloc", a, max_norm, out_a) == 0, lib.moteopt_last_error()
        assert _call(lib, "ws", b, max_norm, out_b, ws) == 0, lib.moteopt_last_error()
        torch.cuda.synchronize()
        # same kernels, same fixed reduction order: the results agree exactly (tolerance 0, bitwise)
        assert out_a.item() == out_b.item(), (call, out_a.item(), out_b.item())
        assert out_a.item() > max_norm   # the clip is active
        for x, y in zip(a, b):
            assert torch.equal(x, y)


@pytest.mark.gpu
def test_noalloc_clip_reports_a_nonfinite_norm_through_out_norm():
    """A NaN grad: the call has no status word for moteopt_read_status, so the non-finite norm shows as a NaN
    out_norm, and the grads are scaled by torch's coefficient for it (NaN), as the workspace entry point does."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mote_b200 import _lib
    lib = _lib.lib
    dev = torch.device("cuda", 0)
    a = _grads(dev, 3, torch.float32)
    a[1][4] = float("nan")
    out = torch.zeros((), device=dev)
    assert _call(lib, "noalloc", a, 1.0, out) == 0, lib.moteopt_last_error()
    torch.cuda.synchronize()
    assert np.isnan(out.item())
    assert all(bool(torch.isnan(g).all()) for g in a)


def test_noalloc_clip_rejects_more_than_its_scratch_holds():
    """The size check runs on the host before any device work, so this runs without a GPU too."""
    from mote_b200 import _lib
    lib = _lib.lib
    n = 1
    ptrs = (C.c_void_p * n)(C.c_void_p(16))     # never dereferenced: the size check comes first
    numels = (C.c_int64 * n)(65536 * 16384 + 1)
    dts = (C.c_int * n)(0)
    rc = lib.moteopt_clip_grad_norm_noalloc(ptrs, numels, dts, n, 1.0, None, None)
    assert rc == -3
    assert b"fixed scratch" in lib.moteopt_last_error()
