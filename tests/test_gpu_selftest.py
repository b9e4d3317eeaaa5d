"""Two device primitives the optimizer's kernels rely on, checked through the C ABI's self-test entry points.

* The shared-divisor quotient. The Newton-Schulz normalisation (mote/train/muon.py:32-33: X / (||X|| + eps)) divides
  every element of a matrix by one norm. The kernels compute that quotient as r = RN(1/d), q = RN(a r), then one
  Markstein correction (e = a - q d by fma, RN(q + e r)), which must equal IEEE division bit for bit. Held against
  torch's fp32 `/` on the GPU (correctly rounded) with torch.equal over the optimizer's ranges (norms 1e-7 .. 1e4,
  entries 1e-9 .. 10), denominators at both ends of that range, tiny and subnormal numerators, zeros and special
  values. The denominator is a norm plus eps = 1e-7, so it never lies below 1e-7; the method needs 1/d to be a
  normal number (d < 2^126), which every finite norm of a training run satisfies.
* The bounded waits. Every wait of the Newton-Schulz kernel gives up after a limit and records
  MOTEOPT_STATUS_WAIT_TIMEOUT; the other CTAs of the launch see that and unwind. The self-test makes the wait run
  out on a counter and on an mbarrier that nothing completes, with a 2 ms limit, and checks that the kernel returns,
  the status bits, how long each CTA waited, and that the GPU keeps working afterwards. No GPU fault is involved.
"""

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mote_b200 import _lib  # noqa: F401
    return torch.device("cuda", 0)


def _divide(a: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    from mote_b200 import _lib as L
    out = torch.empty_like(a)
    L.check(L.lib.moteopt_selftest_divide(C.c_void_p(a.data_ptr()), C.c_void_p(d.data_ptr()),
                                          C.c_void_p(out.data_ptr()), a.numel(),
                                          C.c_void_p(torch.cuda.current_stream().cuda_stream)), "selftest_divide")
    return out


def _loguniform(gen, n, lo, hi, dev):
    e = torch.rand(n, generator=gen, device=dev, dtype=torch.float64) * (np.log(hi) - np.log(lo)) + np.log(lo)
    s = torch.where(torch.rand(n, generator=gen, device=dev) < 0.5, -1.0, 1.0).to(torch.float64)
    return (torch.exp(e) * s).to(torch.float32)


def _mismatch(a, d):
    got = _divide(a, d)
    want = a / d
    bad = ~((got == want) | (torch.isnan(got) & torch.isnan(want)))
    return int(bad.sum().item()), got, want


@pytest.mark.parametrize("num,den", [((1e-9, 10.0), (1e-7, 1e4)),      # the optimizer's entries and norms
                                     ((1e-9, 10.0), (1e-7, 2e-7)),     # norms at the eps floor
                                     ((1e-9, 10.0), (5e3, 1e4)),       # the largest norms
                                     ((1e-30, 1e-9), (1e-7, 1e4)),     # tiny entries
                                     ((1e-45, 1.1e-38), (1e-7, 1e4)),  # subnormal numerators
                                     ((1e-45, 1.1e-38), (5e3, 1e4)),   # subnormal numerators, largest norms
                                     ((1e-3, 1e30), (1e-7, 1e30))])    # far outside the optimizer's ranges
def test_shared_divisor_equals_ieee_division(dev, num, den):
    gen = torch.Generator(device=dev)
    gen.manual_seed(hash((num, den)) & 0xFFFF)
    n = 1 << 24
    for _ in range(4):   # 2^26 pairs per range
        a = _loguniform(gen, n, num[0], num[1], dev)
        d = _loguniform(gen, n, den[0], den[1], dev).abs()
        bad, got, want = _mismatch(a, d)
        if bad:
            i = int((got != want).nonzero()[0].item())
            raise AssertionError(f"{bad} quotients differ, e.g. {a[i].item()!r} / {d[i].item()!r}: "
                                 f"{got[i].item()!r} != {want[i].item()!r}")


def _grad_divide(a: torch.Tensor, d: float) -> torch.Tensor:
    from mote_b200 import _lib as L
    out = torch.empty_like(a)
    L.check(L.lib.moteopt_selftest_grad_divide(C.c_void_p(a.data_ptr()), C.c_float(d), C.c_void_p(out.data_ptr()),
                                               a.numel(), C.c_void_p(torch.cuda.current_stream().cuda_stream)),
            "selftest_grad_divide")
    return out


# token counts and other divisors: small integers, powers of two, significands just above 1 and just below 2, the
# ends of the fast window's divisor range and beyond it
GRAD_DIVISORS = [1.0, 2.0, 3.0, 7.0, 4096.0, 4097.0, 12345.0, 524287.0, 1e6, 3.3554431e7, 1.0000001, 1.9999999,
                 0.1, 1e-7, 2.0 ** -100, 2.0 ** -101, 2.0 ** 99, 2.0 ** 100, 3e38]


@pytest.mark.parametrize("d", GRAD_DIVISORS)
def test_grad_divisor_equals_ieee_division(dev, d):
    """One divisor for a whole pass (the normalisation's four-at-a-time form; also any shared divisor such as a token
    count): a fast path inside a window of |a|, the exact rare path outside it; equal to torch's fp32 `/` bit for bit
    over numerators of 1e-45 .. 1e38 (both signs, groups of four mixing in- and out-of-window values), quotients next
    to the smallest normal and subnormal, zeros, infinities and NaN."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(int(d * 7) & 0xFFFF)
    for lo, hi in ((1e-9, 10.0), (1e-45, 1e-30), (1e-30, 1e38)):
        a = _loguniform(gen, 1 << 23, lo, hi, dev)
        got, want = _grad_divide(a, d), a / torch.tensor(d, dtype=torch.float32, device=dev)
        bad = ~((got == want) | (torch.isnan(got) & torch.isnan(want)))
        assert int(bad.sum().item()) == 0, (d, lo, hi, int(bad.sum().item()))
        assert torch.equal(torch.signbit(got), torch.signbit(want))
    # quotients next to the smallest normal (2^-126), where rounding to 24 bits and then to the subnormal grid could
    # round twice, and next to the smallest subnormal
    x = torch.cat([2.0 ** -126 * (1 - torch.rand(1 << 20, generator=gen, device=dev, dtype=torch.float64) * 2 ** -18),
                   2.0 ** -149 * (0.25 + 4 * torch.rand(1 << 20, generator=gen, device=dev, dtype=torch.float64))])
    a = (x * d).to(torch.float32)
    a = a[torch.isfinite(a)]
    got, want = _grad_divide(a, d), a / torch.tensor(d, dtype=torch.float32, device=dev)
    assert torch.equal(got, want), (d, int((got != want).sum().item()))
    sp = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), float("nan"), 1.4e-45, -1.4e-45, 3.4028235e38],
                      device=dev)
    got, want = _grad_divide(sp, d), sp / torch.tensor(d, dtype=torch.float32, device=dev)
    assert torch.equal(torch.signbit(got), torch.signbit(want))
    assert bool(((got == want) | (torch.isnan(got) & torch.isnan(want))).all()), (got.tolist(), want.tolist())


def test_shared_divisor_special_values(dev):
    nums = torch.tensor([0.0, -0.0, 1.0, -1.0, 3.0, 1e-7, 1e4, 1.17549435e-38, 1.4e-45, 3.4e38, float("inf"),
                         float("nan")], device=dev)
    dens = torch.tensor([1e-7, 1.0000001e-7, 0.1, 1.0, 3.0, 7.0, 1e4, 1e30], device=dev)
    a = nums.repeat_interleave(dens.numel())
    d = dens.repeat(nums.numel())
    bad, got, want = _mismatch(a, d)
    assert bad == 0, [(x, y, g, w) for x, y, g, w in zip(a.tolist(), d.tolist(), got.tolist(), want.tolist()) if g != w]


@pytest.mark.parametrize("mode", [0, 1])
def test_bounded_waits_give_up_and_report_a_timeout(dev, mode):
    """mode 0: a persistent tile's counter wait (and CTA 1 unwinds as soon as it sees CTA 0's timeout);
    mode 1: a pipeline stage's mbarrier wait. Limit 2 ms."""
    from mote_b200 import _lib as L
    from mote_b200 import ops
    limit = 2e-3
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    elapsed = torch.zeros(2, dtype=torch.int64, device=dev)
    L.check(L.lib.moteopt_selftest_wait_timeout(mode, limit, C.c_void_p(counter.data_ptr()),
                                                C.c_void_p(status.data_ptr()), C.c_void_p(elapsed.data_ptr()),
                                                C.c_void_p(torch.cuda.current_stream().cuda_stream)), "selftest_wait")
    torch.cuda.synchronize()
    st = int(status.item())
    t0, t1 = (int(x) * 1e-9 for x in elapsed.tolist())
    assert st & L.STATUS_WAIT_TIMEOUT and st & L.STATUS_ABORTED, st
    assert limit <= t0 < limit + 0.05, (t0, t1)
    if mode == 0:   # CTA 1 stopped on CTA 0's timeout, long before its own limit of 4 x 2 ms
        assert t1 < 4 * limit, (t0, t1)
    else:           # an mbarrier wait ends on its own limit
        assert 4 * limit <= t1 < 4 * limit + 0.05, (t0, t1)
    # the context is usable afterwards: a Newton-Schulz call runs clean
    x = torch.randn(2, 64, 96, device=dev)
    ops.newton_schulz(x, 5)
    s2, _ = ops.read_status(dev)
    assert s2 & 3 == 0
