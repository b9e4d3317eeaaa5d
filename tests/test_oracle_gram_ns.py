"""The Gram Newton-Schulz variant's specification (oracle.moteopt_oracle.gram_newton_schulz), on the CPU. It is an
opt-in alternative to the reference iteration (mote/train/muon.py:26-43), proposed in the reference's research notes
(docs/research/efficiency-campaign-2026-08-23.md:903-911), so it is held to the bar the GPU Newton-Schulz parity
tests set for the reference iteration, not to bit equality: after 5 iterations within 4e-2 relative Frobenius of the
reference's own bf16 outputs, and no farther from the exact (fp64) iteration than those outputs are, plus 3e-3."""

import numpy as np
import pytest

from oracle import moteopt_oracle as O
from tests.conftest import golden
from tests.golden.cases import NS_CASES, ns_input

NS5_TOL = 4e-2      # the 5-iteration bound of tests/test_gpu_parity.py
EXACT_SLACK = 3e-3


@pytest.mark.parametrize("shape", [(40, 40), (48, 64), (64, 48), (3, 24, 40), (2, 130, 72), (96, 200)])
@pytest.mark.parametrize("steps", [1, 2, 5])
def test_equals_the_reference_iteration_in_exact_arithmetic(shape, steps):
    u = ns_input(shape, 1)
    assert O.rel_frob(O.gram_newton_schulz_f64(u, steps), O.newton_schulz_f64(u, steps)) < 1e-11


@pytest.mark.parametrize("name,shape,seed", [c for c in NS_CASES if O.gram_ns_eligible(*c[1][-2:])])
def test_meets_the_newton_schulz_bar_against_the_reference_outputs(name, shape, seed):
    ref = O.bf16_from_bits(golden("ns_reference")[f"{name}_s5"]).reshape(shape)
    u = ns_input(shape, seed)
    g = O.gram_newton_schulz(u, 5)
    exact = O.newton_schulz_f64(u, 5)
    assert O.rel_frob(g, ref) <= NS5_TOL, O.rel_frob(g, ref)
    assert O.rel_frob(g, exact) <= O.rel_frob(ref, exact) + EXACT_SLACK


@pytest.mark.parametrize("shape", [(128, 256), (256, 128), (2, 96, 384), (256, 1024), (192, 640)])
def test_meets_the_newton_schulz_bar_on_wider_shapes(shape):
    u = ns_input(shape, 7)
    g = O.gram_newton_schulz(u, 5)
    o = O.newton_schulz(u, 5)
    exact = O.newton_schulz_f64(u, 5)
    assert O.rel_frob(g, o) <= NS5_TOL
    assert O.rel_frob(g, exact) <= O.rel_frob(o, exact) + EXACT_SLACK
    assert np.array_equal(g, O.bf16_round(g))   # bf16 values, as the kernel would store them


def test_square_matrices_are_left_to_the_reference_iteration():
    """On a square matrix the m x m iterate costs more products than X itself, and R = X X^T squares the condition
    number: in bf16 the variant lands well away from the exact iteration, so it is not offered there."""
    assert not O.gram_ns_eligible(768, 768) and not O.gram_ns_eligible(768, 1535)
    assert O.gram_ns_eligible(768, 1536) and O.gram_ns_eligible(3072, 768)
    u = ns_input((128, 128), 3)
    exact = O.newton_schulz_f64(u, 5)
    assert O.rel_frob(O.gram_newton_schulz(u, 5), exact) > O.rel_frob(O.newton_schulz(u, 5), exact) + EXACT_SLACK


def test_flops_fall_on_every_eligible_shape():
    for m, n in [(768, 1536), (768, 3072), (3072, 768), (512, 2048), (1024, 4096), (128, 1024)]:
        assert O.gram_ns_flops(m, n) < O.ns_flops(m, n)
    assert O.gram_ns_flops(768, 768) > O.ns_flops(768, 768)
    # 768 x 3072: 4 s^2 l + 34 s^3 = 50 s^3 against 5 (4 s^2 l + 2 s^3) = 90 s^3, a 1.8x cut
    assert O.ns_flops(768, 3072) / O.gram_ns_flops(768, 3072) == pytest.approx(90 / 50)


@pytest.mark.parametrize("shape", [(256, 1024), (2, 512, 2048), (1024, 300), (600, 1800), (768, 3072)])
def test_the_kernel_storage_meets_the_same_bar(shape):
    """The GPU kernel's storage (gram_newton_schulz_blocked: R exactly symmetric, T whole; B and the final Q read
    through their upper 256 x 256 tiles) is as accurate as the reference iteration, and stays near the
    specification."""
    u = ns_input(shape, 11)
    g = O.gram_newton_schulz_blocked(u, 5)
    o = O.newton_schulz(u, 5)
    exact = O.newton_schulz_f64(u, 5)
    assert O.rel_frob(g, o) <= NS5_TOL
    assert O.rel_frob(g, exact) <= O.rel_frob(o, exact) + EXACT_SLACK
    assert O.rel_frob(g, O.gram_newton_schulz(u, 5)) <= 2e-2
    assert np.array_equal(g, O.bf16_round(g))


def test_block_symmetric_reads_lower_tiles_through_their_mirrors():
    m = np.arange(600 * 600, dtype=np.float32).reshape(600, 600)
    s = O.block_symmetric(m, 256)
    assert np.array_equal(s[:256, :], m[:256, :]) and np.array_equal(s[256:512, 256:], m[256:512, 256:])
    assert np.array_equal(s[256:512, :256], m[:256, 256:512].T) and np.array_equal(s[512:, 256:512], m[256:512, 512:].T)
    assert np.array_equal(s[512:, 512:], m[512:, 512:])


def test_symmetric_upper_mirrors_every_element_below_the_diagonal():
    m = np.arange(2 * 7 * 7, dtype=np.float32).reshape(2, 7, 7)
    s = O.symmetric_upper(m)
    assert np.array_equal(s, np.swapaxes(s, -1, -2))
    assert np.array_equal(np.triu(s), np.triu(m))
