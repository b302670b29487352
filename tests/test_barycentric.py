"""CPU: the control-barycentric writer's oracle -- the single-rounding fp32
fused multiply-add against exact rational arithmetic (including ties), and
the rounding modes against the reference's own einsum contraction
(proposed/matrix_curvature_phase_frame_weave.py:4196-4201)."""

from fractions import Fraction

import numpy as np
import pytest
import torch

from oracle import barycentric as ob


def _round_f32(x: Fraction) -> np.float32:
    """Exact round-to-nearest-even of a rational to float32."""
    r = np.float32(float(x))
    best = r
    for cand in (np.nextafter(r, np.float32(-np.inf)), np.nextafter(r, np.float32(np.inf))):
        d_best, d_cand = abs(Fraction(float(best)) - x), abs(Fraction(float(cand)) - x)
        if d_cand < d_best or (d_cand == d_best and (cand.view(np.uint32) & 1) == 0):
            best = cand
    return np.float32(best)


def test_fma32_single_rounding():
    g = np.random.default_rng(0)
    a = (g.standard_normal(3000) * np.exp2(g.integers(-20, 20, 3000))).astype(np.float32)
    b = (g.standard_normal(3000) * np.exp2(g.integers(-20, 20, 3000))).astype(np.float32)
    c = (g.standard_normal(3000) * np.exp2(g.integers(-40, 40, 3000))).astype(np.float32)
    # ties: a*b exactly half an ulp of c away, with a tiny extra term of either sign
    one = np.float32(1.0)
    half_ulp = np.float32(2.0 ** -24)
    a = np.concatenate([a, np.full(4, half_ulp), np.array([half_ulp * 3, half_ulp], np.float32)])
    b = np.concatenate([b, np.array([1, -1, 1, -1], np.float32), np.array([1, 1], np.float32)])
    c = np.concatenate([c, np.full(4, one), np.array([one, np.float32(1 + 2.0 ** -23)], np.float32)])
    got = ob.fma32(a, b, c)
    want = np.array([_round_f32(Fraction(float(x)) * Fraction(float(y)) + Fraction(float(z)))
                     for x, y, z in zip(a, b, c)], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_modes_agree_with_reference_einsum():
    g = torch.Generator().manual_seed(4)
    values = torch.randn(1, 2, 880, 16, generator=g)
    weights = torch.softmax(torch.randn(1, 2, generator=g), dim=1)
    ref = torch.einsum("ba,bash->bsh", weights, values.float())[0].numpy()
    l, r = values[0, 0].numpy(), values[0, 1].numpy()
    wl, wr = weights[0].numpy()
    for mode in (1, 2, 3):
        got = ob.mix(mode, l, wl, r, wr)
        assert np.allclose(got, ref, rtol=2e-6, atol=1e-7)


def test_lift_targets_follow_reference_segments():
    """The lift's targets: per segment (memory, then the current frames split
    at the boundary), each non-anchor frame between its nearest anchors of
    that segment; a segment without an anchor, an unbracketed frame or a
    boundary outside the current frames is refused like the reference."""
    from cast_b200.barycentric import lift_targets
    got = lift_targets([0, 1, 2, 5, 6, 9], 10, 2, 4)
    assert [t[:3] for t in got] == [(3, 2, 5), (4, 2, 5), (7, 6, 9), (8, 6, 9)]
    assert got[0][3:5] == (2, 3) and abs(got[1][5] - 2 / 3) < 1e-12
    with pytest.raises(RuntimeError, match="no exact anchor"):
        lift_targets([0, 1, 5, 7], 8, 2, 2)
    with pytest.raises(RuntimeError, match="not bracketed"):
        lift_targets([0, 2, 5], 7, 0, None)
    with pytest.raises(RuntimeError, match="Current boundary"):
        lift_targets([0, 3], 4, 0, 4)
