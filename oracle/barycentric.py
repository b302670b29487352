"""CPU restatement of the control-barycentric two-anchor writer.

TEST INFRASTRUCTURE ONLY: the checker for ``cast_barycentric_pair_write``;
nothing in the product imports it.

Follows ``_direct_control_barycentric_pair_writer``
(``proposed/matrix_control_barycentric_pair_kernel.py:22-112``): per target
row, the left and right anchor frames times their weights, combined with the
rounding its arithmetic mode states (``mul.rn`` / ``add.rn`` / ``fma.rn`` in
fp32).  numpy has no fused multiply-add, so :func:`fma32` computes the exact
``a*b + c`` from float64 pieces and rounds it once to float32.
"""

from __future__ import annotations

import numpy as np

MODES = {"fused": 2, "separate": 1, "left_then_right_fma": 2, "right_then_left_fma": 3}


def fma32(a, b, c) -> np.ndarray:
    """float32 ``round(a*b + c)`` with a single rounding (finite inputs).

    a*b is exact in float64 (48-bit product); hi + lo = a*b + c exactly
    (TwoSum); rounding hi to float32 gives the right answer except when hi is
    exactly halfway between two float32 values and lo != 0, where lo's sign
    decides."""
    a, b, c = (np.asarray(x, dtype=np.float32).astype(np.float64) for x in (a, b, c))
    p = a * b
    hi = p + c
    bb = hi - p
    lo = (p - (hi - bb)) + (c - bb)
    r = hi.astype(np.float32)
    r64 = r.astype(np.float64)
    other = np.nextafter(r, np.where(hi > r64, np.float32(np.inf), np.float32(-np.inf))).astype(np.float32)
    mid = (r64 + other.astype(np.float64)) / 2.0
    tie = (hi == mid) & (hi != r64) & (lo != 0)
    # at an exact tie RN picked the even neighbour; lo says which side is nearer
    toward = np.where(lo > 0, np.maximum(r, other), np.minimum(r, other))
    return np.where(tie, toward, r).astype(np.float32)


def mix(mode: int, l, wl, r, wr) -> np.ndarray:
    l, r = np.asarray(l, np.float32), np.asarray(r, np.float32)
    wl, wr = np.float32(wl), np.float32(wr)
    if mode == 1:
        return ((l * wl).astype(np.float32) + (r * wr).astype(np.float32)).astype(np.float32)
    if mode == 3:
        return fma32(l, wl, (r * wr).astype(np.float32))
    return fma32(r, wr, (l * wl).astype(np.float32))


def pair_write(active, weights, source_pairs, target_frames, output, mode: int):
    """active [A, SC], weights [N, 2], source_pairs [N, 2], target_frames [N];
    writes output [T, SC] in place and returns it."""
    for n, t in enumerate(np.asarray(target_frames)):
        ls, rs = np.asarray(source_pairs)[n]
        wl, wr = np.asarray(weights, np.float32).reshape(-1, 2)[n]
        output[t] = mix(mode, active[ls], wl, active[rs], wr)
    return output
