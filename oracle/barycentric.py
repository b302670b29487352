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

import math

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


def _pool_cells(x: np.ndarray, cells: int) -> np.ndarray:
    """Area pooling of a frame-rate sequence ``[L, C]`` to ``cells`` rows:
    row i averages rows ``floor(i*L/n) .. ceil((i+1)*L/n) - 1``
    (``adaptive_avg_pool1d``, ``proposed/matrix_curvature_phase_frame_weave.py:3562-3582``)."""
    length = x.shape[0]
    if length == cells:
        return x.astype(np.float64)
    out = np.zeros((cells, x.shape[1]))
    for i in range(cells):
        lo, hi = (i * length) // cells, -(-((i + 1) * length) // cells)
        out[i] = x[lo:hi].astype(np.float64).mean(axis=0)
    return out


def _normalize(v: np.ndarray) -> np.ndarray:
    return v / np.maximum(np.linalg.norm(v, axis=-1, keepdims=True), 1e-8)


def lift(active: np.ndarray, active_frames, total: int, memory: int, boundary, plucker: np.ndarray,
         mouse, keyboard, mouse_memory, keyboard_memory, lambdas, mode: int = 2):
    """The control-barycentric lift restated
    (``_control_barycentric_residual_lift``, ``proposed/matrix_curvature_phase_frame_weave.py:3810-4374``)
    for batch 1: ``active [A, S, C]``, ``plucker [>= T*S, P]``, controls
    ``[L, C]`` or None.  Every skipped frame of a segment (memory frames, then
    the current frames, split at ``boundary`` when given) takes its two
    nearest anchors of that segment with
    ``softmax([log1p(-a), log(a)] - lp * (1 - cos cam) - la * (1 - cos act))``
    as weights, camera state the normalised spatial mean of the Plucker rows,
    action state the normalised area-pooled mouse | keyboard controls.
    Returns ``(full [T, S, C], weights [N, 2], targets [(t, l, r)])``."""
    a_count, spatial, channels = active.shape
    frames = [int(f) for f in active_frames]
    cam = _normalize(plucker[: total * spatial].astype(np.float64).reshape(total, spatial, -1).mean(axis=1))
    current = [x for x in (mouse, keyboard) if x is not None]
    if current:
        cur = np.concatenate([_pool_cells(x, total - memory) for x in current], axis=-1)
        mem_parts = [x for x in (mouse_memory, keyboard_memory) if x is not None]
        if memory:
            mem = (np.concatenate([_pool_cells(x, memory) for x in mem_parts], axis=-1) if mem_parts
                   else np.zeros((memory, cur.shape[1])))
            act = np.concatenate([mem, cur], axis=0)
        else:
            act = cur
        act = _normalize(act)
    else:
        act = np.zeros((total, 1))
    segments = ([(0, memory)] if memory else []) + (
        [(memory, total)] if boundary is None else [(memory, memory + boundary), (memory + boundary, total)])
    targets, weights = [], []
    for start, end in segments:
        seg = [f for f in frames if start <= f < end]
        for t in range(start, end):
            if t in frames:
                continue
            left = max(f for f in seg if f < t)
            right = min(f for f in seg if f > t)
            alpha = (t - left) / (right - left)
            logits = []
            for src in (left, right):
                dc = 1.0 - np.clip(cam[t] @ cam[src], -1.0, 1.0)
                da = 1.0 - np.clip(act[t] @ act[src], -1.0, 1.0)
                prior = math.log1p(-alpha) if src == left else math.log(alpha)
                logits.append(prior - lambdas[1] * dc - lambdas[2] * da)
            e = np.exp(np.array(logits) - max(logits))
            weights.append(e / e.sum())
            targets.append((t, left, right))
    w32 = np.array(weights, dtype=np.float32).reshape(-1, 2)
    full = np.zeros((total, spatial * channels), dtype=np.float32)
    pairs = [[frames.index(l), frames.index(r)] for _, l, r in targets]
    pair_write(active.reshape(a_count, -1), w32, pairs, [t for t, _, _ in targets], full, mode)
    for i, f in enumerate(frames):
        full[f] = active[i].reshape(-1)
    return full.reshape(total, spatial, channels), w32, targets
