"""CPU restatement of Phase-Aware Reconstruction (FC-PASM) -- TEST INFRASTRUCTURE ONLY.

Restates the production path of
``WorldAlignedSpectralResidualCorrector._correct_frequency_confidence_pasm_reference``
(``proposed/matrix_world_spectral_residual.py:2771-3662``) with the factory
knobs (``src/interaction_accel/cast_matrix.py:74-96``): reference numerics,
ramp confidence on, temporal consistency off, fused complex weights, lean
in-place write.  Arithmetic is float64/complex128 (the reference runs
float32/complex64); ``tests/`` pin this restatement to outputs of the
reference itself (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

WINDOW = (11, 10)
STRIDE = (8, 8)
PADDING = (4, 5)


@dataclass(frozen=True)
class FCParams:
    """FC-PASM knobs (factory values from ``cast_matrix.py:74-78``)."""

    tau_low: float = 0.50
    tau_high: float = 0.75
    freq_power: float = 2.0
    temperature: float = 0.03
    ramp_confidence: bool = True
    current_anchor_boundary: int = 4


def hann_sym(n: int) -> np.ndarray:
    """``torch.hann_window(n, periodic=False)``."""
    if n == 1:
        return np.ones(1)
    k = np.arange(n)
    return 0.5 - 0.5 * np.cos(2.0 * math.pi * k / (n - 1))


def overlap_window(h: int = WINDOW[0], w: int = WINDOW[1]) -> np.ndarray:
    """sqrt-Hann analysis/synthesis window (``:1836-1851``)."""
    return np.sqrt(np.clip(hann_sym(h)[:, None] * hann_sym(w)[None, :], 0.0, None))


def tile_grid(height: int, width: int) -> tuple[int, int]:
    gh = (height + 2 * PADDING[0] - WINDOW[0]) // STRIDE[0] + 1
    gw = (width + 2 * PADDING[1] - WINDOW[1]) // STRIDE[1] + 1
    return gh, gw


def extract_tiles(x: np.ndarray, window: np.ndarray) -> np.ndarray:
    """``[E,C,H,W]`` -> windowed tiles ``[E,P,C,11,10]`` (``:1940-1984``).

    Reflect padding ``(4,5)``; patches in row-major grid order.
    """
    e, c, h, w = x.shape
    ph, pw = PADDING
    xp = np.pad(x, ((0, 0), (0, 0), (ph, ph), (pw, pw)), mode="reflect")
    gh, gw = tile_grid(h, w)
    wh, ww = WINDOW
    tiles = np.empty((e, gh * gw, c, wh, ww), dtype=np.float64)
    for gy in range(gh):
        for gx in range(gw):
            y0, x0 = gy * STRIDE[0], gx * STRIDE[1]
            tiles[:, gy * gw + gx] = xp[:, :, y0:y0 + wh, x0:x0 + ww]
    return tiles * window


def ola_normalization(height: int, width: int, window: np.ndarray) -> np.ndarray:
    """Cropped fold of ``window**2`` (``:1889-1938``)."""
    gh, gw = tile_grid(height, width)
    ph, pw = PADDING
    acc = np.zeros((height + 2 * ph, width + 2 * pw))
    for gy in range(gh):
        for gx in range(gw):
            y0, x0 = gy * STRIDE[0], gx * STRIDE[1]
            acc[y0:y0 + WINDOW[0], x0:x0 + WINDOW[1]] += window * window
    return acc[ph:ph + height, pw:pw + width]


def overlap_add(tiles: np.ndarray, height: int, width: int, window: np.ndarray) -> np.ndarray:
    """Normalized overlap-add inverse (``:1986-2081``): ``[N,P,C,11,10]`` -> ``[N,C,H,W]``."""
    n, p, c = tiles.shape[:3]
    gh, gw = tile_grid(height, width)
    ph, pw = PADDING
    acc = np.zeros((n, c, height + 2 * ph, width + 2 * pw))
    weighted = tiles * window
    for gy in range(gh):
        for gx in range(gw):
            y0, x0 = gy * STRIDE[0], gx * STRIDE[1]
            acc[:, :, y0:y0 + WINDOW[0], x0:x0 + WINDOW[1]] += weighted[:, gy * gw + gx]
    norm = ola_normalization(height, width, window)
    return acc[:, :, ph:ph + height, pw:pw + width] / norm


def normalized_rfft_radius(h: int, w: int) -> np.ndarray:
    """``_normalized_rfft_radius`` (``:2128-2135``)."""
    fy = np.abs(np.fft.fftfreq(h))
    fx = np.abs(np.fft.rfftfreq(w))
    r = np.sqrt(fy[:, None] ** 2 + fx[None, :] ** 2)
    return r / max(r.max(), 1e-8)


def frequency_threshold(params: FCParams, h: int = WINDOW[0], w: int = WINDOW[1]) -> np.ndarray:
    r = normalized_rfft_radius(h, w)
    return params.tau_low + (params.tau_high - params.tau_low) * r ** params.freq_power


def phat_displacement(unit: np.ndarray, coherence: np.ndarray, spatial=WINDOW) -> np.ndarray:
    """Channel-voted PHAT peak with parabolic sub-pixel refinement (``:2422-2496``)."""
    h, w = spatial
    corr = np.fft.irfft2(unit * coherence, s=(h, w), axes=(-2, -1))
    p = corr.shape[0]
    flat = corr.reshape(p, -1).argmax(axis=1)
    py, px = flat // w, flat % w
    ar = np.arange(p)
    center = corr[ar, py, px]
    xl = corr[ar, py, (px - 1) % w]
    xr = corr[ar, py, (px + 1) % w]
    yu = corr[ar, (py - 1) % h, px]
    yd = corr[ar, (py + 1) % h, px]

    def sub(before, middle, after):
        den = before - 2.0 * middle + after
        safe = np.where(np.abs(den) > 1e-8, den, 1.0)
        return np.where(np.abs(den) > 1e-8, np.clip(0.5 * (before - after) / safe, -0.5, 0.5), 0.0)

    sx = np.where(px >= (w + 1) // 2, px - w, px) + sub(xl, center, xr)
    sy = np.where(py >= (h + 1) // 2, py - h, py) + sub(yu, center, yd)
    return np.stack([sx, sy], axis=-1)


def linear_phase_ramp(disp: np.ndarray, spatial=WINDOW) -> np.ndarray:
    """``exp(-i(wx*dx + wy*dy))`` per tile (``:2498-2521``)."""
    h, w = spatial
    fy = 2.0 * math.pi * np.fft.fftfreq(h)
    fx = 2.0 * math.pi * np.fft.rfftfreq(w)
    ang = -(disp[:, 1, None, None] * fy[None, :, None] + disp[:, 0, None, None] * fx[None, None, :])
    return np.exp(1j * ang)


def endpoint_stats(left: np.ndarray, right: np.ndarray) -> dict:
    """``_frequency_confidence_endpoint_stats`` (``:2298-2363``) on ``[P,C,h,wf]``."""
    cross = right * np.conj(left)
    shared = cross.sum(axis=1)
    mag = np.abs(shared)
    energy = np.abs(cross).sum(axis=1)
    coherence = mag / np.maximum(energy, 1e-8)
    weight = energy.copy()
    weight[:, 0, 0] = 0.0
    denom = np.maximum(weight.sum(axis=(-2, -1)), 1e-8)
    base = np.clip((coherence * weight).sum(axis=(-2, -1)) / denom, 0.0, 1.0)
    unit = np.where(mag > 1e-8, shared / np.maximum(mag, 1e-8), 1.0 + 0.0j)
    theta = np.arctan2(unit.imag, unit.real)
    theta[:, 0, 0] = 0.0
    disp = phat_displacement(unit, coherence)
    pred = linear_phase_ramp(disp)
    circ = np.clip((unit * np.conj(pred)).real, 0.0, 1.0)
    ramp = np.clip((circ * weight).sum(axis=(-2, -1)) / denom, 0.0, 1.0)
    return {
        "theta": theta,
        "base_confidence": base,
        "ramp_confidence": ramp,
        "displacement": disp,
        "coherence": coherence,
        "weight": weight,
        "unit": unit,
    }


def affinity(stats: dict, params: FCParams, tile_confidence: np.ndarray | None = None):
    """Tile confidence and per-frequency affinity ``g`` (``:2137-2206``)."""
    if tile_confidence is None:
        conf = stats["base_confidence"]
        if params.ramp_confidence:
            conf = conf * stats["ramp_confidence"]
        conf = np.clip(conf, 0.0, 1.0)
    else:
        conf = np.asarray(tile_confidence, dtype=np.float64)
    thr = frequency_threshold(params)
    g = 1.0 / (1.0 + np.exp(-(conf[:, None, None] - thr[None]) / params.temperature))
    return conf, g


def mix(left, right, theta, g, alpha: float) -> np.ndarray:
    """Fused barycentric phase mix (``fused_reference_mix``, ``:3195-3224``)."""
    lp = (1.0 - alpha) * np.exp(1j * (g * alpha * theta))
    rp = alpha * np.exp(1j * (-g * (1.0 - alpha) * theta))
    return left * lp[:, None] + right * rp[:, None]


def bracket_targets(exact_local: list[int], current_length: int, boundary: int):
    """Segment-local bracket rule (``:2981-2990``): target -> (li, lf, ri, rf)."""
    out = []
    for t in range(current_length):
        if t in exact_local:
            continue
        same = t < boundary
        cands = [(i, f) for i, f in enumerate(exact_local) if (f < boundary) == same]
        left = [(i, f) for i, f in cands if f < t]
        right = [(i, f) for i, f in cands if f > t]
        if left and right:
            out.append((t, left[-1][0], left[-1][1], right[0][0], right[0][1]))
    return out


def correct(
    full_residual: np.ndarray,
    active_residual: np.ndarray,
    active_frames: list[int],
    memory_length: int,
    height: int,
    width: int,
    params: FCParams = FCParams(),
    tile_confidence: dict | None = None,
    return_intermediates: bool = False,
):
    """FC-PASM correction.

    ``full_residual``: ``[1,T,HW,C]`` float (bf16-representable values);
    ``active_residual``: ``[1,A,HW,C]`` for the sorted ``active_frames``.
    Returns the corrected residual (float64; the caller casts to the residual
    dtype) -- targets replaced, active frames copied, memory untouched.
    ``tile_confidence`` optionally maps ``(left_frame, right_frame)`` to a
    per-tile confidence that replaces base*ramp (``precomputed_tile_confidence``).
    """
    out = full_residual.astype(np.float64).copy()
    t_total = full_residual.shape[1]
    cur_len = t_total - memory_length
    c = full_residual.shape[-1]
    pos = [i for i, f in enumerate(active_frames) if f >= memory_length]
    exact_local = [active_frames[i] - memory_length for i in pos]
    exact = active_residual[0, pos].astype(np.float64).reshape(len(pos), height, width, c)
    exact = exact.transpose(0, 3, 1, 2)
    win = overlap_window()
    tiles = extract_tiles(exact, win)
    spectra = np.fft.rfft2(tiles, axes=(-2, -1))
    targets = bracket_targets(exact_local, cur_len, params.current_anchor_boundary)
    stats_cache: dict = {}
    inter = {"targets": [], "stats": {}, "affinity": {}}
    preds = []
    for (t, li, lf, ri, rf) in targets:
        key = (lf, rf)
        if key not in stats_cache:
            stats_cache[key] = endpoint_stats(spectra[li], spectra[ri])
        st = stats_cache[key]
        tc = None if tile_confidence is None else tile_confidence.get(key)
        conf, g = affinity(st, params, tc)
        alpha = float(t - lf) / float(rf - lf)
        mixed = mix(spectra[li], spectra[ri], st["theta"], g, alpha)
        preds.append(np.fft.irfft2(mixed, s=WINDOW, axes=(-2, -1)))
        inter["targets"].append((t, alpha, lf, rf))
        inter["stats"][key] = st
        inter["affinity"][key] = (conf, g)
    if preds:
        rec = overlap_add(np.stack(preds), height, width, win)  # [N,C,H,W]
        for n, (t, *_rest) in enumerate(targets):
            out[0, memory_length + t] = rec[n].transpose(1, 2, 0).reshape(height * width, c)
    for j, f in enumerate(active_frames):
        out[0, f] = active_residual[0, j]
    if return_intermediates:
        return out, inter
    return out
