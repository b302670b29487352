"""Two-anchor residual writer of the control-barycentric reconstruction (B200).

Drop-in for ``direct_control_barycentric_pair_write``
(``proposed/matrix_control_barycentric_pair_kernel.py:158-204``): same
arguments, checks and result, through ``cast_barycentric_pair_write``.
"""

from __future__ import annotations

import torch

from . import _lib
from .rcsa import _stream

_MODES = {"fused": 0, "separate": 1, "left_then_right_fma": 2, "right_then_left_fma": 3}


def _validate(active_residual, weights, source_pairs, target_frames, output):
    if not active_residual.is_cuda:
        raise ValueError("direct pair writer requires CUDA tensors")
    if active_residual.dtype != torch.float32 or not active_residual.is_contiguous():
        raise ValueError("active residual must be contiguous FP32")
    if active_residual.ndim != 4 or active_residual.shape[0] != 1:
        raise ValueError("active residual must be [1,A,S,C]")
    batch, active_count, spatial, channels = active_residual.shape
    target_count = int(target_frames.numel())
    if weights.shape != (batch, target_count, 2) or weights.dtype != torch.float32:
        raise ValueError("weights must be contiguous FP32 [1,N,2]")
    if not weights.is_contiguous():
        raise ValueError("weights must be contiguous")
    if source_pairs.shape != (target_count, 2) or source_pairs.dtype != torch.int32:
        raise ValueError("source pairs must be int32 [N,2]")
    if source_pairs.device != active_residual.device or not source_pairs.is_contiguous():
        raise ValueError("source pairs must be contiguous on the input device")
    if target_frames.shape != (target_count,) or target_frames.dtype != torch.int32:
        raise ValueError("target frames must be int32 [N]")
    if target_frames.device != active_residual.device or not target_frames.is_contiguous():
        raise ValueError("target frames must be contiguous on the input device")
    if output.ndim != 4 or output.shape[0] != 1:
        raise ValueError("output must be [1,T,S,C]")
    if output.shape[2:] != (spatial, channels):
        raise ValueError("output spatial/channel shape mismatch")
    if output.dtype != torch.float32 or output.device != active_residual.device:
        raise ValueError("output must be FP32 on the input device")
    if not output.is_contiguous():
        raise ValueError("output must be contiguous")
    if target_count <= 0 or active_count not in (4, 5, 6):
        raise ValueError("production candidate requires 4/5/6 Current anchors and targets")
    return target_count, spatial, channels


def direct_control_barycentric_pair_write(active_residual, weights, source_pairs, target_frames,
                                          output, *, block: int = 256,
                                          arithmetic_mode: str = "fused"):
    """``output[0, target_frames[n]] = mix(active[0, pair[n][0]] * w[0,n,0],
    active[0, pair[n][1]] * w[0,n,1])``; ``arithmetic_mode`` fixes the
    rounding ("separate", "left_then_right_fma", "right_then_left_fma"; the
    reference leaves "fused" to its compiler, here it runs as
    "left_then_right_fma").  ``block`` is accepted for the reference's
    signature; the launch shape is chosen here."""
    target_count, spatial, channels = _validate(active_residual, weights, source_pairs,
                                                target_frames, output)
    if block not in (128, 256, 512, 1024):
        raise ValueError("block must be one of 128,256,512,1024")
    if arithmetic_mode not in _MODES:
        raise ValueError(f"unknown arithmetic mode: {arithmetic_mode}")
    P = _lib.ptr
    _lib.call("cast_barycentric_pair_write", P(active_residual), P(weights), P(source_pairs),
              P(target_frames), P(output), int(active_residual.shape[1]), int(output.shape[1]),
              target_count, spatial * channels, _MODES[arithmetic_mode],
              _stream(active_residual.device))
    return output
