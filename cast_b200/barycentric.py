"""The control-barycentric residual lift on the B200.

* :func:`direct_control_barycentric_pair_write` -- drop-in for the
  reference's two-anchor writer ``direct_control_barycentric_pair_write``
  (``proposed/matrix_control_barycentric_pair_kernel.py:158-204``): same
  arguments, checks and result, through ``cast_barycentric_pair_write``.
* :func:`control_barycentric_residual_lift` -- drop-in for the frame weave's
  ``_control_barycentric_residual_lift`` (``proposed/
  matrix_curvature_phase_frame_weave.py:3810-4374``): its control-conditioned
  weights (camera and action state, softmax over the two bracketing anchors)
  in ``cast_barycentric_weights`` and every target row in one writer launch.
"""

from __future__ import annotations

import bisect
import ctypes
import math

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


def lift_targets(anchor_values: list[int], total_temporal: int, memory_temporal: int,
                 current_segment_boundary: int | None):
    """The lift's targets in the reference's order (:4346-4355 segments, then
    every non-anchor frame of a segment between its nearest anchors,
    :4063-4080): ``[(target, left, right, left_index, right_index, alpha)]``
    with indices into ``anchor_values``."""
    segments = []
    if memory_temporal:
        segments.append((0, memory_temporal))
    if current_segment_boundary is None:
        segments.append((memory_temporal, total_temporal))
    else:
        split = memory_temporal + int(current_segment_boundary)
        if not memory_temporal < split < total_temporal:
            raise RuntimeError("invalid control-barycentric Current boundary")
        segments += [(memory_temporal, split), (split, total_temporal)]
    index = {f: i for i, f in enumerate(anchor_values)}
    out = []
    for start, end in segments:
        seg = [f for f in anchor_values if start <= f < end]
        if not seg:
            raise RuntimeError("control-barycentric segment has no exact anchor")
        for frame in range(start, end):
            if frame in index:
                continue
            right = bisect.bisect_left(seg, frame)
            if right == 0 or right == len(seg):
                raise RuntimeError("control-barycentric target is not bracketed by exact anchors")
            lf, rf = seg[right - 1], seg[right]
            out.append((frame, lf, rf, index[lf], index[rf], float(frame - lf) / float(rf - lf)))
    return out


def lift_weights(targets, full_plucker, mouse_cond, keyboard_cond, mouse_cond_memory,
                 keyboard_cond_memory, *, total_temporal: int, memory_temporal: int, spatial: int,
                 lambdas, writer_inputs=None):
    """``cast_barycentric_weights``: the weights ``[B, N, 2]`` of the targets
    from the camera and action state, on the plucker tensor's device.  With
    ``writer_inputs`` (int32 device tensors ``(pairs [N,2], frames [N])``) the
    launch also fills the pair writer's anchor slots and target frames."""
    dev = full_plucker.device
    b = full_plucker.shape[0]
    n = len(targets)
    out = torch.empty(b, n, 2, dtype=torch.float32, device=dev)
    plucker = full_plucker.detach()
    if plucker.dtype not in (torch.float32, torch.bfloat16):
        plucker = plucker.float()
    plucker = plucker.contiguous()

    def cond(x):
        if not isinstance(x, torch.Tensor):
            return None
        if x.ndim != 3:
            raise RuntimeError("control condition must have shape [B,T,C]")
        return x.detach().to(device=dev, dtype=torch.float32).contiguous()

    # the reference pools a sequence only for a non-empty segment (:3570)
    current = [cond(x) for x in (mouse_cond, keyboard_cond) if isinstance(x, torch.Tensor)]
    memory = [cond(x) for x in (mouse_cond_memory, keyboard_cond_memory)
              if memory_temporal and isinstance(x, torch.Tensor)]
    if current and memory and sum(c.shape[-1] for c in memory) != sum(c.shape[-1] for c in current):
        raise RuntimeError("Memory/Current action dimensions disagree")
    if not current:
        memory = []
    # the kernel concatenates slot 0 and slot 1 along channels like the
    # reference's torch.cat of the given sequences
    mouse, keyboard = (current + [None, None])[:2]
    mouse_m, keyboard_m = (memory + [None, None])[:2]
    tgt = (ctypes.c_int32 * (3 * n))(*[v for t in targets for v in t[:3]])
    prior = (ctypes.c_float * (2 * n))(*[v for t in targets
                                         for v in (math.log1p(-t[5]), math.log(t[5]))])
    slots = pairs_dev = frames_dev = None
    if writer_inputs is not None:
        slots = ctypes.cast((ctypes.c_int32 * (2 * n))(*[v for t in targets for v in t[3:5]]),
                            ctypes.c_void_p)
        pairs_dev, frames_dev = (_lib.ptr(x) for x in writer_inputs)
    P = _lib.ptr
    ln = lambda x: 0 if x is None else int(x.shape[1])  # noqa: E731
    ch = lambda x: 0 if x is None else int(x.shape[2])  # noqa: E731
    _lib.call("cast_barycentric_weights", P(plucker), int(plucker.dtype == torch.bfloat16), b,
              int(plucker.shape[1]), int(plucker.shape[2]), int(spatial), int(total_temporal),
              int(memory_temporal), P(mouse), ln(mouse), ch(mouse), P(keyboard), ln(keyboard),
              ch(keyboard), P(mouse_m), ln(mouse_m), ch(mouse_m), P(keyboard_m), ln(keyboard_m),
              ch(keyboard_m), n,
              ctypes.cast(tgt, ctypes.c_void_p), ctypes.cast(prior, ctypes.c_void_p),
              float(lambdas[1]), float(lambdas[2]), P(out), slots, pairs_dev, frames_dev, _stream(dev))
    return out, bool(current)


def control_barycentric_residual_lift(active_residual, active_frames, total_temporal, memory_temporal,
                                      current_segment_boundary, full_plucker, mouse_cond, keyboard_cond,
                                      mouse_cond_memory, keyboard_cond_memory, lambdas,
                                      runtime_optimized=False, runtime_vectorized=False,
                                      runtime_single_write=False, contraction_workspace=None,
                                      control_state_cache=None, weight_cache=None,
                                      runtime_batched_contraction=False,
                                      runtime_direct_pair_kernel=False,
                                      runtime_active_frame_values=None):
    """``MatrixCurvaturePhaseFrameWeave._control_barycentric_residual_lift``
    (``proposed/matrix_curvature_phase_frame_weave.py:3810-4374``) on the
    B200: the reference's checks and targets, every target's weights in one
    launch (``cast_barycentric_weights``, which also writes the writer's
    anchor slots and target frames), every target row in one launch of the
    pair writer (``left_then_right_fma`` rounding), the anchors copied in.
    The reference's control-state and weight caches are not kept: the
    weights are recomputed on the device every call.  Batch 1, fp32 residuals
    (the production Matrix path)."""
    del runtime_vectorized, contraction_workspace, control_state_cache, weight_cache
    del runtime_batched_contraction, runtime_direct_pair_kernel
    batch, active_count, spatial, channels = active_residual.shape
    if batch != 1 or active_residual.dtype != torch.float32:
        raise ValueError("the B200 lift takes batch-1 fp32 residuals")
    if active_count != int(active_frames.numel()):
        raise RuntimeError("active frame/residual cardinality mismatch")
    if runtime_active_frame_values is not None:
        values = tuple(int(v) for v in runtime_active_frame_values)
        if len(values) != active_count:
            raise RuntimeError("reused active-frame list/residual cardinality mismatch")
        if tuple(sorted(set(values))) != values:
            raise RuntimeError("reused active-frame list must be strictly chronological")
        if values[0] < 0 or values[-1] >= total_temporal:
            raise RuntimeError("reused active-frame list is out of range")
        source = "dynamic_selector_cpu_trace"
    else:
        values = tuple(int(v) for v in active_frames.tolist())
        source = "cuda_anchor_readback" if runtime_optimized else "cuda_predicates"
    if full_plucker is None:
        raise RuntimeError("control-barycentric reconstruction requires camera state")
    if full_plucker.ndim != 3 or int(full_plucker.shape[1]) < total_temporal * spatial:
        raise RuntimeError("camera state does not cover the full temporal grid")
    targets = lift_targets(list(values), total_temporal, memory_temporal, current_segment_boundary)
    full = active_residual.new_empty(batch, total_temporal, spatial, channels)
    action_available = any(isinstance(x, torch.Tensor) for x in (mouse_cond, keyboard_cond))
    if targets:
        dev = active_residual.device
        # the weights launch also writes the writer's slots and frames: no copy
        index = torch.empty(3 * len(targets), dtype=torch.int32, device=dev)
        pairs, frames = index[:2 * len(targets)], index[2 * len(targets):]
        weights, action_available = lift_weights(
            targets, full_plucker, mouse_cond, keyboard_cond, mouse_cond_memory, keyboard_cond_memory,
            total_temporal=total_temporal, memory_temporal=memory_temporal, spatial=spatial,
            lambdas=lambdas, writer_inputs=(pairs, frames))
        _lib.call("cast_barycentric_pair_write", _lib.ptr(active_residual.contiguous()), _lib.ptr(weights),
                  _lib.ptr(pairs), _lib.ptr(frames), _lib.ptr(full), active_count, total_temporal,
                  len(targets), spatial * channels, _MODES["left_then_right_fma"], _stream(dev))
    full.index_copy_(1, active_frames.to(device=full.device, dtype=torch.long), active_residual)
    return full, {
        "mode": "control_conditioned_local_two_anchor_residual",
        "control_lambdas": [lambdas[1], lambdas[2]],
        "temporal_prior": "chronological_linear_barycentric",
        "camera_source": "mean_encoded_plucker_per_latent",
        "action_source": "chronological_area_pooled_mouse_keyboard",
        "camera_available": True, "action_available": action_available,
        "control_state_cache_hit": False, "weight_cache_hits": 0, "weight_cache_misses": len(targets),
        "active_frame_source": source, "batched_contraction_calls": 0,
        "direct_pair_kernel_calls": 1 if targets else 0, "targets": len(targets),
        "support_sizes": [2] if targets else [], "nearest_bracketing_exact_anchors_only": True,
        "same_segment_only": True, "exact_anchors_restored": True,
        "backend": "cast_b200",
    }
