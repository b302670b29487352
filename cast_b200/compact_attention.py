"""The frame weave's compact CWCA attention on the B200 kernels.

``compact_cwca_attention`` takes the place of
``MatrixCurvaturePhaseFrameWeave._compact_cwca_attention``
(``proposed/matrix_curvature_phase_frame_weave.py:5643-6125``) for CUDA
tensors.  The pieces of one call:

* packing of the active frames into the compact blocks (:5677-5684) ->
  ``cast_compact_pack`` (one pass over q, k, v, bf16 out);
* the pooled-Q/K ranking (:5687-5701 masked pooled means, :5718-5725 the
  stencil, :5828-5832 ``topk`` of score + 1e6 * stencil) -> ``cast_compact_select``,
  which also writes the per-block int8 codes the attention reads under the
  ``auto`` / ``int8`` precision policies;
* the block-sparse attention (:6086-6094) -> ``cast_rcsa_attention`` with the
  selection's precision modes;
* the scatter back to token order (:6095) -> ``cast_compact_unpack``.

The row degrees (the fixed edge budget split by the closed-loop provider or
the curvature profile, :5726-5817) stay host-side, restated in
:func:`compact_degrees` from the reference's steps; they are a few hundred
integers per layer.  On the two layers where the FC-PASM swap router refines
the selection (the factory's ``routing_active_layers``), the reference's own
method runs instead -- its torch ranking, then the B200 router and attention
through their own seams -- so the transport lookup and pair aliasing of
:5955-6076 are the reference's.
"""

from __future__ import annotations

import math
from bisect import bisect_left

import torch

from . import _lib, compact
from .rcsa import DEFAULT_INT8_TOLERANCE, POLICIES, Workspace, _stream, block_sparse_attention

_WS = Workspace()


def compact_select(q_packed: torch.Tensor, k_packed: torch.Tensor, valid: torch.Tensor,
                   degrees: torch.Tensor, *, block_size: int, grid: tuple[int, int],
                   policy: str = "auto", int8_tolerance: float = DEFAULT_INT8_TOLERANCE):
    """The compact ranking on packed bf16 ``[B,H,blocks*block_size,D]`` q/k
    with ``valid`` (bool or uint8 ``[blocks, block_size]`` or flat) and
    ``degrees`` (``[blocks]``, host or device).  Returns ``(indices int32
    [B,H,blocks,max_degree], counts int32 [B,H,blocks], q_codes, q_scales,
    k_codes, k_scales, qk_mode)`` (codes None under ``bf16``)."""
    if policy not in POLICIES:
        raise ValueError(f"policy must be one of {sorted(POLICIES)}")
    b, h, length, d = q_packed.shape
    if length % block_size or k_packed.shape != q_packed.shape:
        raise ValueError("packed q/k must hold whole blocks of the same shape")
    blocks = length // block_size
    dev = q_packed.device
    deg_host = torch.as_tensor(degrees).to("cpu", torch.int64)
    if deg_host.numel() != blocks:
        raise ValueError("one degree per compact block is required")
    maxdeg = int(deg_host.max())
    deg = deg_host.to(device=dev, dtype=torch.int32)
    vmask = valid.reshape(-1).to(device=dev, dtype=torch.uint8).contiguous()
    idx = torch.empty(b, h, blocks, maxdeg, dtype=torch.int32, device=dev)
    cnt = torch.empty(b, h, blocks, dtype=torch.int32, device=dev)
    quant = policy != "bf16"
    qc = torch.empty_like(q_packed, dtype=torch.int8) if quant else None
    kc = torch.empty_like(k_packed, dtype=torch.int8) if quant else None
    qs = torch.empty(b, h, blocks, dtype=torch.float32, device=dev) if quant else None
    ks = torch.empty(b, h, blocks, dtype=torch.float32, device=dev) if quant else None
    mode = torch.empty(b, h, blocks, dtype=torch.uint8, device=dev) if quant else None
    lib = _lib.load()
    nbytes = lib.cast_compact_select_workspace_bytes(b, h, blocks, block_size, d)
    ws = _WS.get(dev, nbytes)
    P = _lib.ptr
    _lib.call("cast_compact_select", P(q_packed), P(k_packed), P(vmask), b, h, blocks, block_size, d,
              int(grid[0]), int(grid[1]), P(deg), maxdeg, P(idx), P(cnt), P(qc), P(qs), P(kc), P(ks),
              P(mode), POLICIES[policy], float(int8_tolerance), None, P(ws), ws.numel(), _stream(dev))
    return idx, cnt, qc, qs, kc, ks, mode


def compact_degrees(weave, layout, *, layer_index: int, blocks: int, local_max: int, spatial: int,
                    tt: int, compact_frames: int, memory_frames: int, provider, device):
    """Each compact block's degree (the reference's :5726-5817): ``mean_degree``
    for every row, the current rows' share moved by the closed-loop provider
    or the current curvature (largest remainder), then saturation at the block
    count with the overflow given to the first rows with capacity.  The
    arithmetic runs on ``device`` with the same torch operations as the
    reference, so the integers agree with the reference on that device.
    Returns ``(degrees int64 [blocks] on device, mean_degree, budget metadata
    or None)``."""
    mean_degree = min(max(local_max, int(round(weave.sparse_density * blocks))), blocks)
    degrees = torch.full((blocks,), mean_degree, dtype=torch.long, device=device)
    memory_blocks = min(blocks, math.ceil(memory_frames / tt) * spatial)
    current_blocks = blocks - memory_blocks
    meta = None
    if current_blocks > 0 and mean_degree > local_max:
        base = max(local_max, math.ceil(4 * mean_degree / 5))
        current_frames = compact_frames - memory_frames
        active_global = layout.active_frames[layout.active_frames >= layout.memory_temporal]
        if provider is not None:
            current, meta = provider.compact_closed_loop_degrees(
                layer_index=layer_index, active_current=active_global,
                current_frame_origin=layout.memory_temporal, temporal_group_size=tt,
                spatial_blocks=spatial, mean_degree=mean_degree, base_degree=base,
                total_blocks=blocks, memory_blocks=memory_blocks)
            if int(current.numel()) != current_blocks:
                raise RuntimeError("compact Closed-Loop degree layout differs from packed rows")
            degrees[memory_blocks:] = current.reshape(-1)
        else:
            residual = current_blocks * (mean_degree - base)
            curvature = weave._current_curvature(layout.total_temporal - layout.memory_temporal)
            if curvature is not None and current_frames > 0:
                w_frames = curvature.to(device)[active_global - layout.memory_temporal]
                per_cell = []
                for c in range(current_blocks // spatial):
                    lo, hi = c * tt, min(current_frames, (c + 1) * tt)
                    per_cell.append(w_frames[lo:hi].mean() if lo < hi else w_frames.mean())
                weight = torch.stack(per_cell)[:, None].expand(-1, spatial)
                weight = 1.0 + torch.log1p(weight / weight.mean().clamp_min(1e-8))
                raw = residual * weight.reshape(-1) / weight.sum().clamp_min(1e-8)
                bonus = torch.floor(raw).long()
                left = residual - int(bonus.sum().item())
                if left > 0:
                    bonus[torch.argsort(raw - bonus, descending=True, stable=True)[:left]] += 1
                degrees[memory_blocks:] = base + bonus
    degrees.clamp_(max=blocks)
    missing = blocks * mean_degree - int(degrees.sum().item())
    while missing > 0:
        room = torch.nonzero(blocks - degrees > 0).flatten()
        if not int(room.numel()):
            break
        take = min(missing, int(room.numel()))
        degrees[room[:take]] += 1
        missing -= take
    return degrees, mean_degree, meta


def stencil_max(cells: int, nh: int, nw: int) -> int:
    """Largest Manhattan-<=1 neighbourhood (itself included) on the
    (cell, nh, nw) block grid -- ``local.sum(-1).max()`` of :5718-5726."""
    return 1 + sum(min(n - 1, 2) for n in (cells, nh, nw))


def _routes_here(weave, layer_index: int) -> bool:
    router = getattr(weave, "fc_pasm_swap_router", None)
    if router is None:
        return False
    if weave.world_spectral_corrector is not None and bool(
            getattr(weave.world_spectral_corrector, "fc_v21_bypass", False)):
        return False
    active = tuple(int(x) for x in router.config.active_layers)
    return not (weave.routing_skip_inactive_layers and active and layer_index not in active)


def compact_cwca_attention(weave, module, q, k, v, layout, *, original, policy="auto",
                           int8_tolerance=DEFAULT_INT8_TOLERANCE):
    """One compact CWCA attention call of ``weave`` on the B200 (see the module
    docstring); ``original`` is the reference's bound method, used for host
    tensors and on the routing layers."""
    layer_index = int(getattr(module, "block_idx", -1))
    if not q.is_cuda or _routes_here(weave, layer_index):
        return original(module, q, k, v, layout)
    provider = weave.geometry_provider
    provider = provider if (getattr(provider, "mode", None) == "closed_loop"
                            and hasattr(provider, "compact_closed_loop_degrees")) else None
    if provider is not None:
        if layer_index < 0:
            raise RuntimeError("compact Closed-Loop CWCA lacks a layer index")
        provider.begin_compact_layer(layer_index)
    packed, valid, token_to_packed = (layout.compact_block_indices, layout.compact_block_valid,
                                      layout.compact_token_to_packed)
    if packed is None or valid is None or token_to_packed is None:
        raise RuntimeError("compact CWCA layout was not constructed")
    if layout.compact_block_shape is None:
        raise RuntimeError("compact CWCA block shape is missing")
    block_size = int(layout.packed_block_size)
    blocks = int(packed.shape[0])
    tt, th, tw = (int(x) for x in layout.compact_block_shape)
    nh, nw = math.ceil(layout.spatial_height / th), math.ceil(layout.spatial_width / tw)
    spatial = nh * nw
    compact_frames = len(layout.active_frame_values)
    memory_frames = bisect_left(layout.active_frame_values, int(layout.memory_temporal))
    cells = math.ceil(memory_frames / tt) + math.ceil((compact_frames - memory_frames) / tt)
    if blocks != cells * spatial:
        raise RuntimeError("compact CWCA block-grid cardinality mismatch")
    local_max = stencil_max(cells, nh, nw)
    degrees, mean_degree, meta = compact_degrees(
        weave, layout, layer_index=layer_index, blocks=blocks, local_max=local_max,
        spatial=spatial, tt=tt, compact_frames=compact_frames, memory_frames=memory_frames,
        provider=provider, device=q.device)
    if provider is not None:
        if meta is None:
            raise RuntimeError("compact Closed-Loop CWCA did not allocate a feedback budget")
        provider.record_compact_budget(meta, degrees, local_support_preserved=True,
                                       native_qk_topk=True)
    degrees = degrees.to("cpu")
    qp, kp, vp = compact.pack(q, k, v, packed)
    idx, cnt, qc, qs, kc, ks, mode = compact_select(qp, kp, valid, degrees, block_size=block_size,
                                                    grid=(nh, nw), policy=policy,
                                                    int8_tolerance=int8_tolerance)
    key_valid = valid.reshape(-1).to(torch.uint8).contiguous()
    hint = degrees.to(torch.int32).expand(q.shape[0] * qp.shape[1], -1).numpy()
    out_packed = block_sparse_attention(qp, kp, vp, idx, cnt, q_block=block_size, k_block=block_size,
                                        key_valid=key_valid, q_codes=qc, q_scales=qs, k_codes=kc,
                                        k_scales=ks, qk_mode=mode, count_hint=hint)
    output = compact.unpack(out_packed, token_to_packed)
    routing_record = None
    router = getattr(weave, "fc_pasm_swap_router", None)
    if router is not None:
        # an inactive routing layer: the native top-k, recorded as the
        # reference records it (:5867-5903)
        if weave.world_spectral_corrector is not None and bool(
                getattr(weave.world_spectral_corrector, "fc_v21_bypass", False)):
            routing_record = {"layer_index": layer_index, "status": "independent_topk_fallback",
                              "fallback_reason": "fc_v21_bypass", "swap_count": 0,
                              "fc_cache_used": False, "g0_fallback": True, "fixed_budget": True,
                              "fc_v21_bypass": True}
        else:
            corrector = weave.world_spectral_corrector
            if corrector is None:
                raise RuntimeError("FC-PASM routing has no spectral corrector")
            step = int(getattr(corrector, "_step", -1))
            cache = getattr(corrector, "_fc_routing_transport", {})
            routing_record = {
                "layer_index": layer_index, "status": "independent_topk_fallback",
                "fallback_reason": "layer_not_enabled", "swap_count": 0,
                "transport_query_step": step, "transport_query_source_layer": layer_index - 1,
                "transport_available_layers": sorted(
                    int(key[1]) for key in cache
                    if isinstance(key, tuple) and len(key) == 2 and int(key[0]) == step),
                "transport_pair_aliases": [], "fc_cache_used": False, "fixed_budget": True,
                "routing_skip_inactive_layers": True,
            }
        router._records.append(routing_record)
    edges = int(degrees.sum())
    weave._last_compact_attention = {
        "compact_blocks": blocks, "requested_density": weave.sparse_density,
        "mean_degree": float(degrees.float().mean()), "minimum_degree": int(degrees.min()),
        "maximum_degree": int(degrees.max()), "edge_budget": edges,
        "effective_density": float(edges) / float(blocks * blocks), "empty_blocks": 0,
        "budget_source": meta["source"] if meta is not None else "compact_curvature",
        "closed_loop_previous_layer": meta["previous_layer"] if meta is not None else None,
        "closed_loop_feedback_consumed": meta is not None and meta["previous_layer"] is not None,
        "native_qk_topk": True, "local_support_preserved": True,
        "routing_mode": weave.routing_mode, "routing": routing_record,
        "precision_policy": policy,
    }
    return module.o(output.flatten(2).to(q.dtype))
