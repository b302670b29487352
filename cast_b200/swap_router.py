"""FC-PASM fixed-budget swap router on the B200 kernels.

Mirrors ``FCPASMSwapRoutingConfig`` and ``FCPASMLocalCoordinateSwapRouter``
(``proposed/fc_pasm_swap_routing.py:23-62`` and ``:109-1115``): the same
constructor, ``refine`` keywords, fallback records, checks and error
messages.  ``refine`` keeps the reference's host-only gates (layer, grid,
anchors, a missing sketch) and runs everything else on the device with one
host synchronisation per call (the stats read at the end):

* ``cast_swap_objective`` (2 launches) builds the transport operators
  ``M(x) = I + sum_p V_p ((exp(i x g theta) - 1) U_p)`` straight from the
  published sketch (``theta``, ``g``), the coefficient vector and the Hessian
  of the objective (:414-548), and evaluates the transport gates on the
  sketches' mean affinities (:733-820);
* ``cast_swap_route`` (one proxy launch, one launch per round, one closing
  launch) takes the candidates, omission proxies and swap rounds, and the
  row-count statistics the record reports.

``U`` and ``V`` -- the bilinear lift, reflect padding, sqrt-Hann windowed
tiles and rfft2 of the attention grid's basis maps, and the irfft2 /
overlap-add / pooling synthesis of one bin -- depend only on the sketch
geometry and the grid, and are built once per geometry
(:func:`transport_basis`).  :func:`transport_operator` and
:func:`quadratic_terms` restate the reference's per-call torch construction
(:116-268); the tests use them to check the device objective.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F

from . import _lib

_OP_CACHE_KEY = "_cast_b200_operator_cache"


@dataclass(frozen=True)
class FCPASMSwapRoutingConfig:
    candidate_multiplier: int = 2
    num_swap_rounds: int = 1
    swap_eps: float = 1e-6
    lambda_anchor: float = 1.0
    lambda_reconstruction: float = 1.0
    sketch_groups: int = 16
    require_fc_transport: bool = False
    min_transport_affinity: float = 0.0
    min_pair_transport_affinity: float = 0.0
    max_swaps_per_call: int = 0
    active_layers: tuple[int, ...] = ()
    historical_only: bool = False
    same_bank_only: bool = False

    def __post_init__(self) -> None:
        if self.candidate_multiplier < 1:
            raise ValueError("candidate multiplier must be positive")
        if self.num_swap_rounds not in {0, 1, 2}:
            raise ValueError("FC-PASM routing supports zero to two swap rounds")
        if not math.isfinite(self.swap_eps) or self.swap_eps < 0.0:
            raise ValueError("swap epsilon must be finite and non-negative")
        if self.lambda_anchor < 0.0 or self.lambda_reconstruction < 0.0:
            raise ValueError("routing objective weights must be non-negative")
        if self.lambda_anchor + self.lambda_reconstruction <= 0.0:
            raise ValueError("routing objective must contain a positive term")
        if self.sketch_groups < 2 or self.sketch_groups % 2:
            raise ValueError("routing sketch groups must be a positive even number")
        if not 0.0 <= self.min_transport_affinity <= 1.0:
            raise ValueError("minimum FC transport affinity must be in [0, 1]")
        if not 0.0 <= self.min_pair_transport_affinity <= 1.0:
            raise ValueError("minimum pair FC transport affinity must be in [0, 1]")
        if self.max_swaps_per_call < 0:
            raise ValueError("maximum swaps per call must be non-negative")
        if any(layer < 0 for layer in self.active_layers):
            raise ValueError("routing active layers must be non-negative")
        if self.historical_only and self.same_bank_only:
            raise ValueError("historical-only routing already fixes the KV bank")


def _hann_sqrt(n_y: int, n_x: int, device) -> torch.Tensor:
    wy = torch.hann_window(n_y, periodic=False, device=device, dtype=torch.float32)
    wx = torch.hann_window(n_x, periodic=False, device=device, dtype=torch.float32)
    return (wy[:, None] * wx[None, :]).clamp_min(0.0).sqrt()


def transport_operator(transport: dict | None, pair: tuple[int, int], *, spatial_shape: tuple[int, int],
                       exponent: float, device) -> tuple[torch.Tensor, bool]:
    """The [output, input] operator on the ``spatial_shape`` attention grid
    that moves a block map along the FC-PASM transport of ``pair`` by
    ``exponent`` (identity, False when the pair has no usable sketch)."""
    gh, gw = int(spatial_shape[0]), int(spatial_shape[1])
    n = gh * gw
    eye = torch.eye(n, device=device, dtype=torch.float32)
    entry = transport.get("pairs", {}).get(pair) if transport is not None else None
    if not isinstance(entry, dict):
        return eye, False
    theta, aff = entry.get("theta"), entry.get("affinity")
    if not (isinstance(theta, torch.Tensor) and isinstance(aff, torch.Tensor)
            and theta.ndim == 3 and aff.shape == theta.shape):
        return eye, False
    cache = entry.setdefault(_OP_CACHE_KEY, {})
    key = (gh, gw, round(float(exponent), 12), str(device))
    if isinstance(cache.get(key), torch.Tensor):
        return cache[key].to(device), True
    oh, ow = (int(v) for v in transport["output_shape"])
    th_, tw_ = (int(v) for v in transport["transport_shape"])
    wh, ww = (int(v) for v in transport["window_shape"])
    sh, sw = (int(v) for v in transport["stride"])
    ph, pw = (int(v) for v in transport["padding"])
    gy, gx = (int(v) for v in transport["tile_grid"])
    tiles_n = gy * gx
    if theta.shape[0] != tiles_n:
        raise RuntimeError("FC routing frequency tiles do not match the OLA grid")
    win = _hann_sqrt(wh, ww, device)
    # analysis: each basis map lifted to the latent grid, windowed tiles
    lifted = F.interpolate(eye.reshape(n, 1, gh, gw), size=(oh, ow), mode="bilinear", align_corners=False)
    cols = F.unfold(F.pad(lifted, (pw, pw, ph, ph), mode="reflect"), kernel_size=(wh, ww), stride=(sh, sw))
    tiles = cols.transpose(1, 2).reshape(n * tiles_n, 1, wh, ww) * win
    pooled = (th_, tw_) != (wh, ww)
    if pooled:
        tiles = F.avg_pool2d(tiles, 2, 2, ceil_mode=True, count_include_pad=False)
    spec = torch.fft.rfft2(tiles.reshape(n, tiles_n, th_, tw_))
    theta = theta.to(device=device, dtype=torch.float32)
    aff = aff.to(device=device, dtype=torch.float32)
    if theta.shape[-2:] != spec.shape[-2:]:
        raise RuntimeError("FC routing frequency operator has an invalid shape")
    rot = torch.polar(torch.ones_like(theta), float(exponent) * aff * theta)
    moved = torch.fft.irfft2(spec * rot[None], s=(th_, tw_))
    still = torch.fft.irfft2(spec, s=(th_, tw_))
    if pooled:
        moved, still = (F.interpolate(x.reshape(n * tiles_n, 1, th_, tw_), size=(wh, ww), mode="bilinear",
                                      align_corners=False) for x in (moved, still))
    # synthesis: windowed overlap-add normalised by the summed squared window
    size = (oh + 2 * ph, ow + 2 * pw)
    norm = F.fold((win * win).reshape(-1, 1).expand(-1, tiles_n)[None], size, (wh, ww), stride=(sh, sw))
    norm = norm[:, :, ph:ph + oh, pw:pw + ow].clamp_min(1e-8)

    def ola(x):
        folded = F.fold((x.reshape(n, tiles_n, wh, ww) * win).reshape(n, tiles_n, -1).transpose(1, 2),
                        size, (wh, ww), stride=(sh, sw))
        return folded[:, :, ph:ph + oh, pw:pw + ow] / norm

    bh, bw = math.ceil(oh / gh), math.ceil(ow / gw)
    delta = F.avg_pool2d(ola(moved) - ola(still), (bh, bw), (bh, bw), ceil_mode=True, count_include_pad=False)
    if delta.shape[-2:] != (gh, gw):
        raise RuntimeError("FC routing operator did not return the attention grid")
    op = (eye + delta.reshape(n, n)).transpose(0, 1).contiguous()
    cache[key] = op
    return op, True


_BASIS_CACHE: dict = {}


def transport_basis(transport: dict, spatial_shape: tuple[int, int], device):
    """The transport operator's fixed linear parts for one sketch geometry and
    attention grid, as matrices (cached per geometry, grid and device):

    * ``u_re, u_im`` ``[P, F, n]``: the analysis -- each attention-grid basis
      map lifted bilinearly to the latent grid, reflect-padded, cut into the
      ``P`` sqrt-Hann windowed tiles (2x2-pooled when the sketch is coarse)
      and rfft2'd into ``F`` bins per tile;
    * ``v_re, v_im`` ``[P, n, F]``: the synthesis of one tile's spectrum --
      irfft2 (bilinear back to the window when coarse), windowed overlap-add
      normalised by the summed squared window, crop, block pooling to the
      attention grid -- applied to the real and the imaginary unit of each bin.

    The operator the reference builds per (pair, exponent x) is then
    ``M(x) = I + sum_p V_p ((exp(i x g_p theta_p) - 1) * U_p)`` by linearity
    (``irfft2(spec * rot) - irfft2(spec) = irfft2(spec * (rot - 1))``), which
    is what ``cast_swap_objective`` evaluates on the device."""
    gh, gw = int(spatial_shape[0]), int(spatial_shape[1])
    geo = tuple(tuple(int(v) for v in transport[k]) for k in
                ("output_shape", "transport_shape", "window_shape", "stride", "padding", "tile_grid"))
    key = (gh, gw, geo, str(device))
    hit = _BASIS_CACHE.get(key)
    if hit is not None:
        return hit
    (oh, ow), (th_, tw_), (wh, ww), (sh, sw), (ph, pw), (gy, gx) = geo
    n, tiles_n = gh * gw, gy * gx
    cpu = torch.device("cpu")
    win = _hann_sqrt(wh, ww, cpu)
    eye = torch.eye(n, dtype=torch.float32)
    lifted = F.interpolate(eye.reshape(n, 1, gh, gw), size=(oh, ow), mode="bilinear", align_corners=False)
    cols = F.unfold(F.pad(lifted, (pw, pw, ph, ph), mode="reflect"), kernel_size=(wh, ww), stride=(sh, sw))
    tiles = cols.transpose(1, 2).reshape(n * tiles_n, 1, wh, ww) * win
    pooled = (th_, tw_) != (wh, ww)
    if pooled:
        tiles = F.avg_pool2d(tiles, 2, 2, ceil_mode=True, count_include_pad=False)
    spec = torch.fft.rfft2(tiles.reshape(n, tiles_n, th_, tw_))       # [n, P, th, twf]
    fb = spec.shape[-2] * spec.shape[-1]
    u = spec.reshape(n, tiles_n, fb).permute(1, 2, 0)                    # [P, F, n]
    size = (oh + 2 * ph, ow + 2 * pw)
    norm = F.fold((win * win).reshape(-1, 1).expand(-1, tiles_n)[None], size, (wh, ww), stride=(sh, sw))
    norm = norm[:, :, ph:ph + oh, pw:pw + ow].clamp_min(1e-8)
    bh, bw = math.ceil(oh / gh), math.ceil(ow / gw)
    v = []
    for unit in (1.0, 1.0j):
        z = torch.zeros(tiles_n, fb, tiles_n, fb, dtype=torch.complex64)  # [P, F, tile, bin]
        idx = torch.arange(tiles_n)
        for f in range(fb):
            z[idx, f, idx, f] = unit
        x = torch.fft.irfft2(z.reshape(tiles_n * fb, tiles_n, spec.shape[-2], spec.shape[-1]),
                             s=(th_, tw_))
        if pooled:
            x = F.interpolate(x.reshape(-1, 1, th_, tw_), size=(wh, ww), mode="bilinear",
                              align_corners=False)
        x = (x.reshape(tiles_n * fb, tiles_n, wh, ww) * win).reshape(tiles_n * fb, tiles_n, -1)
        folded = F.fold(x.transpose(1, 2), size, (wh, ww), stride=(sh, sw))
        out = folded[:, :, ph:ph + oh, pw:pw + ow] / norm
        out = F.avg_pool2d(out, (bh, bw), (bh, bw), ceil_mode=True, count_include_pad=False)
        if out.shape[-2:] != (gh, gw):
            raise RuntimeError("FC routing operator did not return the attention grid")
        v.append(out.reshape(tiles_n, fb, n).permute(0, 2, 1))        # [P, n, F]
    basis = {
        "u_re": u.real.contiguous().to(device), "u_im": u.imag.contiguous().to(device),
        "v_re": v[0].contiguous().to(device), "v_im": v[1].contiguous().to(device),
        "tiles": tiles_n, "bins": fb, "n": n, "freq_shape": (int(spec.shape[-2]), int(spec.shape[-1])),
    }
    _BASIS_CACHE[key] = basis
    return basis


def operator_from_basis(basis: dict, theta: torch.Tensor, affinity: torch.Tensor, exponent: float):
    """``M(x)`` ``[out, in]`` from the basis matrices (the arithmetic of the
    device kernel, in torch; used by the tests as the kernel's checker)."""
    ang = float(exponent) * affinity.reshape(basis["tiles"], basis["bins"]).float() * \
        theta.reshape(basis["tiles"], basis["bins"]).float()
    c, s = torch.cos(ang) - 1.0, torch.sin(ang)                          # rot - 1
    ur, ui = basis["u_re"].to(ang.device), basis["u_im"].to(ang.device)
    wr = c[..., None] * ur - s[..., None] * ui                             # [P, F, n]
    wi = c[..., None] * ui + s[..., None] * ur
    m = torch.einsum("pof,pfj->oj", basis["v_re"].to(ang.device), wr) + \
        torch.einsum("pof,pfj->oj", basis["v_im"].to(ang.device), wi)
    return torch.eye(basis["n"], device=ang.device) + m


def quadratic_terms(*, temporal_cells: int, spatial: int, exact_frames: tuple[int, ...],
                    temporal_group_size: int, current_boundary: int, transport: dict | None,
                    lambda_anchor: float, lambda_reconstruction: float, device):
    """(coefficient [R], Hessian [R,R], transport used) of the routing
    objective over the current rows: anchor rows weighted by their cell's
    Exact-anchor count, and for every skipped target t between anchors l < r
    of one segment, |A_t e_l + B_t e_r|^2 with A_t = (1-a) M(a),
    B_t = a M(-(1-a)), a = (t-l)/(r-l) (:414-548)."""
    cells, sp = temporal_cells, spatial
    grid = ((int(transport.get("attention_spatial_h", 1)), int(transport.get("attention_spatial_w", sp)))
            if transport is not None else (1, sp))
    cell_of = {int(f): min(int(f) // int(temporal_group_size), cells - 1) for f in exact_frames}
    count = torch.zeros(cells, dtype=torch.float32)
    for f in exact_frames:
        count[cell_of[int(f)]] += 1.0
    coef = (count * float(lambda_anchor)).repeat_interleave(sp).to(device)
    hess = torch.zeros(cells * sp, cells * sp, dtype=torch.float32, device=device)
    used = False
    lam = float(lambda_reconstruction)
    for left, right in zip(exact_frames, exact_frames[1:]):
        if (left < current_boundary) != (right < current_boundary):
            continue
        lc, rc = cell_of[int(left)], cell_of[int(right)]
        ls, rs = slice(lc * sp, (lc + 1) * sp), slice(rc * sp, (rc + 1) * sp)
        for target in range(left + 1, right):
            a = float(target - left) / float(right - left)
            m_l, f_l = transport_operator(transport, (int(left), int(right)), spatial_shape=grid,
                                          exponent=a, device=device)
            m_r, f_r = transport_operator(transport, (int(left), int(right)), spatial_shape=grid,
                                          exponent=-(1.0 - a), device=device)
            used = used or f_l or f_r
            A, Bm = (1.0 - a) * m_l, a * m_r
            if lc == rc:
                C = A + Bm
                hess[ls, ls] += lam * (C.transpose(0, 1) @ C)
            else:
                hess[ls, ls] += lam * (A.transpose(0, 1) @ A)
                hess[rs, rs] += lam * (Bm.transpose(0, 1) @ Bm)
                hess[ls, rs] += lam * (A.transpose(0, 1) @ Bm)
                hess[rs, ls] += lam * (Bm.transpose(0, 1) @ A)
    return coef.contiguous(), hess.contiguous(), used


class FCPASMLocalCoordinateSwapRouter:
    """Refine compact pooled-Q/K routes without changing the row budgets."""

    def __init__(self, config) -> None:
        self.config = config
        self._records: list[dict[str, Any]] = []
        self._ws: torch.Tensor | None = None
        self._obj_bufs: dict = {}
        self._keep: list = []

    def _fallback(self, layer_index: int, reason: str, baseline, **extra):
        record = {"layer_index": int(layer_index), "status": "independent_topk_fallback",
                  "fallback_reason": reason, "swap_count": 0, **extra, "fixed_budget": True}
        self._records.append(record)
        return baseline, record

    def _workspace(self, nbytes: int, device) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < nbytes or self._ws.device != device:
            self._ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        return self._ws

    def refine(self, *, score, pooled_value, selected, counts, local, memory_blocks, spatial_shape,
               exact_current_frames, temporal_group_size, current_boundary, transport, layer_index):
        """Zero, one or two single-swap rounds on the device (:616-1077)."""
        call = self.enqueue(score=score, pooled_value=pooled_value, selected=selected, counts=counts,
                            local=local, memory_blocks=memory_blocks, spatial_shape=spatial_shape,
                            exact_current_frames=exact_current_frames,
                            temporal_group_size=temporal_group_size, current_boundary=current_boundary,
                            transport=transport, layer_index=layer_index)
        if isinstance(call, tuple):  # a host-side gate returned the reference's fallback
            return call
        return self.finish(call)

    def enqueue(self, *, score, pooled_value, selected, counts, local, memory_blocks, spatial_shape,
                exact_current_frames, temporal_group_size, current_boundary, transport, layer_index):
        """The device part of :meth:`refine`: the host gates, then the
        objective and the swap kernels enqueued on the current stream with no
        host synchronisation (capturable in a CUDA graph once the transport
        basis and the buffers exist).  Returns the fallback ``(selected,
        record)`` of a host gate, or the call state :meth:`finish` reads."""
        cfg = self.config
        if score.ndim != 4 or pooled_value.ndim != 4:
            raise ValueError("routing requires BHQK score and BHKD pooled values")
        if score.shape[:2] != pooled_value.shape[:2] or score.shape[-1] != pooled_value.shape[-2]:
            raise ValueError("routing score/value layouts differ")
        if selected.shape[:3] != score.shape[:3] or counts.shape != score.shape[:3]:
            raise ValueError("routing selection/count layouts differ")
        if local.shape != score.shape[-2:]:
            raise ValueError("routing local stencil has invalid shape")
        score = score.detach()
        pooled_value = pooled_value.detach()
        baseline = selected.clone()
        if cfg.active_layers and layer_index not in cfg.active_layers:
            return self._fallback(layer_index, "layer_not_enabled", baseline)
        B, H, Q, K = score.shape
        current_rows = Q - int(memory_blocks)
        spatial = int(spatial_shape[0] * spatial_shape[1])
        if current_rows <= 0 or current_rows % spatial:
            return self._fallback(layer_index, "no_rectangular_current_rows", baseline, fc_cache_used=False)
        cells = current_rows // spatial
        frames = tuple(int(f) for f in exact_current_frames)
        if tuple(sorted(set(frames))) != frames:
            raise ValueError("routing Exact Current frames must be unique and chronological")
        same_seg = [(l, r) for l, r in zip(frames, frames[1:])
                    if (l < current_boundary) == (r < current_boundary)]
        has_skipped = any(r - l > 1 for l, r in same_seg)
        if cfg.num_swap_rounds == 0 or len(frames) < 2 or not has_skipped:
            reason = ("zero_swap_rounds" if cfg.num_swap_rounds == 0
                      else "fewer_than_two_exact_anchors" if len(frames) < 2 else "no_skipped_frames")
            return self._fallback(layer_index, reason, baseline, fc_cache_used=False)
        pairs = transport.get("pairs", {}) if isinstance(transport, dict) else {}
        matching = [pairs[(l, r)] for l, r in same_seg
                    if r - l > 1 and isinstance(pairs.get((l, r)), dict)
                    and isinstance(pairs[(l, r)].get("theta"), torch.Tensor)]
        if cfg.require_fc_transport and not matching:
            return self._fallback(layer_index, "missing_previous_layer_fc_transport", baseline,
                                  matching_transport_affinity=0.0, fc_cache_used=False, g0_fallback=True)
        dev = score.device
        if dev.type != "cuda":
            raise ValueError("the swap router runs on a CUDA device")
        sel = selected.to(torch.int64).contiguous()
        S = sel.shape[-1]
        D = pooled_value.shape[-1]
        if D % cfg.sketch_groups:
            raise ValueError("value width must be divisible by sketch groups")
        stream = torch.cuda.current_stream(dev).cuda_stream
        stats = torch.empty(14, dtype=torch.float64, device=dev)
        obj = self._objective(cells=cells, spatial=spatial, spatial_shape=spatial_shape, frames=frames,
                              same_seg=same_seg, pairs=pairs, transport=transport,
                              group=int(temporal_group_size), boundary=int(current_boundary),
                              stats=stats, device=dev, stream=stream)
        cache_used = obj["sketched"] or bool(matching)
        lib = _lib.load()
        nbytes = lib.cast_swap_route_workspace_bytes(B, H, Q, K, D, S, int(memory_blocks),
                                                     cfg.candidate_multiplier, int(cfg.historical_only),
                                                     cfg.sketch_groups)
        ws = self._workspace(nbytes, dev)
        sc = score.float().contiguous()
        pv = pooled_value.float().contiguous()
        cn = counts.to(torch.int64).contiguous()
        lo = local.to(torch.uint8).contiguous()
        _lib.call("cast_swap_route", sc.data_ptr(), pv.data_ptr(), sel.data_ptr(), cn.data_ptr(),
                  lo.data_ptr(), _lib.ptr(obj["row_gate"]), obj["gate"].data_ptr(), obj["coef"].data_ptr(),
                  obj["hess"].data_ptr(), B, H, Q, K, D, S, int(memory_blocks), cfg.candidate_multiplier,
                  cfg.num_swap_rounds, float(cfg.swap_eps), cfg.sketch_groups, cfg.max_swaps_per_call,
                  int(cfg.historical_only), int(cfg.same_bank_only), stats.data_ptr(), ws.data_ptr(),
                  ws.numel(), stream)
        if sel.data_ptr() != selected.data_ptr():
            selected.copy_(sel)
        return {"stats": stats, "stream": stream, "selected": selected, "baseline": baseline,
                "layer_index": layer_index, "memory_blocks": int(memory_blocks), "K": K,
                "same_seg": same_seg, "matching": bool(matching), "cache_used": cache_used}

    def finish(self, call: dict):
        """Reads the stats of an enqueued call (the one host synchronisation),
        applies the reference's checks and returns ``(selected, record)``."""
        cfg = self.config
        stats, stream, selected, baseline = call["stats"], call["stream"], call["selected"], call["baseline"]
        layer_index, memory_blocks, K = call["layer_index"], call["memory_blocks"], call["K"]
        same_seg, matching, cache_used = call["same_seg"], call["matching"], call["cache_used"]
        st = stats.cpu().tolist()
        _lib.check_device(stream, "cast_swap_route")
        swaps, before, after, gained, max_swappable = st[0], st[1], st[2], st[3], int(st[4])
        gate, match_aff, gate_cells = int(st[5]), float(st[6]), int(st[7])
        if gate == 1:
            return self._fallback(layer_index, "weak_previous_layer_fc_transport", baseline,
                                  matching_transport_affinity=match_aff, fc_cache_used=False,
                                  g0_fallback=True)
        if gate == 2:
            return self._fallback(layer_index, "no_strong_transport_pair_cells", baseline,
                                  matching_transport_affinity=match_aff,
                                  min_pair_transport_affinity=cfg.min_pair_transport_affinity,
                                  pair_gate_cells=0, fc_cache_used=bool(matching))
        if max_swappable == 0:  # nothing was swappable: the kernels changed nothing
            return self._fallback(layer_index, "no_swappable_kv_selected", baseline)
        swaps = int(swaps)
        min_k, max_k, budget = int(st[8]), int(st[9]), int(st[10])
        hist_before, hist_after, current_changed = int(st[11]), int(st[12]), bool(st[13])
        if cfg.same_bank_only and hist_before != hist_after:
            raise RuntimeError("same-bank FC-PASM routing changed Memory KV counts")
        if cfg.historical_only and hist_after != hist_before:
            raise RuntimeError("FC-PASM routing changed a historical-KV row budget")
        if cfg.historical_only and current_changed:
            raise RuntimeError("FC-PASM routing modified Current-KV support")
        if after > before + 1e-5 * max(abs(before), 1.0):
            raise RuntimeError("FC-PASM swap increased its refinement objective")
        terms = sum(max(0, r - l - 1) for l, r in same_seg)
        f64 = lambda v: torch.tensor(v, dtype=torch.float32)  # noqa: E731
        record = {
            "layer_index": int(layer_index), "status": "refined",
            "candidate_multiplier": cfg.candidate_multiplier,
            "candidate_max": min(memory_blocks if cfg.historical_only else K,
                                 cfg.candidate_multiplier * max_swappable),
            "swap_rounds": cfg.num_swap_rounds, "max_swaps_per_call": cfg.max_swaps_per_call,
            "swap_count": swaps, "objective_before": f64(before), "objective_after": f64(after),
            "objective_improvement": f64(before - after),
            "average_swap_improvement": f64(gained / swaps if swaps else 0.0),
            "anchor_term_weight": cfg.lambda_anchor,
            "reconstruction_term_weight": cfg.lambda_reconstruction,
            "reconstruction_terms": terms, "fc_cache_used": cache_used,
            "matching_transport_affinity": match_aff,
            "min_pair_transport_affinity": cfg.min_pair_transport_affinity,
            "pair_gate_cells": gate_cells, "g0_fallback": not cache_used, "fixed_budget": True,
            "historical_only": cfg.historical_only, "same_bank_only": cfg.same_bank_only,
            "historical_budget_before": hist_before, "historical_budget_after": hist_after,
            "current_kv_support_unchanged": not current_changed,
            "minimum_k": min_k, "maximum_k": max_k,
            "budget_before": budget, "budget_after": budget,
            "unique_indices": True, "local_support_preserved": True,
        }
        self._records.append(record)
        return selected, record

    def _objective(self, *, cells, spatial, spatial_shape, frames, same_seg, pairs, transport, group,
                   boundary, stats, device, stream):
        """Launches ``cast_swap_objective``: host tables of the skipped targets
        and the anchor pairs (pointers to the published sketch tensors, no
        host synchronisation), buffers kept per shape."""
        cfg = self.config
        grid = ((int(transport.get("attention_spatial_h", 1)), int(transport.get("attention_spatial_w", spatial)))
                if isinstance(transport, dict) else (1, spatial))
        n = grid[0] * grid[1]
        if n != spatial:
            raise RuntimeError("FC routing operator did not return the attention grid")
        cell_of = {f: min(f // group, cells - 1) for f in frames}
        count = [0.0] * cells
        for f in frames:
            count[cell_of[f]] += 1.0
        tgt_theta, tgt_aff, tgt_alpha, tgt_cells = [], [], [], []
        pr_mean, pr_val, pr_cells, pr_match = [], [], [], []
        keep = []  # tensors the launch reads, alive until it is enqueued
        sketched = False
        for left, right in same_seg:
            if right - left <= 1:
                continue
            entry = pairs.get((left, right))
            theta = aff = None
            if isinstance(entry, dict):
                t_, a_ = entry.get("theta"), entry.get("affinity")
                if isinstance(t_, torch.Tensor) and isinstance(a_, torch.Tensor) and t_.shape == a_.shape \
                        and t_.ndim == 3:
                    theta = t_.to(device=device, dtype=torch.float32).contiguous()
                    aff = a_.to(device=device, dtype=torch.float32).contiguous()
                    keep += [theta, aff]
            mean = entry.get("mean_affinity", 0.0) if isinstance(entry, dict) else 0.0
            if isinstance(mean, torch.Tensor):
                mean = mean.detach().to(device=device, dtype=torch.float32).reshape(())
                keep.append(mean)
                pr_mean.append(mean.data_ptr())
                pr_val.append(0.0)
            else:
                pr_mean.append(None)
                pr_val.append(float(mean))
            pr_cells += [min((left + 1) // group, cells - 1), min((right - 1) // group, cells - 1)]
            pr_match.append(int(theta is not None))
            for t in range(left + 1, right):
                tgt_theta.append(theta.data_ptr() if theta is not None else None)
                tgt_aff.append(aff.data_ptr() if aff is not None else None)
                tgt_alpha.append(float(t - left) / float(right - left))
                tgt_cells += [cell_of[left], cell_of[right]]
                sketched = sketched or theta is not None
        basis = transport_basis(transport, grid, device) if sketched else None
        if basis is not None:
            for t_ in (x for x in keep if x.ndim == 3):
                if t_.shape[0] != basis["tiles"]:
                    raise RuntimeError("FC routing frequency tiles do not match the OLA grid")
                if tuple(t_.shape[-2:]) != basis["freq_shape"]:
                    raise RuntimeError("FC routing frequency operator has an invalid shape")
        R, T = cells * n, len(tgt_alpha)
        key = (R, T, str(device))
        bufs = self._obj_bufs.get(key)
        if bufs is None:
            bufs = {"coef": torch.empty(R, device=device), "hess": torch.empty(R, R, device=device),
                    "row_gate": torch.empty(R, dtype=torch.uint8, device=device),
                    "gate": torch.empty(1, dtype=torch.int32, device=device),
                    "ops": torch.empty(2 * T, n, n, device=device)}
            self._obj_bufs[key] = bufs
        arr = lambda ct, v: (ct * len(v))(*v)  # noqa: E731
        P = _lib.ptr
        pair_gate = cfg.min_pair_transport_affinity > 0.0
        _lib.call(
            "cast_swap_objective", n, basis["tiles"] if basis else 0, basis["bins"] if basis else 0,
            P(basis["u_re"]) if basis else None, P(basis["u_im"]) if basis else None,
            P(basis["v_re"]) if basis else None, P(basis["v_im"]) if basis else None, cells,
            arr(_lib.ctypes.c_float, count), T, arr(_lib.c_void_p, tgt_theta), arr(_lib.c_void_p, tgt_aff),
            arr(_lib.ctypes.c_double, tgt_alpha), arr(_lib.ctypes.c_int32, tgt_cells), len(pr_val),
            arr(_lib.c_void_p, pr_mean), arr(_lib.ctypes.c_float, pr_val), arr(_lib.ctypes.c_int32, pr_cells),
            arr(_lib.ctypes.c_int32, pr_match), int(cfg.require_fc_transport),
            float(cfg.min_transport_affinity), float(cfg.min_pair_transport_affinity),
            float(cfg.lambda_anchor), float(cfg.lambda_reconstruction), P(bufs["coef"]), P(bufs["hess"]),
            P(bufs["row_gate"]) if pair_gate else None, P(bufs["gate"]), stats.data_ptr(),
            P(bufs["ops"]), stream)
        self._keep = keep
        return {"coef": bufs["coef"], "hess": bufs["hess"], "gate": bufs["gate"],
                "row_gate": bufs["row_gate"] if pair_gate else None, "sketched": sketched}

    def summary(self) -> dict[str, Any]:
        rows = []
        for raw in self._records:
            row = {}
            for k, v in raw.items():
                if isinstance(v, torch.Tensor):
                    c = v.detach().float().cpu()
                    row[k] = float(c.item()) if c.numel() == 1 else [float(x) for x in c.flatten().tolist()]
                else:
                    row[k] = v
            rows.append(row)
        c = self.config
        return {"routing_mode": "fc_pasm_swap",
                "config": {"candidate_multiplier": c.candidate_multiplier,
                           "num_swap_rounds": c.num_swap_rounds, "swap_eps": c.swap_eps,
                           "lambda_anchor": c.lambda_anchor,
                           "lambda_reconstruction": c.lambda_reconstruction,
                           "sketch_groups": c.sketch_groups,
                           "require_fc_transport": c.require_fc_transport,
                           "min_transport_affinity": c.min_transport_affinity,
                           "min_pair_transport_affinity": c.min_pair_transport_affinity,
                           "max_swaps_per_call": c.max_swaps_per_call,
                           "active_layers": list(c.active_layers),
                           "historical_only": c.historical_only, "same_bank_only": c.same_bank_only},
                "records": rows}

    def reset(self) -> None:
        self._records.clear()
