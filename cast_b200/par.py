"""Host side of Phase-Aware Reconstruction (FC-PASM) on B200.

``FCPASMCorrector.correct`` has the keyword signature of
``WorldAlignedSpectralResidualCorrector.correct``
(``proposed/matrix_world_spectral_residual.py:5283-5296``) and the behaviour of
its production FC-PASM path with the factory knobs
(``_correct_frequency_confidence_pasm_reference``, ``:2771-3662``): the same
``first_chunk`` / ``no_memory`` fallbacks, and an in-place write of the
reconstructed skipped frames plus ``corrected[:, active_frames] =
active_residual`` (lean runtime, ``:3638-3645``).  The spectral work runs in
the CUDA kernels of ``libcast_b200.so``; there is no CPU path.
"""

from __future__ import annotations

import torch

from . import _lib

TILES = 18
FREQS = 66
MAX_PAIRS = 16                        # castk::kParMaxPairs
STATS_PER_PAIR = TILES * (2 * FREQS + 5)  # theta, confidence, g, displacement, base, ramp
MEANS_AT = MAX_PAIRS * STATS_PER_PAIR    # per-pair mean affinities, then the layer's
STATS_FLOATS = MEANS_AT + MAX_PAIRS + 1
_COUNT_CACHE: dict = {}  # device -> the constant affinity support count (18 * 66)


def bracket_targets(anchors: list[int], current_length: int, boundary: int):
    """Skipped current frames with their anchor pair, as the segment-local
    bracket rule of ``_correct_frequency_confidence_pasm_reference`` walks
    them (``:2981-3060``, ``:3225-3232``): chronological targets, each between
    the nearest anchors on either side within its own segment (frames below
    ``boundary`` and frames at or above it never pair).  Returns
    ``(targets, pair_of_target, pairs)`` with ``pairs`` the distinct
    ``(left, right)`` anchor frames in order of first use -- the order in
    which ``cast_par_fcpasm`` lays out its per-pair statistics."""
    targets, pair_of_target, pairs = [], [], []
    anchor_set = set(anchors)
    for t in range(current_length):
        if t in anchor_set:
            continue
        same = t < boundary
        seg = [f for f in anchors if (f < boundary) == same]
        left = [f for f in seg if f < t]
        right = [f for f in seg if f > t]
        if not left or not right:
            continue
        pair = (left[-1], right[0])
        if pair not in pairs:
            pairs.append(pair)
        targets.append(t)
        pair_of_target.append(pairs.index(pair))
    return targets, pair_of_target, pairs


class FCPASMCorrector:
    """FC-PASM corrector with the frozen factory knobs (``cast_matrix.py:74-96``).

    Besides the reconstruction it keeps the reference corrector's routing
    state: after a corrected layer whose successor runs the swap router it
    publishes the detached endpoint transport sketch (per target: the
    anchor pair's per-frequency phase ``theta`` and affinity ``g``, both
    ``[18, 11, 6]``) in the format of ``_publish_fc_routing_transport``
    (``proposed/matrix_world_spectral_residual.py:577-658``), read back by
    :meth:`fc_pasm_routing_transport`, and it updates
    ``_fc_previous_mean_affinity`` (``:3667-3669``).  Both come from the
    statistics the PAR kernels already compute, so publishing costs no
    extra kernel work.
    """

    mode = "frequency_confidence_phase_aligned_spectral_mixing"

    def __init__(
        self,
        *,
        fc_tau_low: float = 0.50,
        fc_tau_high: float = 0.75,
        fc_freq_power: float = 2.0,
        fc_temperature: float = 0.03,
        fc_ramp_confidence: bool = True,
        current_anchor_boundary: int = 4,
        record_stats: bool = False,
    ):
        if not 0.0 <= fc_tau_low <= fc_tau_high <= 1.0:
            raise ValueError("FC-PASM thresholds must satisfy 0 <= low <= high <= 1")
        if fc_freq_power <= 0.0 or fc_temperature <= 0.0:
            raise ValueError("FC-PASM frequency power and temperature must be positive")
        if not 1 <= int(current_anchor_boundary) <= 13:
            raise ValueError("current_anchor_boundary must be in [1,13]")
        self.fc_tau_low = float(fc_tau_low)
        self.fc_tau_high = float(fc_tau_high)
        self.fc_freq_power = float(fc_freq_power)
        self.fc_temperature = float(fc_temperature)
        self.fc_ramp_confidence = bool(fc_ramp_confidence)
        self.current_anchor_boundary = int(current_anchor_boundary)
        self.record_stats = bool(record_stats)
        self._chunk = 0
        self._step = 0
        self._records: list[dict] = []
        self._workspace: dict = {}
        self.last_stats: torch.Tensor | None = None
        # routing state (:492, :530, :541): the published sketches by
        # (step, layer), the layers whose successor routes (None: all), and
        # the mean affinity of the last corrected layer
        self._fc_routing_transport: dict = {}
        self._fc_routing_publish_layers: frozenset | None = None
        self._fc_previous_mean_affinity: torch.Tensor | None = None

    def begin_model_call(self, *, geometry=None, chunk_index: int, step_index: int, device=None) -> None:
        """``WorldAlignedSpectralResidualCorrector.begin_model_call`` (``:544-556``)."""
        del geometry, device
        self._chunk = int(chunk_index)
        self._step = int(step_index)
        self._fc_routing_transport.clear()

    def should_publish_fc_routing_transport(self, layer_index: int) -> bool:
        """Whether a router at ``layer_index + 1`` can read this layer's sketch (:532-542)."""
        layers = self._fc_routing_publish_layers
        return layers is None or int(layer_index) in layers

    def fc_pasm_routing_transport(self, *, layer_index: int):
        """The previous layer's sketch in this model call, or None (:660-668)."""
        source = int(layer_index) - 1
        if source < 0:
            return None
        return self._fc_routing_transport.get((int(self._step), source))

    def _publish(self, layer_index, anchors, pairs, stats, h, w):
        # every value below is a view into the statistics the kernels wrote:
        # publishing launches nothing
        theta, affinity = stats_views(stats, len(pairs))
        self._fc_previous_mean_affinity = stats[MEANS_AT + MAX_PAIRS]
        if not self.should_publish_fc_routing_transport(layer_index):
            return
        count = _COUNT_CACHE.get(stats.device)
        if count is None:
            count = torch.full((), TILES * FREQS, dtype=torch.long, device=stats.device)
            _COUNT_CACHE[stats.device] = count
        published = {}
        for i, key in enumerate(pairs):
            published[key] = {
                "theta": theta[i], "affinity": affinity[i], "mean_affinity": stats[MEANS_AT + i],
                "mean_affinity_reduction": "all_tile_frequencies",
                "affinity_support_count": count, "affinity_total_count": TILES * FREQS,
            }
        self._fc_routing_transport[(int(self._step), int(layer_index))] = {
            "source_layer": int(layer_index), "source_step": int(self._step),
            "exact_frames": tuple(int(f) for f in anchors), "tile_grid": (3, 6),
            "output_shape": (int(h), int(w)), "transport_shape": (11, 10),
            "window_shape": (11, 10), "stride": (8, 8), "padding": (4, 5), "pairs": published,
            "detached": True, "endpoint_only": True,
            "transport_formula": "per_frequency_exp(i*g*theta)",
        }

    def _ws(self, device, nbytes: int) -> torch.Tensor:
        buf = self._workspace.get(device)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._workspace[device] = buf
        return buf

    def correct(
        self,
        *,
        layer_index: int,
        full_input: torch.Tensor | None,
        full_residual: torch.Tensor,
        active_residual: torch.Tensor,
        active_frames: torch.Tensor,
        memory_length: int,
        spatial_height: int,
        spatial_width: int,
        coarse_probe_residual: torch.Tensor | None = None,
        active_frame_values: tuple[int, ...] | None = None,
        tile_confidence: torch.Tensor | None = None,
    ) -> torch.Tensor:
        del full_input, coarse_probe_residual
        fallback = None
        if self._chunk == 0:
            fallback = "first_chunk"
        elif memory_length <= 0:
            fallback = "no_memory"
        if fallback is not None:
            self._records.append({"layer_index": int(layer_index), "status": "temporal_fallback",
                                  "fallback_reason": fallback})
            return full_residual
        if full_residual.dim() != 4 or full_residual.shape[0] != 1 or active_residual.shape[0] != 1:
            raise RuntimeError("FC-PASM requires Matrix batch size one")
        for name, t in (("full_residual", full_residual), ("active_residual", active_residual)):
            if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
        if active_frame_values is None:
            active_frame_values = tuple(int(x) for x in active_frames.tolist())
        frames = list(active_frame_values)
        if tuple(sorted(set(frames))) != tuple(frames):
            raise RuntimeError("FC-R active-frame values must be sorted and unique")
        if len(frames) != active_residual.shape[1]:
            raise RuntimeError("active frame count differs from active_residual")
        t_total, hw, c = full_residual.shape[1:]
        if hw != spatial_height * spatial_width:
            raise RuntimeError("residual token count differs from the latent grid")
        anchors = [f - int(memory_length) for f in frames if f >= memory_length]
        targets, pair_of_target, pairs = bracket_targets(
            anchors, t_total - int(memory_length), self.current_anchor_boundary)
        lib = _lib.load()
        nbytes = lib.cast_par_fcpasm_workspace_bytes(t_total, spatial_height, spatial_width, c)
        ws = self._ws(full_residual.device, nbytes)
        frames_arr = (_lib.ctypes.c_int32 * len(frames))(*frames)
        stats = None
        if self.record_stats or targets:
            stats = torch.empty(STATS_FLOATS, dtype=torch.float32, device=full_residual.device)
        if tile_confidence is not None:
            tile_confidence = tile_confidence.to(device=full_residual.device,
                                                 dtype=torch.float32).contiguous()
        _lib.call(
            "cast_par_fcpasm", full_residual.data_ptr(), active_residual.data_ptr(),
            _lib.ctypes.cast(frames_arr, _lib.c_void_p), len(frames), t_total, int(memory_length),
            spatial_height, spatial_width, c, self.fc_tau_low, self.fc_tau_high,
            self.fc_freq_power, self.fc_temperature, int(self.fc_ramp_confidence),
            self.current_anchor_boundary, _lib.ptr(tile_confidence), _lib.ptr(stats), ws.data_ptr(),
            ws.numel(), torch.cuda.current_stream(full_residual.device).cuda_stream,
        )
        self.last_stats = stats
        if targets:
            self._publish(layer_index, anchors, pairs, stats, spatial_height, spatial_width)
        self._records.append({"layer_index": int(layer_index), "status": "corrected",
                              "target_frames": targets,
                              "target_anchor_pairs": [list(pairs[i]) for i in pair_of_target]})
        return full_residual


def stats_views(stats: torch.Tensor, n_pairs: int):
    """``theta`` and affinity ``g`` of every anchor pair, ``[n_pairs, 18, 11, 6]``
    views into the statistics block (no copy, no synchronisation)."""
    blk = stats[: n_pairs * STATS_PER_PAIR].view(n_pairs, STATS_PER_PAIR)
    theta = blk[:, : TILES * FREQS].view(n_pairs, TILES, 11, 6)
    g0 = TILES * FREQS + TILES
    affinity = blk[:, g0: g0 + TILES * FREQS].view(n_pairs, TILES, 11, 6)
    return theta, affinity


def unpack_stats(stats: torch.Tensor, n_pairs: int) -> list[dict]:
    """Splits the per-pair statistics block (written whenever a call has targets)."""
    per = STATS_PER_PAIR
    out = []
    for i in range(n_pairs):
        s = stats[i * per:(i + 1) * per]
        o = 0
        theta = s[o:o + TILES * FREQS].view(TILES, 11, 6); o += TILES * FREQS
        conf = s[o:o + TILES]; o += TILES
        g = s[o:o + TILES * FREQS].view(TILES, 11, 6); o += TILES * FREQS
        disp = s[o:o + 2 * TILES].view(TILES, 2); o += 2 * TILES
        base = s[o:o + TILES]; o += TILES
        ramp = s[o:o + TILES]
        out.append({"theta": theta, "confidence": conf, "affinity": g, "displacement": disp,
                    "base_confidence": base, "ramp_confidence": ramp})
    return out
