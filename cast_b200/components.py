"""Drop-in integration with the CAST reference package.

``make_cast_components()`` returns the reference's own frozen component
triple (``src/interaction_accel/cast_matrix.py:24-107``) with the hot path
swapped for the B200 kernels, so ``frame_weave.install(model)`` and the
Matrix DiT attention hook keep their call signatures.  Seams replaced (every
one routes CUDA tensors to the kernels; CPU tensors keep the reference's own
code, and :func:`patched_seams` lists what is installed):

* ``MatrixJiTSpatialAcceleration._longcat_active`` and
  ``MatrixCausalFrameLayerRelay._longcat_asymmetric`` (the block-sparse
  attention launch seams) -> :func:`cast_b200.rcsa.longcat_active` /
  :func:`cast_b200.rcsa.longcat_asymmetric`;
* ``MatrixTrajectoryAdaptiveBudgetAttentionCompiler.select`` (TABA pooled-QK
  selection, ``proposed/qk_uncertainty_tangent_attention.py:988-1082``, which
  the factory's attention compiler reaches through ``super().select``) ->
  :class:`cast_b200.select.TABASelector` given the compiler's compiled row
  degrees, with the reference's checks, certificate and report;
* the frame weave's ``direct_control_barycentric_pair_write`` (the
  control-barycentric lift's two-anchor writer) ->
  :func:`cast_b200.barycentric.direct_control_barycentric_pair_write`;
* ``MatrixCurvaturePhaseFrameWeave._control_barycentric_residual_lift`` (the
  whole lift: camera / action state, every target's weights, the rows) ->
  :func:`cast_b200.barycentric.control_barycentric_residual_lift` for batch-1
  fp32 residuals;
* the weave's ``world_spectral_corrector.correct`` (FC-PASM reference
  numerics) -> :class:`cast_b200.par.FCPASMCorrector` with the corrector's
  own FC knobs; it publishes the FC routing transport into the reference
  corrector's own cache, so the weave's swap router reads it;
* the weave's ``fc_pasm_swap_router.refine`` ->
  :class:`cast_b200.swap_router.FCPASMLocalCoordinateSwapRouter`;
* ``MatrixCurvaturePhaseFrameWeave._compact_cwca_attention`` (the compact
  layers' packing, pooled-Q/K ranking, block-sparse attention and scatter) ->
  :func:`cast_b200.compact_attention.compact_cwca_attention`, with the QK^T
  precision policy given to :func:`make_cast_components` (``"auto"``: int8
  QK^T where its predicted logit error stays below the tolerance); on the
  router's layers the reference's method keeps the ranking and hands it to
  the B200 router and attention.

The reference package itself (its orchestration, CAFS, degree budgets, the
memory compiler) is not part of this repository; it is imported from the
caller's environment.
"""

from __future__ import annotations

import importlib
import math

import torch

from . import _lib, barycentric, compact_attention, rcsa, swap_router
from .par import FCPASMCorrector
from .select import TABASelector

_PATCHED: dict = {}
# QK^T precision of the compact layers' attention (make_cast_components)
_SETTINGS = {"precision": "auto", "int8_tolerance": rcsa.DEFAULT_INT8_TOLERANCE}

# FC knobs of the reference corrector that change its arithmetic, with the
# value the B200 path implements (the factory's, cast_matrix.py:74-96).  A
# corrector configured otherwise keeps the reference's own ``correct``.
_FC_KNOBS = {
    "fc_reference_numerics": True, "fc_lean_runtime": True, "fc_fused_complex_weights": True,
    "fc_temporal_consistency": False, "fc_trust_eta": 0.0, "fc_layer_gate_threshold": -1.0,
    "fc_pair_gate_threshold": -1.0, "fc_transport_tile_topk": 0, "fc_zero_transport_fastpath": False,
    "fc_v21_bypass": False, "fc_v21_blend": 0.0, "fc_coarse_transport": False,
    "fc_legacy_lowfreq_index_bug": False, "fc_triton_phase_mix": False,
    "fc_triton_accurate_phase_mix": False, "fc_triton_batched_mix": False,
    "fc_triton_phat_peak": False, "fc_triton_ramp_confidence": False,
    "fc_triton_reference_lowfreq": False,
}


def _ref(name: str):
    try:
        return importlib.import_module(f"interaction_accel.methods.proposed.{name}")
    except ImportError as exc:  # pragma: no cover - depends on the caller's env
        raise ImportError(
            "the CAST reference package (interaction_accel) must be importable to use "
            "make_cast_components(); the kernels themselves are in cast_b200.rcsa/par"
        ) from exc


def _taba_select(self, q, k, *, geometry_indices, geometry_counts, latent_hw, block_shape):
    """``MatrixTrajectoryAdaptiveBudgetAttentionCompiler.select`` on the B200
    for CUDA tensors: the reference's argument checks (:999-1009), the CUDA
    pooled-QK selection given ``self._row_degrees``, the selection
    certificate (:1047-1061) and the reference's report (:1063-1082)."""
    if not (q.is_cuda and k.is_cuda):
        return _PATCHED["taba_select"](self, q, k, geometry_indices=geometry_indices,
                                       geometry_counts=geometry_counts, latent_hw=latent_hw,
                                       block_shape=block_shape)
    qk = _ref("qk_uncertainty_tangent_attention")
    if q.shape != k.shape or q.ndim != 4:
        raise ValueError("TABA requires equal B,H,L,D Q/K")
    if self._row_degrees is None or self._ray_motion is None:
        raise RuntimeError("TABA budgets were not compiled")
    if tuple(int(v) for v in block_shape) != self._block_shape:
        raise RuntimeError("TABA runtime block shape differs from compilation")
    fixed = geometry_counts[0, 0].detach().to("cpu", torch.long)
    if fixed.numel() != self._num_blocks or not torch.all(fixed == self._degree):
        raise RuntimeError("TABA baseline layout does not have fixed K")
    degrees = self._row_degrees
    cached = getattr(self, "_cast_b200_taba", None)
    if cached is None or cached[0] is not degrees:
        sel = TABASelector(self._block_shape)
        sel.set_row_degrees(degrees)
        cached = (degrees, sel)
        self._cast_b200_taba = cached
    selected, counts, _, scores = cached[1].select(
        q, k, geometry_indices=None, geometry_counts=None, latent_hw=latent_hw,
        block_shape=block_shape, return_scores=True)
    # the certificate: no repeated block in a row, every stencil block kept
    batch, heads, n, maxdeg = selected.shape
    height, width = (int(v) for v in latent_hw)
    _, th, tw = self._block_shape
    nh, nw = math.ceil(height / th), math.ceil(width / tw)
    ids = torch.arange(n, device=q.device)
    t_id, h_id, w_id = ids // (nh * nw), (ids % (nh * nw)) // nw, ids % nw
    local = ((t_id[:, None] - t_id[None]).abs() + (h_id[:, None] - h_id[None]).abs()
             + (w_id[:, None] - w_id[None]).abs()) <= 1
    valid = torch.arange(maxdeg, device=q.device)[None, None, None] < counts[..., None]
    sel64 = selected.long()
    duplicates = int(torch.count_nonzero((sel64[..., 1:] == sel64[..., :-1]) & valid[..., 1:]).item())
    chosen = torch.gather(local[None, None].expand(batch, heads, -1, -1), -1, sel64) & valid
    expected = int(local.sum().item()) * batch * heads
    missing = expected - int(chosen.sum().item())
    _lib.check_device(torch.cuda.current_stream(q.device).cuda_stream, "cast_taba_select")
    if duplicates or missing:
        raise RuntimeError("TABA selection certificate failed")
    report = qk.QKUncertaintyTangentSelectionReport(
        batch_heads=batch * heads, query_rows=self._num_blocks, edges_per_row=self._degree,
        row_duplicate_violations=duplicates, selected_orientation_violations=0,
        max_orientation_violations_per_row=0, mean_selected_ray_cosine=0.0,
        mean_selected_qk_cosine=float(scores.mean().item()), qk_read_for_selection=True,
        selector_count=1, protected_local_edges=expected, missing_local_edges=missing,
        mean_geometry_gate=0.0, max_geometry_gate=0.0, budget_min=int(degrees.min().item()),
        budget_max=int(degrees.max().item()), budget_total=int(degrees.sum().item()),
        mean_ray_motion=float(self._ray_motion.mean().item()),
        max_ray_motion=float(self._ray_motion.max().item()),
        trajectory_complexity_kind=self.trajectory_complexity_kind,
        mean_first_order_motion=float(self._first_order_motion.mean().item()),
    )
    return selected, counts, report


def _compact_cwca(self, module, q, k, v, layout):
    """``MatrixCurvaturePhaseFrameWeave._compact_cwca_attention`` on the B200."""
    original = _PATCHED["compact_cwca"].__get__(self, type(self))
    return compact_attention.compact_cwca_attention(
        self, module, q, k, v, layout, original=original, policy=_SETTINGS["precision"],
        int8_tolerance=_SETTINGS["int8_tolerance"])


def _lift(cls, active_residual, active_frames, total_temporal, memory_temporal, current_segment_boundary,
          full_plucker, *args, **kwargs):
    """``MatrixCurvaturePhaseFrameWeave._control_barycentric_residual_lift``
    on the B200 for batch-1 fp32 CUDA residuals; other inputs keep the
    reference's method."""
    if (isinstance(active_residual, torch.Tensor) and active_residual.is_cuda
            and active_residual.dtype == torch.float32 and active_residual.ndim == 4
            and active_residual.shape[0] == 1 and isinstance(full_plucker, torch.Tensor)
            and full_plucker.device == active_residual.device):
        return barycentric.control_barycentric_residual_lift(
            active_residual, active_frames, total_temporal, memory_temporal, current_segment_boundary,
            full_plucker, *args, **kwargs)
    return _PATCHED["lift"](
        cls, active_residual, active_frames, total_temporal, memory_temporal, current_segment_boundary,
        full_plucker, *args, **kwargs)


def install_kernels() -> None:
    """Replaces the reference's static seams: the attention launches, the
    TABA selection, the compact CWCA attention, the pair writer and the
    control-barycentric lift (idempotent)."""
    jit = _ref("matrix_jit_spatial_acceleration")
    weave = _ref("matrix_curvature_phase_frame_weave")
    qk = _ref("qk_uncertainty_tangent_attention")
    if "longcat_active" not in _PATCHED:
        _PATCHED["longcat_active"] = jit.MatrixJiTSpatialAcceleration._longcat_active
        jit.MatrixJiTSpatialAcceleration._longcat_active = staticmethod(rcsa.longcat_active)
    if "longcat_asymmetric" not in _PATCHED:
        _PATCHED["longcat_asymmetric"] = weave.MatrixCausalFrameLayerRelay._longcat_asymmetric
        weave.MatrixCausalFrameLayerRelay._longcat_asymmetric = staticmethod(rcsa.longcat_asymmetric)
    if "pair_write" not in _PATCHED:
        # the weave calls the writer through its own module-level name
        _PATCHED["pair_write"] = weave.direct_control_barycentric_pair_write
        weave.direct_control_barycentric_pair_write = barycentric.direct_control_barycentric_pair_write
    if "taba_select" not in _PATCHED:
        cls = qk.MatrixTrajectoryAdaptiveBudgetAttentionCompiler
        _PATCHED["taba_select"] = cls.select
        cls.select = _taba_select
    if "compact_cwca" not in _PATCHED:
        _PATCHED["compact_cwca"] = weave.MatrixCurvaturePhaseFrameWeave._compact_cwca_attention
        weave.MatrixCurvaturePhaseFrameWeave._compact_cwca_attention = _compact_cwca
    if "lift" not in _PATCHED:
        cls = weave.MatrixCurvaturePhaseFrameWeave
        # the undecorated function of the classmethod, rebound per call
        _PATCHED["lift"] = cls.__dict__["_control_barycentric_residual_lift"].__func__
        cls._control_barycentric_residual_lift = classmethod(_lift)


def uninstall_kernels() -> None:
    """Restores the reference's original seams."""
    if "longcat_active" in _PATCHED:
        jit = _ref("matrix_jit_spatial_acceleration")
        jit.MatrixJiTSpatialAcceleration._longcat_active = staticmethod(_PATCHED.pop("longcat_active"))
    if "longcat_asymmetric" in _PATCHED:
        weave = _ref("matrix_curvature_phase_frame_weave")
        weave.MatrixCausalFrameLayerRelay._longcat_asymmetric = staticmethod(
            _PATCHED.pop("longcat_asymmetric"))
    if "pair_write" in _PATCHED:
        weave = _ref("matrix_curvature_phase_frame_weave")
        weave.direct_control_barycentric_pair_write = _PATCHED.pop("pair_write")
    if "taba_select" in _PATCHED:
        qk = _ref("qk_uncertainty_tangent_attention")
        qk.MatrixTrajectoryAdaptiveBudgetAttentionCompiler.select = _PATCHED.pop("taba_select")
    if "compact_cwca" in _PATCHED:
        weave = _ref("matrix_curvature_phase_frame_weave")
        weave.MatrixCurvaturePhaseFrameWeave._compact_cwca_attention = _PATCHED.pop("compact_cwca")
    if "lift" in _PATCHED:
        weave = _ref("matrix_curvature_phase_frame_weave")
        weave.MatrixCurvaturePhaseFrameWeave._control_barycentric_residual_lift = classmethod(
            _PATCHED.pop("lift"))


def unsupported_fc_knob(ref_corrector) -> str | None:
    """The first FC knob of a reference corrector that the B200 path does not
    implement (None when it runs the factory's FC-PASM path)."""
    if getattr(ref_corrector, "mode", None) != FCPASMCorrector.mode:
        return "mode"
    for name, want in _FC_KNOBS.items():
        if getattr(ref_corrector, name, want) != want:
            return name
    return None


def corrector_from_reference(ref_corrector) -> FCPASMCorrector:
    """An FC-PASM corrector carrying a reference corrector's FC knobs."""
    return FCPASMCorrector(
        fc_tau_low=ref_corrector.fc_tau_low, fc_tau_high=ref_corrector.fc_tau_high,
        fc_freq_power=ref_corrector.fc_freq_power, fc_temperature=ref_corrector.fc_temperature,
        fc_ramp_confidence=ref_corrector.fc_ramp_confidence,
        current_anchor_boundary=ref_corrector.current_anchor_boundary,
    )


def attach(weave) -> None:
    """Routes a reference weave's FC-PASM corrections through the B200 kernels.

    The reference corrector keeps its bookkeeping (``begin_model_call``, the
    layer schedule and the causal V21 switch, records); only the correction
    itself runs on the kernels, for CUDA residuals under the factory's knobs.
    The B200 corrector shares the reference corrector's routing cache, so the
    transport sketch it publishes is the one ``fc_pasm_routing_transport``
    hands to the swap router, and it keeps ``_fc_previous_mean_affinity``
    current.  Calls that stay on the reference's code are counted in
    ``ref._cast_b200_reference_calls`` by reason.
    """
    ref = getattr(weave, "world_spectral_corrector", None)
    if ref is None or getattr(ref, "_cast_b200", False):
        return
    fast = corrector_from_reference(ref)
    fast._fc_routing_transport = ref._fc_routing_transport  # cleared in place per model call
    original = ref.correct
    unsupported = unsupported_fc_knob(ref)
    ref._cast_b200_reference_calls = {}

    def correct(**kwargs):
        layer = int(kwargs["layer_index"])
        reason = unsupported
        if reason is None and not kwargs["full_residual"].is_cuda:
            reason = "host_tensors"
        if reason is None and (ref.fc_active_layers and layer not in ref.fc_active_layers):
            reason = "layer_schedule_bypass"      # the reference returns at once (:5297-5307)
        if reason is None and not ref._fc_runtime_active:
            reason = "causal_v21_bypass"          # likewise (:5308-5327)
        if reason is not None:
            ref._cast_b200_reference_calls[reason] = ref._cast_b200_reference_calls.get(reason, 0) + 1
            return original(**kwargs)
        fast._chunk = ref._chunk
        fast._step = ref._step
        fast._fc_routing_publish_layers = getattr(ref, "_fc_routing_publish_layers", None)
        out = fast.correct(**kwargs)
        record = dict(fast._records[-1])
        if record["status"] == "corrected":
            ref._fc_previous_mean_affinity = fast._fc_previous_mean_affinity
        record.update(chunk_index=ref._chunk, step_index=ref._step, mode=ref.mode, backend="cast_b200")
        ref._records.append(record)
        return out

    ref.correct = correct
    ref._cast_b200_original_correct = original
    ref._cast_b200 = True
    attach_router(weave)


def attach_router(weave) -> None:
    """Runs a reference weave's FC-PASM swap routing (its
    ``fc_pasm_swap_router``, built at proposed/matrix_curvature_phase_frame_
    weave.py:585-604 and called at :6040) through ``cast_swap_route`` for
    CUDA tensors; the router keeps the reference's config object."""
    ref = getattr(weave, "fc_pasm_swap_router", None)
    if ref is None or getattr(ref, "_cast_b200", False):
        return
    fast = swap_router.FCPASMLocalCoordinateSwapRouter(ref.config)
    original = ref.refine

    def refine(**kwargs):
        if not kwargs["score"].is_cuda:
            return original(**kwargs)
        selected, record = fast.refine(**kwargs)
        ref._records.append(record)
        return selected, record

    ref.refine = refine
    ref._cast_b200 = True


def patched_seams(weave=None) -> dict:
    """Which reference seams currently route to the B200 kernels."""
    jit = _ref("matrix_jit_spatial_acceleration")
    wv = _ref("matrix_curvature_phase_frame_weave")
    qk = _ref("qk_uncertainty_tangent_attention")
    out = {
        "longcat_active": jit.MatrixJiTSpatialAcceleration._longcat_active is rcsa.longcat_active,
        "longcat_asymmetric": wv.MatrixCausalFrameLayerRelay._longcat_asymmetric is rcsa.longcat_asymmetric,
        "pair_write": wv.direct_control_barycentric_pair_write is barycentric.direct_control_barycentric_pair_write,
        "taba_select": qk.MatrixTrajectoryAdaptiveBudgetAttentionCompiler.select is _taba_select,
        "compact_cwca": wv.MatrixCurvaturePhaseFrameWeave._compact_cwca_attention is _compact_cwca,
        "lift": wv.MatrixCurvaturePhaseFrameWeave.__dict__["_control_barycentric_residual_lift"].__func__
        is _lift,
    }
    if weave is not None:
        out["correct"] = bool(getattr(getattr(weave, "world_spectral_corrector", None), "_cast_b200", False))
        out["refine"] = bool(getattr(getattr(weave, "fc_pasm_swap_router", None), "_cast_b200", False))
    return out


def make_cast_components(*, precision: str = "auto",
                         int8_tolerance: float = rcsa.DEFAULT_INT8_TOLERANCE):
    """``make_cast_components()`` with the B200 hot path installed.

    ``precision`` is the compact layers' QK^T policy: ``"auto"`` (int8 where
    the predicted logit error of the int8 product stays below
    ``int8_tolerance``, bf16 elsewhere), ``"bf16"`` (the reference's numerics)
    or ``"int8"``."""
    if precision not in rcsa.POLICIES:
        raise ValueError(f"precision must be one of {sorted(rcsa.POLICIES)}")
    _SETTINGS.update(precision=precision, int8_tolerance=float(int8_tolerance))
    factory = importlib.import_module("interaction_accel.cast_matrix")
    install_kernels()
    memory, attention, weave = factory.make_cast_components()
    attach(weave)
    return memory, attention, weave


__all__ = [
    "make_cast_components", "install_kernels", "uninstall_kernels", "attach", "attach_router",
    "corrector_from_reference", "unsupported_fc_knob", "patched_seams", "TABASelector",
]
