"""Drop-in integration with the CAST reference package.

``make_cast_components()`` returns the reference's own frozen component
triple (``src/interaction_accel/cast_matrix.py:24-107``) with the hot path
swapped for the B200 kernels, so ``frame_weave.install(model)`` and the
Matrix DiT attention hook keep their call signatures:

* ``MatrixJiTSpatialAcceleration._longcat_active`` and
  ``MatrixCausalFrameLayerRelay._longcat_asymmetric`` (the block-sparse
  attention launch seams) -> :func:`cast_b200.rcsa.longcat_active` /
  :func:`cast_b200.rcsa.longcat_asymmetric`;
* the weave's ``world_spectral_corrector.correct`` (FC-PASM reference
  numerics) -> :class:`cast_b200.par.FCPASMCorrector` with the corrector's
  own FC knobs;
* ``attention_compiler.select`` (TABA pooled-QK selection) -> the CUDA
  selection given the compiler's compiled row degrees;
* the frame weave's ``direct_control_barycentric_pair_write`` (the
  control-barycentric lift's two-anchor writer) ->
  :func:`cast_b200.barycentric.direct_control_barycentric_pair_write`.

The reference package itself (its orchestration, CAFS, degree budgets, the
memory compiler) is not part of this repository; it is imported from the
caller's environment.
"""

from __future__ import annotations

import importlib

from . import barycentric, rcsa, swap_router
from .par import FCPASMCorrector
from .select import TABASelector

_PATCHED: dict = {}


def _ref(name: str):
    try:
        return importlib.import_module(f"interaction_accel.methods.proposed.{name}")
    except ImportError as exc:  # pragma: no cover - depends on the caller's env
        raise ImportError(
            "the CAST reference package (interaction_accel) must be importable to use "
            "make_cast_components(); the kernels themselves are in cast_b200.rcsa/par"
        ) from exc


def install_kernels() -> None:
    """Replaces the reference's static attention launch seams (idempotent)."""
    jit = _ref("matrix_jit_spatial_acceleration")
    weave = _ref("matrix_curvature_phase_frame_weave")
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


def uninstall_kernels() -> None:
    """Restores the reference's original launch seams."""
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

    The reference corrector keeps its bookkeeping (``begin_model_call``,
    records); only ``correct`` is replaced, for the FC-PASM mode with the
    factory's lean reference-numerics knobs.
    """
    ref = getattr(weave, "world_spectral_corrector", None)
    if ref is None:
        return
    fast = corrector_from_reference(ref)
    original = ref.correct

    def correct(**kwargs):
        if ref.mode != FCPASMCorrector.mode or not kwargs["full_residual"].is_cuda:
            return original(**kwargs)
        fast._chunk = ref._chunk
        fast._step = ref._step
        return fast.correct(**kwargs)

    ref.correct = correct
    ref._cast_b200_original_correct = original
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


def make_cast_components():
    """``make_cast_components()`` with the B200 hot path installed."""
    factory = importlib.import_module("interaction_accel.cast_matrix")
    install_kernels()
    memory, attention, weave = factory.make_cast_components()
    attach(weave)
    return memory, attention, weave


__all__ = [
    "make_cast_components", "install_kernels", "uninstall_kernels", "attach", "attach_router",
    "corrector_from_reference", "TABASelector",
]
