"""CPU oracle for the CAST RCSA/PAR hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package (``cast_b200``) imports this package.  Only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker or
as the timed CPU baseline -- never as the thing measured on the GPU.

Modules:

* ``oracle.rcsa``  -- pooled-QK block scoring, top-k block selection, the
  per-block symmetric int8 quantiser, and block-sparse attention (bf16 path and
  exact int8 simulation).  Restated from
  ``proposed/qk_uncertainty_tangent_attention.py:988-1082``,
  ``proposed/reciprocal_joint_attention.py:64-103``,
  ``proposed/matrix_curvature_phase_frame_weave.py:5677-5831`` and the sampled
  softmax oracle ``proposed/matrix_jit_spatial_acceleration.py:821-877``.
* ``oracle.par``   -- Phase-Aware Reconstruction (FC-PASM reference numerics),
  restated from ``proposed/matrix_world_spectral_residual.py:1836-3662``.

Pinning: the restatements are checked against golden vectors produced by the
reference's own code (``tests/golden/make_golden.py``), except where the
reference has no implementation: the int8 quantiser (no reference function)
and the external ``_attn_fwd_bsa_align`` kernel (not vendored; its
restatement follows the reference's sampled explicit-softmax oracle).  Those
two are marked "parity unpinned by the reference" and are pinned only by this
repository's own golden vectors.
"""
