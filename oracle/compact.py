"""CPU restatement of the compact-layout packing with the RoPE phase.

TEST INFRASTRUCTURE ONLY: the checker for ``cast_compact_pack`` /
``cast_compact_unpack``; nothing in the product imports it.

Follows, in numpy:

* ``MatrixCurvaturePhaseFrameWeave._apply_compact_rope_phase``
  (``proposed/matrix_curvature_phase_frame_weave.py:5565-5574``): the
  (even, odd) pairs of ``value.float()`` times the complex64 phase, each
  product and sum rounded in fp32 (a complex64 multiply);
* the packing of ``_compact_cwca_attention`` (:5677-5684): gather by the
  clamped block indices, transpose to ``[B,H,P,D]``, zero the padding; then
  the bf16 cast of the attention launch
  (``proposed/matrix_jit_spatial_acceleration.py:679-681``);
* the output scatter ``output_packed[:, token_to_packed]`` (:6095).

Pinned by ``tests/golden/compact_pack.npz``, made by running those
reference functions and lines (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def apply_rope_phase(value: np.ndarray, phase_re: np.ndarray, phase_im: np.ndarray) -> np.ndarray:
    """value fp32 [B,L,H,D]; phase [L,Hp,D/2] (Hp = 1 or H) -> fp32 [B,L,H,D]."""
    b, l, h, d = value.shape
    x = value.astype(np.float32).reshape(b, l, h, d // 2, 2)
    a, bb = x[..., 0], x[..., 1]
    c = phase_re.astype(np.float32)[None]
    s = phase_im.astype(np.float32)[None]
    re = (a * c).astype(np.float32) - (bb * s).astype(np.float32)
    im = (a * s).astype(np.float32) + (bb * c).astype(np.float32)
    return np.stack([re.astype(np.float32), im.astype(np.float32)], axis=-1).reshape(b, l, h, d)


def pack(q, k, v, block_indices, phase_re=None, phase_im=None):
    """q/k/v fp32 values [B,L,H,D]; block_indices int [P] (-1 padding).

    Returns bf16 bit patterns ``[B,H,P,D]`` for q, k and v.
    """
    if phase_re is not None:
        q = apply_rope_phase(q, phase_re, phase_im)
        k = apply_rope_phase(k, phase_re, phase_im)
    idx = np.asarray(block_indices).reshape(-1)
    flat = np.maximum(idx, 0)
    mask = idx >= 0
    out = []
    for x in (q, k, v):
        p = x[:, flat].transpose(0, 2, 1, 3).astype(np.float32).copy()
        p[:, :, ~mask] = 0.0
        out.append(bf16_bits(p))
    return tuple(out)


def unpack(packed_bits: np.ndarray, token_to_packed: np.ndarray) -> np.ndarray:
    """bf16 bits [B,H,P,D] -> [B,L,H,D] in token order."""
    return packed_bits.transpose(0, 2, 1, 3)[:, np.asarray(token_to_packed)]


def stable_layout(block_id: np.ndarray, n_blocks: int, block_size: int):
    """Packed slots of a compact layout: tokens grouped by block id in token
    order (the stable grouping of ``proposed/matrix_curvature_phase_frame_
    weave.py:5269-5289``).  Returns (block_indices [n_blocks, block_size]
    with -1 padding, token_to_packed [L])."""
    order = np.argsort(block_id, kind="stable")
    counts = np.bincount(block_id, minlength=n_blocks)
    assert (counts <= block_size).all()
    starts = np.cumsum(counts) - counts
    ranks = np.arange(order.size) - np.repeat(starts, counts)
    flat_pos = block_id[order] * block_size + ranks
    block_indices = np.full(n_blocks * block_size, -1, dtype=np.int64)
    block_indices[flat_pos] = order
    token_to_packed = np.empty(block_id.size, dtype=np.int64)
    token_to_packed[order] = flat_pos
    return block_indices.reshape(n_blocks, block_size), token_to_packed


def compact_rope_phase(coords, freqs, memory_length, memory_latent_idx, predict_latent_idx):
    """The per-token RoPE phase of a compact layout
    (``proposed/matrix_curvature_phase_frame_weave.py:5484-5563``): the
    temporal coordinate remapped to the memory / prediction latent indices,
    then the (t, h, w) axes of the frequency table (split 22/21/21 of the 64
    pairs) gathered and concatenated.  ``freqs`` complex ``[pos, 64]`` ->
    ``[L, 1, 64]``, or ``[H, pos, 64]`` -> ``[L, H, 64]``."""
    coords = np.asarray(coords)
    freqs = np.asarray(freqs)
    half = 64
    split = [half - 2 * (half // 3), half // 3, half // 3]
    bounds = np.cumsum([0] + split)
    raw_t = coords[:, 0]
    mem = np.asarray(memory_latent_idx, dtype=np.int64)
    pred_lo, pred_hi = predict_latent_idx
    pred = np.arange(pred_lo, pred_hi, dtype=np.int64)
    temporal = np.where(raw_t < memory_length, mem[np.minimum(raw_t, len(mem) - 1)],
                        pred[np.clip(raw_t - memory_length, 0, len(pred) - 1)])
    index = (temporal, coords[:, 1], coords[:, 2])
    parts = []
    for a, idx in enumerate(index):
        if freqs.ndim == 3:
            parts.append(freqs[:, idx, bounds[a]:bounds[a + 1]].transpose(1, 0, 2))
        else:
            parts.append(freqs[idx, bounds[a]:bounds[a + 1]][:, None, :])
    return np.concatenate(parts, axis=-1).astype(np.complex64)
