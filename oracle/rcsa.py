"""CPU restatement of the RCSA hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA kernels in ``cast_b200/csrc``.  It is
never imported by the product package.

Arithmetic contract shared with the CUDA kernels (so that block indices and
int8 codes can be compared bit-exactly):

* Block sums: row ``r`` of a block goes to partial ``r % SUM_LANES``; each
  partial accumulates its rows in increasing order in float32 (correctly
  rounded IEEE float32 adds, starting from 0), then the partials are widened
  to float64 and added in order ``0..SUM_LANES-1`` (IEEE float64 adds).
* Pooled vectors follow ``F.normalize(mean, dim=-1)``
  (``proposed/qk_uncertainty_tangent_attention.py:1021-1022``):
  ``mean = sum / count``; ``ss = lane_tree_sum(mean*mean)``;
  ``n = mean / max(sqrt(ss), 1e-12)``.
* Scores are ``lane_tree_sum(qn * kn)`` in float64
  (``proposed/qk_uncertainty_tangent_attention.py:1023``).
* ``lane_tree_sum`` over D dims (D a multiple of 32): lane ``l`` of 32 sums
  the products of dims ``l, l+32, ...`` in increasing order, then the 32 lane
  values are combined by an xor-butterfly over distances 16, 8, 4, 2, 1.
  Every multiply and add is a separately rounded IEEE float64 operation.
* The reference computes these quantities in float32; float64 with a fixed
  order is used here so that selection is reproducible on any device.  The
  reference's float32 result agrees except at score near-ties (gap below
  ~1e-6), which ``tests/`` report with the gap.
* int8 quantiser (defined by this project; the reference has none):
  ``s = amax/127`` in float32 (``s = 1`` if ``amax == 0``),
  ``code = clip(rint_half_even(x / s), -127, 127)`` with IEEE float32 division.
"""

from __future__ import annotations

import math

import numpy as np

SUM_LANES = 16
NORM_EPS = 1e-12
LOCAL_BONUS = 1.0e6

CAUSAL_NONE = 0
CAUSAL_BLOCK = 1


# ---------------------------------------------------------------------------
# block geometry
# ---------------------------------------------------------------------------


def contiguous_block_index(length: int, block_size: int) -> np.ndarray:
    """Token index of every (block, row) for packed contiguous blocks.

    Rows past ``length`` are -1 (padding).  This is the packed layout the
    launch seam receives (``proposed/matrix_jit_spatial_acceleration.py:663-729``).
    """
    nb = -(-length // block_size)
    idx = np.arange(nb * block_size, dtype=np.int64).reshape(nb, block_size)
    idx[idx >= length] = -1
    return idx


def grid_block_index(
    temporal: int, height: int, width: int, block_shape: tuple[int, int, int]
) -> np.ndarray:
    """Token index of every (block, row) in ``_tile_visual_tensor`` order.

    Follows ``proposed/reciprocal_joint_attention.py:64-103``: the visual grid
    ``[T,H,W]`` is zero-padded up to multiples of ``(tt,th,tw)`` and blocks are
    enumerated ``(t,h,w)`` block-major, rows ``(t,h,w)`` within a block.
    Padding rows are -1 (they contribute zeros but count in the mean).
    """
    tt, th, tw = block_shape
    nt, nh, nw = -(-temporal // tt), -(-height // th), -(-width // tw)
    out = np.full((nt * nh * nw, tt * th * tw), -1, dtype=np.int64)
    for bt in range(nt):
        for bh in range(nh):
            for bw in range(nw):
                b = (bt * nh + bh) * nw + bw
                r = 0
                for it in range(tt):
                    for ih in range(th):
                        for iw in range(tw):
                            t, h, w = bt * tt + it, bh * th + ih, bw * tw + iw
                            if t < temporal and h < height and w < width:
                                out[b, r] = (t * height + h) * width + w
                            r += 1
    return out


# ---------------------------------------------------------------------------
# pooled block statistics + int8 quantiser
# ---------------------------------------------------------------------------


def block_sums(x: np.ndarray, index: np.ndarray, valid: np.ndarray | None = None):
    """Per-block sums with the interleaved fixed order (float32 partials,
    float64 combination; see the module docstring).

    ``x``: ``[..., L, D]`` float32 holding bf16-representable values.
    ``index``: ``[NB, S]`` token index per row (-1 = padding).
    ``valid``: optional ``[L]`` bool; invalid tokens are treated as zero and do
    not count (``proposed/matrix_curvature_phase_frame_weave.py:5696-5699``).
    Returns ``(sums [..., NB, D] f64, count [NB] int)``.
    """
    lead = x.shape[:-2]
    nb, s = index.shape
    d = x.shape[-1]
    x32 = x.astype(np.float32)
    rows = -(-s // SUM_LANES) * SUM_LANES
    gathered = np.zeros(lead + (nb, rows, d), dtype=np.float32)
    ok = index >= 0
    if valid is not None:
        ok = ok & np.where(index >= 0, valid[np.clip(index, 0, None)], False)
    safe = np.clip(index, 0, None)
    g = x32[..., safe.reshape(-1), :].reshape(lead + (nb, s, d))
    g = np.where(ok[..., None], g, np.float32(0.0))
    gathered[..., :s, :] = g
    partial = np.zeros(lead + (nb, SUM_LANES, d), dtype=np.float32)
    for step in range(rows // SUM_LANES):
        partial = partial + gathered[..., step * SUM_LANES:(step + 1) * SUM_LANES, :]
    wide = partial.astype(np.float64)
    total = wide[..., 0, :].copy()
    for p in range(1, SUM_LANES):
        total = total + wide[..., p, :]
    count = ok.sum(axis=1)
    return total, count


def lane_tree_sum(prod: np.ndarray) -> np.ndarray:
    """Sum over the last axis in the CUDA warp order (see module docstring)."""
    d = prod.shape[-1]
    if d % 32:
        raise ValueError("lane_tree_sum needs a multiple of 32 dims")
    part = prod[..., 0:32].copy()
    for j in range(1, d // 32):
        part = part + prod[..., 32 * j:32 * j + 32]
    lanes = np.arange(32)
    for s in (16, 8, 4, 2, 1):
        part = part + part[..., lanes ^ s]
    return part[..., 0]


def pooled_normalized(sums: np.ndarray, count_denominator: np.ndarray) -> np.ndarray:
    """``F.normalize(sum/count)`` in float64 with the fixed operation order."""
    den = np.maximum(count_denominator, 1).astype(np.float64)
    mean = sums / den[:, None]
    ss = lane_tree_sum(mean * mean)
    norm = np.maximum(np.sqrt(ss), NORM_EPS)
    return mean / norm[..., None]


def block_amax(x: np.ndarray, index: np.ndarray, valid: np.ndarray | None = None):
    """Per-block max |x| over valid rows, float32."""
    lead = x.shape[:-2]
    nb, s = index.shape
    ok = index >= 0
    if valid is not None:
        ok = ok & np.where(index >= 0, valid[np.clip(index, 0, None)], False)
    safe = np.clip(index, 0, None)
    g = np.abs(x[..., safe.reshape(-1), :].reshape(lead + (nb, s, x.shape[-1])))
    g = np.where(ok[..., None], g, 0.0)
    return g.max(axis=(-1, -2)).astype(np.float32)


def quant_scale(amax: np.ndarray) -> np.ndarray:
    amax = amax.astype(np.float32)
    s = amax / np.float32(127.0)
    return np.where(amax > 0, s, np.float32(1.0)).astype(np.float32)


def quantize_blocks(
    x: np.ndarray, block_size: int, valid: np.ndarray | None = None
) -> tuple[np.ndarray, np.ndarray]:
    """Per-block symmetric int8 codes for packed contiguous blocks.

    Returns ``(codes int8 [..., L, D], scales float32 [..., NB])``.  Padding /
    invalid tokens get code 0.
    """
    length = x.shape[-2]
    index = contiguous_block_index(length, block_size)
    scales = quant_scale(block_amax(x, index, valid))
    nb = index.shape[0]
    tok_block = np.minimum(np.arange(length) // block_size, nb - 1)
    s_tok = scales[..., tok_block][..., None]
    q = np.rint(x.astype(np.float32) / s_tok)
    codes = np.clip(q, -127, 127).astype(np.int8)
    if valid is not None:
        codes = np.where(valid[:, None], codes, np.int8(0))
    return codes, scales


# ---------------------------------------------------------------------------
# scores + top-k
# ---------------------------------------------------------------------------


def pooled_scores(qn: np.ndarray, kn: np.ndarray) -> np.ndarray:
    """``qn [..., NQ, D] @ kn [..., NK, D]^T`` in the CUDA warp order."""
    return lane_tree_sum(qn[..., :, None, :] * kn[..., None, :, :])


def rcsa_select_from_scores(
    scores: np.ndarray, n_query_blocks: int, budget: int
) -> tuple[np.ndarray, np.ndarray]:
    """Historical top-budget + block-causal current rule.

    ``scores``: ``[B,H,NQ,NK]``; the last ``NQ`` key blocks are the current
    chunk (query block ``i`` is current key block ``NK-NQ+i``).  Each row keeps
    the ``min(budget, NK-NQ)`` historical blocks of highest score (ties to the
    lower block index, as ``argsort(stable=True)`` in
    ``proposed/qk_uncertainty_tangent_attention.py:978-980``) in rank order,
    followed by current blocks ``0..i`` ascending.  Unused slots are -1.
    """
    b, h, nq, nk = scores.shape
    n_hist = nk - n_query_blocks
    keep = min(budget, n_hist)
    maxdeg = keep + n_query_blocks
    sel = np.full((b, h, nq, maxdeg), -1, dtype=np.int32)
    cnt = np.zeros((b, h, nq), dtype=np.int32)
    for i in range(nq):
        hist = scores[:, :, i, :n_hist]
        order = np.argsort(-hist, axis=-1, kind="stable")[..., :keep]
        sel[:, :, i, :keep] = order
        cur = n_hist + np.arange(i + 1)
        sel[:, :, i, keep:keep + i + 1] = cur
        cnt[:, :, i] = keep + i + 1
    return sel, cnt


def block_grid_local(nt: int, nh: int, nw: int) -> np.ndarray:
    """Manhattan-<=1 stencil over the (t,h,w) block grid
    (``proposed/qk_uncertainty_tangent_attention.py:1029-1039``)."""
    ids = np.arange(nt * nh * nw)
    spatial = nh * nw
    t, rem = ids // spatial, ids % spatial
    hh, ww = rem // nw, rem % nw
    dist = (
        np.abs(t[:, None] - t[None, :])
        + np.abs(hh[:, None] - hh[None, :])
        + np.abs(ww[:, None] - ww[None, :])
    )
    return dist <= 1


def taba_select_from_scores(
    scores: np.ndarray, local: np.ndarray, row_degrees: np.ndarray
) -> tuple[np.ndarray, np.ndarray]:
    """TABA ranking: ``argsort(score + 1e6*local, desc, stable)[..., :maxdeg]``.

    The reference adds the stencil bonus in float32
    (``proposed/qk_uncertainty_tangent_attention.py:1040-1042``), which rounds
    local scores to a 1/16 grid; that rounding is reproduced so that the tie
    order between local blocks matches.
    """
    s32 = scores.astype(np.float32)
    ranking = np.where(local[None, None], s32 + np.float32(LOCAL_BONUS), s32)
    maxdeg = int(row_degrees.max())
    order = np.argsort(-ranking.astype(np.float64), axis=-1, kind="stable")
    sel = order[..., :maxdeg].astype(np.int32)
    b, h = scores.shape[:2]
    cnt = np.broadcast_to(row_degrees.astype(np.int32), (b, h, len(row_degrees))).copy()
    return sel, cnt


def rcsa_select(q: np.ndarray, k: np.ndarray, block_size: int, budget: int,
                q_valid: np.ndarray | None = None, k_valid: np.ndarray | None = None):
    """Full RCSA selection on packed Q ``[B,H,Lq,D]`` / K ``[B,H,Lk,D]``.

    ``q_valid`` / ``k_valid``: optional bool ``[Lq]`` / ``[Lk]`` token
    validity of the compact packing; invalid tokens count as zero and leave the
    pooled-mean denominator (``proposed/matrix_curvature_phase_frame_weave.py:5696-5699``).
    Returns ``(sel, cnt, q_norm, k_norm, scores)``.
    """
    qi = contiguous_block_index(q.shape[-2], block_size)
    ki = contiguous_block_index(k.shape[-2], block_size)
    qs, qc = block_sums(q, qi, q_valid)
    ks, kc = block_sums(k, ki, k_valid)
    qn = pooled_normalized(qs, qc)
    kn = pooled_normalized(ks, kc)
    sc = pooled_scores(qn, kn)
    sel, cnt = rcsa_select_from_scores(sc, qi.shape[0], budget)
    return sel, cnt, qn, kn, sc


def taba_select(
    q: np.ndarray,
    k: np.ndarray,
    latent_hw: tuple[int, int],
    block_shape: tuple[int, int, int],
    row_degrees: np.ndarray,
):
    """TABA ``select`` restated (``proposed/qk_uncertainty_tangent_attention.py:988-1082``)."""
    height, width = latent_hw
    temporal = q.shape[-2] // (height * width)
    index = grid_block_index(temporal, height, width, block_shape)
    s = index.shape[1]
    qs, _ = block_sums(q, index)
    ks, _ = block_sums(k, index)
    den = np.full(index.shape[0], s, dtype=np.int64)  # zero padding counts
    qn = pooled_normalized(qs, den)
    kn = pooled_normalized(ks, den)
    sc = pooled_scores(qn, kn)
    tt, th, tw = block_shape
    local = block_grid_local(-(-temporal // tt), -(-height // th), -(-width // tw))
    sel, cnt = taba_select_from_scores(sc, local, row_degrees)
    return sel, cnt, sc


def compact_pack(x: np.ndarray, block_indices: np.ndarray) -> np.ndarray:
    """Token-order ``[B, L, H, D]`` -> packed ``[B, H, P, D]``: slot ``p`` holds
    token ``block_indices[p]``, zeros where it is -1
    (``proposed/matrix_curvature_phase_frame_weave.py:5677-5684``)."""
    flat = block_indices.reshape(-1)
    out = np.zeros((x.shape[0], x.shape[2], flat.size, x.shape[3]), dtype=x.dtype)
    ok = flat >= 0
    out[:, :, ok] = np.transpose(x[:, flat[ok]], (0, 2, 1, 3))
    return out


def compact_select(q_packed: np.ndarray, k_packed: np.ndarray, valid: np.ndarray, block_size: int,
                   grid: tuple[int, int, int], row_degrees: np.ndarray):
    """The compact path's ranking (``proposed/matrix_curvature_phase_frame_weave.py``
    :5687-5701 masked pooled means, :5718-5725 the stencil on the
    (cell, nh, nw) grid, :5828-5832 ``topk`` of score + 1e6 * stencil): the
    first ``max(row_degrees)`` blocks of every row in (rank descending, index
    ascending) order, counts ``row_degrees``.  ``valid``: bool ``[P]``."""
    index = contiguous_block_index(q_packed.shape[-2], block_size)
    qs, qc = block_sums(q_packed, index, valid)
    ks, kc = block_sums(k_packed, index, valid)
    sc = pooled_scores(pooled_normalized(qs, qc), pooled_normalized(ks, kc))
    sel, cnt = taba_select_from_scores(sc, block_grid_local(*grid), row_degrees)
    return sel, cnt, sc


# ---------------------------------------------------------------------------
# block-sparse attention
# ---------------------------------------------------------------------------


def block_sparse_attention(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    indices: np.ndarray,
    counts: np.ndarray,
    query_block: int,
    key_block: int,
    key_valid: np.ndarray | None = None,
    sm_scale: float | None = None,
    q_codes: np.ndarray | None = None,
    q_scales: np.ndarray | None = None,
    k_codes: np.ndarray | None = None,
    k_scales: np.ndarray | None = None,
    heads: list[int] | None = None,
    rows: np.ndarray | None = None,
) -> np.ndarray:
    """Explicit softmax over the allowed, valid keys of each query block.

    Restates the reference's sampled oracle
    (``proposed/matrix_jit_spatial_acceleration.py:836-858``): bf16-rounded
    q/k/v upcast, logits ``q.k / sqrt(D)``, softmax over exactly the keys of
    the listed blocks that are valid.  With ``q_codes``/``k_codes`` given, the
    logits are instead the exact int8 simulation
    ``(qc . kc) * s_q[qblock] * s_k[kblock] * sm_scale``.
    Query rows whose key set is empty produce zeros.  Returns float64
    ``[B,H,Lq,D]`` (only ``heads`` filled when given; with ``rows``, only
    those row offsets within every query block, the others left zero).
    """
    b, h, lq, d = q.shape
    lk = k.shape[-2]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(d)
    out = np.zeros((b, h, lq, v.shape[-1]), dtype=np.float64)
    nqb = -(-lq // query_block)
    hs = range(h) if heads is None else heads
    int8 = q_codes is not None
    for bi in range(b):
        for hi in hs:
            for qb in range(nqb):
                r0, r1 = qb * query_block, min(lq, (qb + 1) * query_block)
                rsel = np.arange(r0, r1) if rows is None else r0 + rows[rows < r1 - r0]
                n = int(counts[bi, hi, qb])
                blocks = [int(x) for x in indices[bi, hi, qb, :n]]
                keys = []
                kscale = []
                for kb in blocks:
                    k0, k1 = kb * key_block, min(lk, (kb + 1) * key_block)
                    toks = np.arange(k0, k1)
                    if key_valid is not None:
                        toks = toks[key_valid[toks]]
                    keys.append(toks)
                    if int8:
                        kscale.append(np.full(len(toks), float(k_scales[bi, hi, kb])))
                if not keys:
                    continue
                toks = np.concatenate(keys)
                if len(toks) == 0:
                    continue
                if int8:
                    qc = q_codes[bi, hi, rsel].astype(np.float64)
                    kc = k_codes[bi, hi, toks].astype(np.float64)
                    logits = (qc @ kc.T) * (
                        float(q_scales[bi, hi, qb]) * np.concatenate(kscale)[None, :]
                    ) * sm_scale
                else:
                    qf = q[bi, hi, rsel].astype(np.float64)
                    kf = k[bi, hi, toks].astype(np.float64)
                    logits = (qf @ kf.T) * sm_scale
                logits = logits - logits.max(axis=1, keepdims=True)
                w = np.exp(logits)
                w = w / w.sum(axis=1, keepdims=True)
                out[bi, hi, rsel] = w @ v[bi, hi, toks].astype(np.float64)
    return out


def attention_error_stats(reference: np.ndarray, candidate: np.ndarray) -> dict:
    """Same statistics as ``_equivalence_stats``
    (``proposed/matrix_jit_spatial_acceleration.py:880-897``)."""
    r = reference.astype(np.float64).reshape(-1)
    c = candidate.astype(np.float64).reshape(-1)
    delta = c - r
    return {
        "relative_l2": float(np.linalg.norm(delta) / (np.linalg.norm(r) + 1e-12)),
        "cosine": float(np.dot(r, c) / (np.linalg.norm(r) * np.linalg.norm(c) + 1e-30)),
        "mae": float(np.abs(delta).mean()),
        "max_abs": float(np.abs(delta).max()),
    }
