"""CPU restatement of the FC-PASM fixed-budget swap router (test infrastructure).

Only the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use
this module, as the checker of the CUDA swap-router kernels.

Reference: ``src/interaction_accel/methods/proposed/fc_pasm_swap_routing.py``
(``estimate_block_omission_error`` :64-106, ``_objective_terms`` :414-548,
``_objective_value`` :550-614, ``refine`` :616-1077).  The reference builds
the coupled quadratic objective term by term; here the same objective is
written as one block Hessian over the current rows,

    J(e) = sum_i c_i |e_i|^2 + e^T H e,

with ``c_i`` = lambda_anchor x (Exact anchors in row i's temporal cell) and
``H`` the sum over skipped targets t of lambda_rec x [A_t B_t]^T [A_t B_t]
placed on (left cell, right cell) -- A_t = (1-alpha) M(alpha),
B_t = alpha M(-(1-alpha)), M the transport operator on the attention grid
(the identity where no transport is present).  The coordinate-descent
improvement of replacing one row error e_r by e_r + d is then
sum_g a_r (2 e_rg d_g + d_g^2) + 2 b_rg d_g with a_r = c_r + H_rr and
b_r = (H e)_r - H_rr e_r, which is what the reference evaluates.

Parity is pinned by ``tests/golden/swap_*.npz``, written by running
the reference's own ``refine`` (``tests/golden/make_golden.py --only swap``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

F32 = np.float32


@dataclass
class SwapConfig:
    """The numeric fields of the reference's ``FCPASMSwapRoutingConfig`` (:23-62)."""

    candidate_multiplier: int = 2
    num_swap_rounds: int = 1
    swap_eps: float = 1e-6
    lambda_anchor: float = 1.0
    lambda_reconstruction: float = 1.0
    sketch_groups: int = 16
    max_swaps_per_call: int = 0
    historical_only: bool = False
    same_bank_only: bool = False


def softmax_rows(score: np.ndarray) -> np.ndarray:
    s = score.astype(F32)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m, dtype=F32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)


def omission_proxy(prob, pooled_value, cand, groups, eps=1e-6):
    """``estimate_block_omission_error`` (:64-106): prob [B,H,Q,K],
    pooled_value [B,H,K,D], cand [B,H,Q,L] -> proxy [B,H,Q,L,G]."""
    v = pooled_value.astype(F32)
    out = np.einsum("bhqk,bhkd->bhqd", prob.astype(np.float64), v.astype(np.float64)).astype(F32)
    cv = np.take_along_axis(v[:, :, None], cand[..., None].astype(np.int64), axis=3)  # [B,H,Q,L,D]
    cp = np.take_along_axis(prob, cand.astype(np.int64), axis=-1).astype(F32)
    scale = (cp / (F32(1.0) - cp + F32(eps))).astype(F32)
    proxy = (scale[..., None] * (out[..., None, :] - cv)).astype(F32)
    D = v.shape[-1]
    return proxy.reshape(*proxy.shape[:-1], groups, D // groups).mean(-1, dtype=np.float64).astype(F32)


def frame_cell(frame: int, group: int, cells: int) -> int:
    return min(int(frame) // int(group), cells - 1)


def skipped_targets(exact_frames, boundary):
    """(left, right, alpha) for every skipped frame between consecutive Exact
    anchors of the same Current segment (:451-456, :586-590)."""
    out = []
    for left, right in zip(exact_frames, exact_frames[1:]):
        if (left < boundary) != (right < boundary):
            continue
        for t in range(left + 1, right):
            out.append((int(left), int(right), float(t - left) / float(right - left)))
    return out


def quadratic_terms(*, cells, spatial, exact_frames, group, boundary, lam_a, lam_r, operator=None):
    """(coefficient c [R], Hessian H [R,R]) of the objective over the current
    rows (R = cells x spatial), float64.  ``operator(pair, exponent)`` returns
    the [spatial, spatial] transport operator (identity when ``None``)."""
    R = cells * spatial
    eye = np.eye(spatial)
    op = (lambda pair, x: eye) if operator is None else operator
    cnt = np.zeros(cells)
    for f in exact_frames:
        cnt[frame_cell(f, group, cells)] += 1.0
    c = np.repeat(cnt * lam_a, spatial)
    H = np.zeros((R, R))
    for left, right, alpha in skipped_targets(exact_frames, boundary):
        A = (1.0 - alpha) * np.asarray(op((left, right), alpha), dtype=np.float64)
        Bm = alpha * np.asarray(op((left, right), -(1.0 - alpha)), dtype=np.float64)
        lc, rc = frame_cell(left, group, cells), frame_cell(right, group, cells)
        ls, rs = slice(lc * spatial, (lc + 1) * spatial), slice(rc * spatial, (rc + 1) * spatial)
        if lc == rc:
            C = A + Bm
            H[ls, ls] += lam_r * C.T @ C
        else:
            H[ls, ls] += lam_r * A.T @ A
            H[rs, rs] += lam_r * Bm.T @ Bm
            H[ls, rs] += lam_r * A.T @ Bm
            H[rs, ls] += lam_r * Bm.T @ A
    return c, H


def objective(err, c, H):
    """J = sum_i c_i |e_i|^2 + e^T H e over [B,H,R,G] errors (float64)."""
    e = err.astype(np.float64)
    return float((c[None, None, :, None] * e * e).sum() + np.einsum("rs,bhsg,bhrg->", H, e, e))


def topk_desc(x, k):
    """Indices of the k largest entries per row, larger first, lower index first on ties."""
    order = np.argsort(-x, axis=-1, kind="stable")
    return order[..., :k]


def refine(*, score, pooled_value, selected, counts, local, memory_blocks, spatial, exact_frames,
           group, boundary, config: SwapConfig, operator=None, row_gate=None):
    """The numeric body of ``refine`` (:616-1077) after its fallback gates:
    candidates, omission proxies, then up to ``num_swap_rounds`` single-swap
    coordinate-descent rounds.  Returns (selected', stats)."""
    cfg = config
    B, Hh, Q, K = score.shape
    S = selected.shape[-1]
    R = Q - memory_blocks
    cells = R // spatial
    sel = selected.astype(np.int64).copy()
    cnt = counts.astype(np.int64)
    valid_sel = np.arange(S)[None, None, None] < cnt[..., None]
    swappable = valid_sel & (sel < memory_blocks) if cfg.historical_only else valid_sel
    maxk = int(swappable.sum(-1).max())
    cand_blocks = memory_blocks if cfg.historical_only else K
    L = min(cand_blocks, cfg.candidate_multiplier * maxk)
    ranking = (score[..., :cand_blocks].astype(F32)
               + local[:, :cand_blocks][None, None].astype(F32) * F32(1e6)).astype(F32)
    cand = topk_desc(ranking, L)
    prob = softmax_rows(score)
    proxy = omission_proxy(prob, pooled_value, cand, cfg.sketch_groups)
    limit = np.minimum(swappable.sum(-1) * cfg.candidate_multiplier, cand_blocks)
    cand_valid = np.arange(L)[None, None, None] < limit[..., None]

    def membership(cur):
        vs = np.arange(S)[None, None, None] < cnt[..., None]
        return ((cand[..., None] == cur[..., None, :]) & vs[..., None, :]).any(-1)

    retained = membership(sel)
    err = (proxy * (cand_valid & ~retained)[..., None]).sum(-2, dtype=np.float64).astype(F32)
    cur_err = err[:, :, memory_blocks:].astype(np.float64)
    c, Hm = quadratic_terms(cells=cells, spatial=spatial, exact_frames=exact_frames, group=group,
                            boundary=boundary, lam_a=cfg.lambda_anchor,
                            lam_r=cfg.lambda_reconstruction, operator=operator)
    before = objective(cur_err, c, Hm)
    swaps, improvement, chosen = 0, 0.0, []
    for _ in range(cfg.num_swap_rounds):
        a = c + np.diag(Hm)
        bl = np.einsum("rs,bhsg->bhrg", Hm, cur_err) - np.diag(Hm)[None, None, :, None] * cur_err
        retained = membership(sel)
        vs = np.arange(S)[None, None, None] < cnt[..., None]
        sel_local = np.take_along_axis(np.broadcast_to(local[None, None], (B, Hh, Q, K)), sel, -1)
        removable = vs & ~sel_local
        if cfg.historical_only:
            removable &= sel < memory_blocks
        addable = cand_valid & ~retained
        match = (cand[..., :, None] == sel[..., None, :])  # [B,H,Q,L,S]
        rem = np.einsum("bhqlg,bhqls->bhqsg", proxy.astype(np.float64), match.astype(np.float64))[:, :, memory_blocks:]
        add = proxy[:, :, memory_blocks:].astype(np.float64)
        d = rem[..., :, None, :] - add[..., None, :, :]  # [B,H,R,S,L,G]
        imp = (a[None, None, :, None, None, None] * (2.0 * cur_err[..., None, None, :] * d + d * d)
               + 2.0 * bl[..., None, None, :] * d).sum(-1)
        ok = removable[:, :, memory_blocks:, :, None] & addable[:, :, memory_blocks:, None, :]
        if row_gate is not None:
            ok &= np.asarray(row_gate, dtype=bool)[None, None, :, None, None]
        if cfg.same_bank_only:
            ok &= (sel[:, :, memory_blocks:, :, None] < memory_blocks) == (
                cand[:, :, memory_blocks:, None, :] < memory_blocks)
        imp = np.where(ok, imp, np.inf)
        flat = imp.reshape(B, Hh, R, S * L)
        best = flat.min(-1)
        arg = flat.argmin(-1)
        strongest = int(np.argmin(best.reshape(-1)))
        do = best.reshape(-1)[strongest] < -cfg.swap_eps
        if cfg.max_swaps_per_call and swaps >= cfg.max_swaps_per_call:
            break
        if not do:
            break
        b, h, r = np.unravel_index(strongest, (B, Hh, R))
        s_slot, l_slot = divmod(int(arg[b, h, r]), L)
        q = memory_blocks + r
        sel[b, h, q, s_slot] = cand[b, h, q, l_slot]
        cur_err[b, h, r] += rem[b, h, r, s_slot] - add[b, h, r, l_slot]
        swaps += 1
        improvement += -float(best[b, h, r])
        chosen.append((int(b), int(h), int(q), s_slot, int(cand[b, h, q, l_slot])))
    after = objective(cur_err, c, Hm)
    return sel, {"swap_count": swaps, "objective_before": before, "objective_after": after,
                 "improvement": improvement, "candidate_max": L, "swaps": chosen,
                 "error": cur_err.astype(F32), "proxy": proxy, "candidates": cand}


def pair_row_gate(*, exact_frames, boundary, group, cells, spatial, affinity_of, threshold):
    """Rows a swap may touch under the per-pair affinity gate (:785-820):
    the cells of skipped targets whose anchor pair's mean affinity reaches
    ``threshold``.  ``affinity_of(pair)`` gives the pair's mean affinity."""
    gate = np.zeros(cells, dtype=bool)
    for left, right in zip(exact_frames, exact_frames[1:]):
        if right - left <= 1 or (left < boundary) != (right < boundary):
            continue
        if affinity_of((left, right)) < threshold:
            continue
        for t in range(left + 1, right):
            gate[frame_cell(t, group, cells)] = True
    return np.repeat(gate, spatial)
