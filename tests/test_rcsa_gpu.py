"""RCSA parity on the GPU: CUDA kernels (through the C ABI) vs the CPU oracle.

Bars: selected block indices, int8 codes and scales bit-exact; attention
within max-abs 2e-2 / mean-abs 2e-3 of the oracle's bf16 path (and of the
exact int8 simulation for int8 QK^T).
"""

import math
import os

import numpy as np
import pytest
import torch

from cast_b200 import rcsa, workloads
from oracle import rcsa as orc

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _np(t):
    return t.detach().float().cpu().numpy()


def _rand_problem(heads, lq_blocks, lk_hist, block, d=128, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(1, heads, lq_blocks * block, d, generator=g) * scale).bfloat16()
    k = (torch.randn(1, heads, (lk_hist + lq_blocks) * block, d, generator=g) * scale).bfloat16()
    v = (torch.randn(1, heads, (lk_hist + lq_blocks) * block, d, generator=g) * scale).bfloat16()
    return q, k, v


def _check_selection(sel, q, k, block, budget):
    o_sel, o_cnt, _, _, scores = orc.rcsa_select(_np(q), _np(k), block, budget)
    got = sel.indices.cpu().numpy()
    if not np.array_equal(got, o_sel):
        bad = np.argwhere(got != o_sel)[:5]
        raise AssertionError(f"selected blocks differ at {bad.tolist()}")
    assert np.array_equal(sel.counts.cpu().numpy(), o_cnt)
    return o_sel, o_cnt


def _check_codes(sel, q, k, block):
    qc, qs = orc.quantize_blocks(_np(q), block)
    kc, ks = orc.quantize_blocks(_np(k), block)
    assert np.array_equal(sel.q_scales.cpu().numpy(), qs)
    assert np.array_equal(sel.k_scales.cpu().numpy(), ks)
    assert np.array_equal(sel.q_codes.cpu().numpy(), qc)
    assert np.array_equal(sel.k_codes.cpu().numpy(), kc)
    return qc, qs, kc, ks


def _errs(out, ref):
    d = np.abs(_np(out).astype(np.float64) - ref)
    return float(d.max()), float(d.mean())


# 1040-row blocks leave rows for the loop after the 8-deep unrolled loads
# (16 row partials x 8 rows per step)
@pytest.mark.parametrize("block,nq,nh,budget", [(128, 2, 6, 3), (880, 2, 5, 2), (64, 2, 8, 4),
                                                (1040, 2, 4, 2)])
def test_select_quant_bitexact(cuda, block, nq, nh, budget):
    q, k, v = _rand_problem(2, nq, nh, block, seed=block)
    sel = rcsa.select_quant(q.cuda(), k.cuda(), block_size=block, budget=budget, policy="int8")
    torch.cuda.synchronize()
    _check_selection(sel, q, k, block, budget)
    _check_codes(sel, q, k, block)
    assert bool((sel.qk_mode == 1).all())


@pytest.mark.parametrize("d", [128, 64])
def test_select_quant_valid_mask(cuda, d):
    """Compact-packing validity (proposed/matrix_curvature_phase_frame_weave.py:5696-5699):
    padded tokens hold large garbage here, so any leak into the sums, the
    amax or the pooled-mean denominator changes the selection or the codes."""
    block, nq, nh, budget = 128, 2, 6, 3
    q, k, _ = _rand_problem(2, nq, nh, block, d=d, seed=7)
    g = torch.Generator().manual_seed(8)
    q_valid = torch.rand(q.shape[2], generator=g) > 0.2
    k_valid = torch.rand(k.shape[2], generator=g) > 0.2
    k_valid[2 * block:3 * block] = False  # a fully padded history block
    q = torch.where(q_valid[None, None, :, None], q, torch.full_like(q, 60.0))
    k = torch.where(k_valid[None, None, :, None], k, torch.full_like(k, -70.0))
    sel = rcsa.select_quant(q.cuda(), k.cuda(), block_size=block, budget=budget, policy="int8",
                            return_pooled=True, q_valid=q_valid.to(torch.uint8).cuda(),
                            k_valid=k_valid.to(torch.uint8).cuda())
    torch.cuda.synchronize()
    qv, kv = q_valid.numpy(), k_valid.numpy()
    o_sel, o_cnt, qn, kn, _ = orc.rcsa_select(_np(q), _np(k), block, budget, q_valid=qv, k_valid=kv)
    assert np.array_equal(sel.indices.cpu().numpy(), o_sel)
    assert np.array_equal(sel.counts.cpu().numpy(), o_cnt)
    pooled = sel.pooled.cpu().numpy()
    assert np.array_equal(pooled[:, :, :nq], qn) and np.array_equal(pooled[:, :, nq:], kn)
    qc, qs = orc.quantize_blocks(_np(q), block, qv)
    kc, ks = orc.quantize_blocks(_np(k), block, kv)
    assert np.array_equal(sel.q_scales.cpu().numpy(), qs) and np.array_equal(sel.k_scales.cpu().numpy(), ks)
    assert np.array_equal(sel.q_codes.cpu().numpy(), qc) and np.array_equal(sel.k_codes.cpu().numpy(), kc)


@pytest.mark.parametrize("masked", [False, True])
def test_auto_policy_codes_where_read(cuda, masked):
    """Auto policy: codes are written after the selection, only for the
    blocks an int8 query block reads (its own Q block, the K blocks it
    selected); there they equal the int8 policy's codes bit for bit, and the
    scales equal for every block."""
    w = workloads.config2(heads=4)
    q, k = w.q.cuda(), w.k.cuda()
    kw = {}
    if masked:
        g = torch.Generator().manual_seed(3)
        kw = dict(q_valid=(torch.rand(q.shape[2], generator=g) > 0.1).to(torch.uint8).cuda(),
                  k_valid=(torch.rand(k.shape[2], generator=g) > 0.1).to(torch.uint8).cuda())
    auto = rcsa.select_quant(q, k, block_size=880, budget=8, policy="auto", **kw)
    full = rcsa.select_quant(q, k, block_size=880, budget=8, policy="int8", **kw)
    torch.cuda.synchronize()
    assert torch.equal(auto.indices, full.indices) and torch.equal(auto.counts, full.counts)
    assert torch.equal(auto.q_scales, full.q_scales) and torch.equal(auto.k_scales, full.k_scales)
    mode = auto.qk_mode.cpu()
    assert bool(mode.any()) and not bool(mode.all())
    idx, cnt = auto.indices.cpu(), auto.counts.cpu()
    n_q = n_k = 0
    for h in range(4):
        needed = set()
        for qb in range(4):
            if mode[0, h, qb]:
                sl = slice(qb * 880, (qb + 1) * 880)
                assert torch.equal(auto.q_codes[0, h, sl], full.q_codes[0, h, sl])
                needed.update(int(x) for x in idx[0, h, qb, :cnt[0, h, qb]])
                n_q += 1
        for kb in sorted(needed):
            sl = slice(kb * 880, (kb + 1) * 880)
            assert torch.equal(auto.k_codes[0, h, sl], full.k_codes[0, h, sl])
            n_k += 1
    print(f"auto policy: {n_q} int8 query blocks, {n_k} K blocks quantised of {4 * 36}")


def test_select_quant_d64_config1_golden(cuda):
    w = workloads.config1()
    g = np.load(os.path.join(GOLDEN, "cfg1_select.npz"))
    qa = np.load(os.path.join(GOLDEN, "cfg1_quant_attn.npz"))
    q = w.q.bfloat16()
    k = w.k.bfloat16()
    # config 1 is fp32 data; the kernels take bf16, so compare against the
    # oracle on the same bf16-rounded tensors, and check the fp32 golden
    # selection survives bf16 rounding of the inputs.
    sel = rcsa.select_quant(q.cuda(), k.cuda(), block_size=64, budget=4, policy="int8")
    torch.cuda.synchronize()
    _check_selection(sel, q, k, 64, 4)
    assert np.array_equal(sel.indices.cpu().numpy(), g["budget_selected"])
    assert qa["q_scales"].shape == sel.q_scales.shape


def test_attention_modes_small(cuda):
    block, nq, nh, budget = 128, 2, 6, 3
    q, k, v = _rand_problem(2, nq, nh, block, seed=11)
    sel = rcsa.select_quant(q.cuda(), k.cuda(), block_size=block, budget=budget, policy="int8")
    o_sel, o_cnt = _check_selection(sel, q, k, block, budget)
    qc, qs, kc, ks = _check_codes(sel, q, k, block)
    ref_bf16 = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, block, block)
    ref_int8 = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, block, block,
                                          q_codes=qc, q_scales=qs, k_codes=kc, k_scales=ks)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    out_b = rcsa.block_sparse_attention(qd, kd, vd, sel.indices, sel.counts, q_block=block, k_block=block)
    out_i = rcsa.block_sparse_attention(qd, kd, vd, sel.indices, sel.counts, q_block=block, k_block=block,
                                        q_codes=sel.q_codes, q_scales=sel.q_scales,
                                        k_codes=sel.k_codes, k_scales=sel.k_scales)
    torch.cuda.synchronize()
    mb, ab = _errs(out_b, ref_bf16)
    mi, ai = _errs(out_i, ref_int8)
    print(f"bf16 vs oracle: max {mb:.2e} mean {ab:.2e}; int8 vs int8-sim: max {mi:.2e} mean {ai:.2e}")
    assert mb < MAX_ABS and ab < MEAN_ABS
    assert mi < MAX_ABS and ai < MEAN_ABS


@pytest.mark.parametrize("mode", ["bf16", "int8"])
def test_attention_frame_blocks_masking(cuda, mode):
    """880-token blocks: 7 query tiles (3 pairs + 1 single) and 7 key tiles
    per block, the last one masked to 112 keys."""
    block, nq, nh, budget = 880, 2, 4, 2
    q, k, v = _rand_problem(2, nq, nh, block, seed=5)
    sel = rcsa.select_quant(q.cuda(), k.cuda(), block_size=block, budget=budget, policy="int8")
    o_sel, o_cnt = _check_selection(sel, q, k, block, budget)
    kw = {}
    oracle_kw = {}
    if mode == "int8":
        qc, qs, kc, ks = _check_codes(sel, q, k, block)
        kw = dict(q_codes=sel.q_codes, q_scales=sel.q_scales, k_codes=sel.k_codes, k_scales=sel.k_scales)
        oracle_kw = dict(q_codes=qc, q_scales=qs, k_codes=kc, k_scales=ks)
    ref = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, block, block, **oracle_kw)
    out = rcsa.block_sparse_attention(q.cuda(), k.cuda(), v.cuda(), sel.indices, sel.counts,
                                      q_block=block, k_block=block, **kw)
    torch.cuda.synchronize()
    m, a = _errs(out, ref)
    print(f"{mode}: max {m:.2e} mean {a:.2e}")
    assert m < MAX_ABS and a < MEAN_ABS


def test_longcat_active_dropin_key_valid(cuda):
    """The _longcat_active seam: [nBlocks,S] key-valid mask, a fully masked
    block, rows whose allowed keys are all invalid (-> zeros), and a padded
    index list (count < max_degree)."""
    block, heads, nb = 128, 2, 6
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, heads, nb * block, 128, generator=g).bfloat16()
    k = torch.randn(1, heads, nb * block, 128, generator=g).bfloat16()
    v = torch.randn(1, heads, nb * block, 128, generator=g).bfloat16()
    valid = torch.rand(nb, block, generator=g) > 0.3
    valid[2] = False  # a fully masked block
    idx = torch.full((1, heads, nb, 4), -1, dtype=torch.int32)
    cnt = torch.zeros(1, heads, nb, dtype=torch.int32)
    for h in range(heads):
        for i in range(nb):
            choice = torch.randperm(nb, generator=g)[:3].to(torch.int32)
            n = 1 + (i + h) % 3
            idx[0, h, i, :n] = choice[:n]
            cnt[0, h, i] = n
    idx[0, 0, 1, 0] = 2  # row list made only of the masked block
    cnt[0, 0, 1] = 1
    out = rcsa.longcat_active(q.cuda(), k.cuda(), v.cuda(), idx.cuda(), cnt.cuda(), valid.cuda(), block)
    torch.cuda.synchronize()
    ref = orc.block_sparse_attention(_np(q), _np(k), _np(v), idx.numpy(), cnt.numpy(), block, block,
                                     key_valid=valid.reshape(-1).numpy())
    m, a = _errs(out, ref)
    assert m < MAX_ABS and a < MEAN_ABS
    assert float(out[0, 0, block:2 * block].abs().max()) == 0.0


@pytest.mark.parametrize("mode", ["bf16", "int8"])
def test_attention_cut_items(cuda, mode):
    """Items cut along their key tiles (balance=True) against whole items and
    the oracle: random counts including 0 and max_degree, a fully masked key
    block, ragged Lk, and count hints that are too small, too large or
    absent (parts that run past their planned range, or are empty).  Two
    calls in a row give identical bits (the arrival counters reset)."""
    block, heads, nqb, nkb = 880, 2, 2, 7
    g = torch.Generator().manual_seed(21)
    lk = nkb * block - 300
    q = torch.randn(1, heads, nqb * block, 128, generator=g).bfloat16()
    k = torch.randn(1, heads, lk, 128, generator=g).bfloat16()
    v = torch.randn(1, heads, lk, 128, generator=g).bfloat16()
    valid = torch.rand(lk, generator=g) > 0.2
    valid[3 * block:4 * block] = False
    max_degree = 6
    idx = torch.full((1, heads, nqb, max_degree), -1, dtype=torch.int32)
    cnt = torch.tensor([[[0, max_degree], [3, 5]]], dtype=torch.int32)
    for h in range(heads):
        for i in range(nqb):
            idx[0, h, i, :cnt[0, h, i]] = torch.randperm(nkb, generator=g)[:cnt[0, h, i]].to(torch.int32)
    kw, okw = {}, {}
    if mode == "int8":
        kp = torch.cat([k, torch.zeros(1, heads, nkb * block - lk, 128, dtype=k.dtype)], dim=2)
        sel = rcsa.select_quant(q.cuda(), kp.cuda(), block_size=block, budget=2, policy="int8")
        kw = dict(q_codes=sel.q_codes, q_scales=sel.q_scales,
                  k_codes=sel.k_codes[:, :, :lk].contiguous(), k_scales=sel.k_scales)
        qc, qs = orc.quantize_blocks(_np(q), block)
        kc, ks = orc.quantize_blocks(_np(kp), block)
        okw = dict(q_codes=qc, q_scales=qs, k_codes=kc[:, :, :lk], k_scales=ks)
    ref = orc.block_sparse_attention(_np(q), _np(k), _np(v), idx.numpy(), cnt.numpy(), block, block,
                                     key_valid=valid.numpy(), **okw)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    common = dict(q_block=block, k_block=block, key_valid=valid.to(torch.uint8).cuda(), return_lse=True, **kw)
    # without a workspace no item is cut, but tail pairs may run as single tiles
    whole, lse_w = rcsa.block_sparse_attention(qd, kd, vd, idx.cuda(), cnt.cuda(), balance=False, **common)
    torch.cuda.synchronize()
    m, a = _errs(whole, ref)
    assert m < MAX_ABS and a < MEAN_ABS
    for hint in (None, np.full((1, heads, nqb), 1), np.full((1, heads, nqb), max_degree),
                 np.array([[[2, 6], [1, 4]]] * 1)):
        outs = [rcsa.block_sparse_attention(qd, kd, vd, idx.cuda(), cnt.cuda(), count_hint=hint, **common)
                for _ in range(2)]
        torch.cuda.synchronize()
        (o1, l1), (o2, l2) = outs
        assert torch.equal(o1, o2) and torch.equal(l1, l2)
        m, a = _errs(o1, ref)
        print(f"{mode} hint {None if hint is None else hint.ravel().tolist()}: max {m:.2e} mean {a:.2e}")
        assert m < MAX_ABS and a < MEAN_ABS
        assert float((o1.float() - whole.float()).abs().max()) < MAX_ABS
        fin = torch.isfinite(lse_w)
        assert torch.equal(fin, torch.isfinite(l1))
        assert float((l1[fin] - lse_w[fin]).abs().max()) < 1e-3
    # the item with no key block writes zeros
    assert float(o1[0, 0, :block].abs().max()) == 0.0


def test_rcsa_config2_two_heads(cuda):
    """Config 2 shape (880-token frames, 32 history + 4 current, budget 8) on
    heads 0-1 of the seeded config-2 tensors, through the full RCSA call."""
    w = workloads.config2()
    q, k, v = (t[:, :2].contiguous() for t in (w.q, w.k, w.v))
    gold = np.load(os.path.join(GOLDEN, "cfg2_select_h2.npz"))
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    results = {}
    for policy in ("bf16", "auto", "int8"):
        out, sel = rcsa.rcsa_attention(qd, kd, vd, block_size=880, budget=8, policy=policy)
        torch.cuda.synchronize()
        results[policy] = (out, sel)
    sel = results["int8"][1]
    o_sel, o_cnt = _check_selection(sel, q, k, 880, 8)
    # the reference's float32 pooled scores give the same selection
    assert np.array_equal(o_sel, gold["selected"])
    qc, qs, kc, ks = _check_codes(sel, q, k, 880)
    ref_bf16 = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, 880, 880)
    ref_int8 = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, 880, 880,
                                          q_codes=qc, q_scales=qs, k_codes=kc, k_scales=ks)
    mb, ab = _errs(results["bf16"][0], ref_bf16)
    mi, ai = _errs(results["int8"][0], ref_int8)
    ma, aa = _errs(results["auto"][0], ref_bf16)
    print(f"bf16 {mb:.2e}/{ab:.2e} int8-vs-sim {mi:.2e}/{ai:.2e} auto-vs-bf16 {ma:.2e}/{aa:.2e} "
          f"modes {results['auto'][1].qk_mode.flatten().tolist()}")
    assert mb < MAX_ABS and ab < MEAN_ABS
    assert mi < MAX_ABS and ai < MEAN_ABS
    assert ma < MAX_ABS and aa < MEAN_ABS


def test_rcsa_config3_two_heads(cuda):
    """Config 3 shape (anchor queries 0 and 3 over 128 history frames + the
    two anchor key frames, budget 16) generated with 2 heads, through the full
    RCSA call."""
    w = workloads.config3(heads=2)
    q, k, v = w.q, w.k, w.v
    gold = np.load(os.path.join(GOLDEN, "cfg3_select_h2.npz"))
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    results = {}
    for policy in ("bf16", "auto", "int8"):
        out, sel = rcsa.rcsa_attention(qd, kd, vd, block_size=880, budget=w.budget, policy=policy)
        torch.cuda.synchronize()
        results[policy] = (out, sel)
    sel = results["int8"][1]
    o_sel, o_cnt = _check_selection(sel, q, k, 880, w.budget)
    # the reference's float32 pooled scores give the same selection
    assert np.array_equal(o_sel, gold["selected"]) and np.array_equal(o_cnt, gold["counts"])
    assert o_sel.shape == (1, 2, 2, 18)
    qc, qs, kc, ks = _check_codes(sel, q, k, 880)
    ref_bf16 = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, 880, 880)
    ref_int8 = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, 880, 880,
                                          q_codes=qc, q_scales=qs, k_codes=kc, k_scales=ks)
    mb, ab = _errs(results["bf16"][0], ref_bf16)
    mi, ai = _errs(results["int8"][0], ref_int8)
    ma, aa = _errs(results["auto"][0], ref_bf16)
    print(f"bf16 {mb:.2e}/{ab:.2e} int8-vs-sim {mi:.2e}/{ai:.2e} auto-vs-bf16 {ma:.2e}/{aa:.2e} "
          f"modes {results['auto'][1].qk_mode.flatten().tolist()}")
    assert mb < MAX_ABS and ab < MEAN_ABS
    assert mi < MAX_ABS and ai < MEAN_ABS
    assert ma < MAX_ABS and aa < MEAN_ABS


def test_rcsa_config2_full_properties(cuda):
    """All 24 heads at full size: structure of the selection, code
    reconstruction bound, finite outputs, and int8/bf16 agreement where the
    policy chose int8."""
    w = workloads.config2(device="cuda")
    out_a, sel = rcsa.rcsa_attention(w.q, w.k, w.v, block_size=880, budget=8, policy="auto")
    out_b, _ = rcsa.rcsa_attention(w.q, w.k, w.v, block_size=880, budget=8, policy="bf16")
    torch.cuda.synchronize()
    idx = sel.indices.cpu()
    cnt = sel.counts.cpu()
    assert idx.shape == (1, 24, 4, 12)
    for i in range(4):
        assert bool((cnt[0, :, i] == 8 + i + 1).all())
        hist = idx[0, :, i, :8]
        assert bool((hist >= 0).all()) and bool((hist < 32).all())
        assert bool((hist.sort(dim=-1).values.diff(dim=-1) > 0).all())
        assert bool((idx[0, :, i, 8:9 + i] == torch.arange(32, 33 + i)).all())
    # under the auto policy only int8 query blocks have Q codes
    deq = sel.q_codes.float() * sel.q_scales.repeat_interleave(880, dim=2)[..., None]
    int8_rows = sel.qk_mode.bool().repeat_interleave(880, dim=2)[..., None]
    err = torch.where(int8_rows, (deq - w.q.float()).abs(), torch.zeros_like(deq))
    assert bool(sel.qk_mode.any())
    assert float(err.max()) <= float(sel.q_scales.max()) * 0.5 + 1e-6
    assert bool(torch.isfinite(out_a.float()).all())
    diff = (out_a.float() - out_b.float()).abs()
    assert float(diff.mean()) < MEAN_ABS and float(diff.max()) < MAX_ABS


def test_taba_select_config1_golden(cuda):
    """TABA full-layer selection (cast_taba_select) on config 1 against the
    reference's own ``select`` output and the oracle."""
    from cast_b200.select import TABASelector

    g = np.load(os.path.join(GOLDEN, "cfg1_select.npz"))
    w = workloads.config1()
    q = w.meta["q_full"].bfloat16()
    k = w.k.bfloat16()
    sel = TABASelector((1, 8, 8))
    sel.set_row_degrees(torch.from_numpy(g["taba_row_degrees"]))
    idx, cnt, report, scores = sel.select(q.cuda(), k.cuda(), geometry_indices=None,
                                          geometry_counts=None, latent_hw=(8, 8),
                                          block_shape=(1, 8, 8), return_scores=True)
    torch.cuda.synchronize()
    o_sel, o_cnt, o_sc = orc.taba_select(_np(q), _np(k), (8, 8), (1, 8, 8), g["taba_row_degrees"])
    assert np.array_equal(scores.cpu().numpy(), o_sc)
    assert np.array_equal(idx.cpu().numpy(), o_sel)
    assert np.array_equal(cnt.cpu().numpy(), o_cnt)
    assert np.array_equal(idx.cpu().numpy(), g["taba_selected"])
    assert report.budget_max == int(g["taba_row_degrees"].max())


@pytest.mark.parametrize("block_shape", [(1, 4, 8), (2, 11, 10), (1, 22, 40)])
def test_taba_select_ragged_grid_bitexact(cuda, block_shape):
    """22x40 latent (config-2 frame grid) tiled by block shapes that leave
    ragged edge tiles; per-row degrees vary."""
    from cast_b200.select import TABASelector

    gen = torch.Generator().manual_seed(11)
    t, hl, wl, d, heads = 4, 22, 40, 128, 3
    q = torch.randn(1, heads, t * hl * wl, d, generator=gen).bfloat16()
    k = (torch.randn(1, heads, t * hl * wl, d, generator=gen) + 0.3 * q.float()).bfloat16()
    tt, th, tw = block_shape
    nblocks = -(-t // tt) * -(-hl // th) * -(-wl // tw)
    degrees = torch.randint(1, min(nblocks, 20) + 1, (nblocks,), generator=gen)
    sel = TABASelector(block_shape)
    sel.set_row_degrees(degrees)
    idx, cnt, _, scores = sel.select(q.cuda(), k.cuda(), geometry_indices=None,
                                     geometry_counts=None, latent_hw=(hl, wl),
                                     block_shape=block_shape, return_scores=True)
    torch.cuda.synchronize()
    o_sel, o_cnt, o_sc = orc.taba_select(_np(q), _np(k), (hl, wl), block_shape, degrees.numpy())
    assert np.array_equal(scores.cpu().numpy(), o_sc)
    assert np.array_equal(idx.cpu().numpy(), o_sel)
    assert np.array_equal(cnt.cpu().numpy(), o_cnt)


def test_host_plan_matches_device_plan(cuda):
    """RCSAHostPlan (pinned host inputs, head groups with overlapped copies)
    gives the device plan's selection and, within the attention bars, its
    output; two calls in a row give the same bits."""
    w = workloads.config2(heads=4)
    hq, hk, hv = (t.pin_memory() for t in (w.q, w.k, w.v))
    hout = torch.empty(w.q.shape, dtype=torch.bfloat16).pin_memory()
    hp = rcsa.RCSAHostPlan(1, 4, w.q.shape[2], w.k.shape[2], 128, block_size=880, budget=8,
                           groups=3, device="cuda")
    hp(hq, hk, hv, hout)
    torch.cuda.synchronize()
    first = hout.clone()
    hp(hq, hk, hv, hout)
    torch.cuda.synchronize()
    assert torch.equal(first, hout)
    dp = rcsa.RCSAPlan(1, 4, w.q.shape[2], w.k.shape[2], 128, block_size=880, budget=8, device="cuda")
    ref = dp(w.q.cuda(), w.k.cuda(), w.v.cuda())
    torch.cuda.synchronize()
    for (h0, h1), plan in zip(hp.heads, hp.plans):
        assert torch.equal(plan.indices, dp.indices[:, h0:h1])
        assert torch.equal(plan.qk_mode, dp.qk_mode[:, h0:h1])
    d = (hout.float() - ref.float().cpu()).abs()
    assert float(d.max()) < MAX_ABS and float(d.mean()) < MEAN_ABS
    # only the selected value blocks crossed the link; copying every value
    # block gives the same bits
    full_bytes = sum(t.numel() * 2 for t in (hq, hk, hv))
    assert hp.last_h2d_bytes < full_bytes and hp.last_d2h_bytes == hout.numel() * 2
    hv_all = rcsa.RCSAHostPlan(1, 4, w.q.shape[2], w.k.shape[2], 128, block_size=880, budget=8,
                               groups=3, device="cuda", v_selected=False)
    hout2 = torch.empty_like(hout).pin_memory()
    hv_all(hq, hk, hv, hout2)
    assert hv_all.last_h2d_bytes == full_bytes
    assert torch.equal(hout2, hout)


def test_host_plan_copies_exactly_the_selected_values(cuda):
    """The value blocks a selected-values call copies are the union of its
    heads' selections (with the default gap merging, plus short gaps between
    them): poisoning every other block of the host values with NaN leaves the
    output finite and unchanged."""
    w = workloads.config2(heads=2)
    hq, hk, hv = (t.pin_memory() for t in (w.q, w.k, w.v))
    hp = rcsa.RCSAHostPlan(1, 2, w.q.shape[2], w.k.shape[2], 128, block_size=880, budget=8,
                           groups=2, device="cuda")
    hout = torch.empty(w.q.shape, dtype=torch.bfloat16).pin_memory()
    hp(hq, hk, hv, hout)
    first = hout.clone()
    used = np.zeros((2, -(-w.k.shape[2] // 880)), dtype=bool)
    for (h0, h1), plan in zip(hp.heads, hp.plans):
        idx, cnt = plan.indices.cpu().numpy(), plan.counts.cpu().numpy()
        for h in range(h1 - h0):
            for qb in range(idx.shape[2]):
                used[h0 + h, idx[0, h, qb, :cnt[0, h, qb]]] = True
    assert not used.all()
    poisoned = hv.clone().pin_memory()
    for h in range(2):
        for b in np.flatnonzero(~used[h]):
            poisoned[0, h, b * 880:(b + 1) * 880] = float("nan")
    hp2 = rcsa.RCSAHostPlan(1, 2, w.q.shape[2], w.k.shape[2], 128, block_size=880, budget=8,
                            groups=2, device="cuda")
    hp2(hq, hk, poisoned, hout)
    assert torch.equal(hout, first)
    assert hp2.last_h2d_bytes == hp.last_h2d_bytes
    # with no gap merging, exactly the selected blocks' rows cross
    hp0 = rcsa.RCSAHostPlan(1, 2, w.q.shape[2], w.k.shape[2], 128, block_size=880, budget=8,
                            groups=2, device="cuda", value_gap=0)
    hp0(hq, hk, poisoned, hout)
    assert torch.equal(hout, first)
    assert hp0.last_h2d_bytes == sum(t.numel() * 2 for t in (hq, hk)) + int(used.sum()) * 880 * 128 * 2


ROW_SAMPLE = np.array([0, 1, 2, 63, 64, 127, 128, 255, 256, 383, 384, 511, 512, 639, 640, 767, 768, 800,
                       860, 879])


def _full_size(w, gold_name):
    """Every head at full size: selection, counts, int8 codes and scales
    bit-exact against the oracle (and the selection against the reference-
    derived golden), attention on 20 sampled rows of every query block of
    every head against the oracle's bf16 path (bf16 and auto policies) and
    its exact int8 simulation (int8 policy)."""
    qd, kd, vd = w.q.cuda(), w.k.cuda(), w.v.cuda()
    results = {}
    for policy in ("bf16", "auto", "int8"):
        out, sel = rcsa.rcsa_attention(qd, kd, vd, block_size=880, budget=w.budget, policy=policy)
        torch.cuda.synchronize()
        results[policy] = (out.cpu(), sel)
    del qd, kd, vd
    sel = results["int8"][1]
    q, k, v = _np(w.q), _np(w.k), _np(w.v)
    o_sel, o_cnt, _, _, _ = orc.rcsa_select(q, k, 880, w.budget)
    np.testing.assert_array_equal(sel.indices.cpu().numpy(), o_sel)
    np.testing.assert_array_equal(sel.counts.cpu().numpy(), o_cnt)
    gold = np.load(os.path.join(GOLDEN, gold_name))
    np.testing.assert_array_equal(o_sel, gold["selected"])
    for policy in ("bf16", "auto"):  # every policy selects the same blocks
        np.testing.assert_array_equal(results[policy][1].indices.cpu().numpy(), o_sel)
    qc, qs = orc.quantize_blocks(q, 880)
    kc, ks = orc.quantize_blocks(k, 880)
    np.testing.assert_array_equal(sel.q_scales.cpu().numpy(), qs)
    np.testing.assert_array_equal(sel.k_scales.cpu().numpy(), ks)
    np.testing.assert_array_equal(sel.q_codes.cpu().numpy(), qc)
    np.testing.assert_array_equal(sel.k_codes.cpu().numpy(), kc)
    ref_b = orc.block_sparse_attention(q, k, v, o_sel, o_cnt, 880, 880, rows=ROW_SAMPLE)
    ref_i = orc.block_sparse_attention(q, k, v, o_sel, o_cnt, 880, 880, q_codes=qc, q_scales=qs,
                                       k_codes=kc, k_scales=ks, rows=ROW_SAMPLE)
    nqb = q.shape[2] // 880
    rows = (np.arange(nqb)[:, None] * 880 + ROW_SAMPLE[None]).reshape(-1)
    errs = {}
    for policy, ref in (("bf16", ref_b), ("auto", ref_b), ("int8", ref_i)):
        got = results[policy][0].float().numpy()[:, :, rows].astype(np.float64)
        d = np.abs(got - ref[:, :, rows])
        errs[policy] = (float(d.max()), float(d.mean()))
        at = np.unravel_index(int(d.argmax()), d.shape)
        print(f"{gold_name} {policy}: max {d.max():.4e} at (b,h,row,d)={tuple(int(x) for x in at)} "
              f"got {got[at]:.5f} ref {ref[:, :, rows][at]:.5f}; |ref| max {np.abs(ref[:, :, rows]).max():.3f}")
        assert d.max() < MAX_ABS and d.mean() < MEAN_ABS, (policy, errs[policy])
    # the pure int8 policy against the bf16 path: measured, reported
    got = results["int8"][0].float().numpy()[:, :, rows].astype(np.float64)
    d = np.abs(got - ref_b[:, :, rows])
    print(f"{gold_name}: errors {errs}; int8 policy vs bf16 path max {d.max():.3e} mean {d.mean():.3e}; "
          f"auto int8 fraction {float(results['auto'][1].qk_mode.float().mean()):.3f}")
    return d


def test_rcsa_config2_all_heads_bitexact(cuda):
    _full_size(workloads.config2(), "cfg2_select_h24.npz")


def test_rcsa_config3_all_heads_bitexact(cuda):
    _full_size(workloads.config3(heads=24), "cfg3_select_h24.npz")


@pytest.mark.parametrize("block", [110, 88, 440])
def test_attention_any_block_size(cuda, block):
    """Blocks that are not multiples of 16 (the compact path's 1x11x10 = 110,
    1x11x8 = 88 and 2x11x20 = 440): key blocks start anywhere in the key
    validity mask (byte loads where the 16-byte ones would be misaligned),
    both precisions, with and without a mask, against the oracle."""
    nq, nh, budget = 2, 5, 2
    q, k, v = _rand_problem(2, nq, nh, block, seed=block)
    g = torch.Generator().manual_seed(block)
    valid = (torch.rand(k.shape[2], generator=g) > 0.15)
    for kv in (None, valid):
        kvd = None if kv is None else kv.to(torch.uint8).cuda()
        sel = rcsa.select_quant(q.cuda(), k.cuda(), block_size=block, budget=budget, policy="int8",
                                k_valid=kvd)
        torch.cuda.synchronize()
        kvn = None if kv is None else kv.numpy()
        o_sel, o_cnt, _, _, _ = orc.rcsa_select(_np(q), _np(k), block, budget, k_valid=kvn)
        assert np.array_equal(sel.indices.cpu().numpy(), o_sel)
        qc, qs = orc.quantize_blocks(_np(q), block)
        kc, ks = orc.quantize_blocks(_np(k), block, kvn)
        ref_b = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, block, block, key_valid=kvn)
        ref_i = orc.block_sparse_attention(_np(q), _np(k), _np(v), o_sel, o_cnt, block, block, key_valid=kvn,
                                           q_codes=qc, q_scales=qs, k_codes=kc, k_scales=ks)
        qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
        out_b = rcsa.block_sparse_attention(qd, kd, vd, sel.indices, sel.counts, q_block=block,
                                            k_block=block, key_valid=kvd)
        out_i = rcsa.block_sparse_attention(qd, kd, vd, sel.indices, sel.counts, q_block=block,
                                            k_block=block, key_valid=kvd, q_codes=sel.q_codes,
                                            q_scales=sel.q_scales, k_codes=sel.k_codes,
                                            k_scales=sel.k_scales)
        torch.cuda.synchronize()
        for out, ref in ((out_b, ref_b), (out_i, ref_i)):
            m, a = _errs(out, ref)
            assert m < MAX_ABS and a < MEAN_ABS, (block, kv is not None, m, a)


def test_unselected_values_never_reach_the_output(cuda):
    """A key block's last 128-row tile reaches 16 rows into the next block
    (880 = 6 x 128 + 112); those rows are masked, and the block-structured
    value map brings them in as zeros.  Non-finite values in every block no
    query block of the head selected leave the output bit-identical."""
    w = workloads.config2(heads=2)
    plan = rcsa.RCSAPlan(1, 2, w.q.shape[2], w.k.shape[2], 128, block_size=880, budget=8, device="cuda")
    q, k, v = w.q.cuda(), w.k.cuda(), w.v.cuda()
    clean = plan(q, k, v).clone()
    idx, cnt = plan.indices.cpu().numpy(), plan.counts.cpu().numpy()
    nkb = w.k.shape[2] // 880
    used = np.zeros((2, nkb), dtype=bool)
    for h in range(2):
        for qb in range(idx.shape[2]):
            used[h, idx[0, h, qb, :cnt[0, h, qb]]] = True
    # some unselected block follows a selected one (its first rows are read)
    assert any(used[h, b] and not used[h, b + 1] for h in range(2) for b in range(nkb - 1))
    vp = v.clone()
    for h in range(2):
        for b in np.flatnonzero(~used[h]):
            vp[0, h, b * 880:(b + 1) * 880] = float("nan") if b % 2 else float("inf")
    dirty = plan(q, k, vp)
    torch.cuda.synchronize()
    assert torch.equal(dirty, clean)


@pytest.mark.parametrize("config", [2, 3])
@pytest.mark.parametrize("policy", ["int8", "auto", "bf16"])
def test_every_output_row_is_written(cuda, config, policy):
    """Every query row of the layer gets its output, whatever work split the
    planner chose: an output buffer filled with NaN comes back finite."""
    w = workloads.config2() if config == 2 else workloads.config3(heads=24)
    q, k, v = w.q.cuda(), w.k.cuda(), w.v.cuda()
    plan = rcsa.RCSAPlan(1, q.shape[1], q.shape[2], k.shape[2], 128, block_size=880, budget=w.budget,
                         policy=policy, device=cuda)
    plan.select(q, k)
    out = torch.full_like(q, float("nan"))
    plan.attend(q, k, v, out=out)
    plan.check()
    bad = ~torch.isfinite(out)
    if bad.any():
        h, r, _ = (int(x) for x in torch.nonzero(bad[0])[0])
        pytest.fail(f"{int(bad.sum())} outputs not written, first at head {h} row {r}")
