"""CPU: the auto policy's int8 QK^T choice against the exact softmax.

The selection kernel gives a (b, h, query block) int8 QK^T where the
predicted logit error of the int8 product (uniform quantisation noise of the
per-block scales, times the logit spread) is at most the tolerance.  On
config 2 and config 3 at full size (all 24 heads), every query block that
choice sends to int8 must keep the exact int8 simulation, rounded to the bf16
output, within half the 2e-2 output bar of the exact softmax on the sampled
rows the GPU parity tests read."""

import numpy as np
import pytest
import torch

from cast_b200 import rcsa, workloads
from oracle import rcsa as orc

ROWS = np.array([0, 1, 2, 63, 64, 127, 128, 255, 256, 383, 384, 511, 512, 639, 640, 767, 768, 800, 860, 879])


def predicted_error(q, k, qs, ks, sel, cnt):
    """The kernel's predictor (select_quant.cuh, budget_select_kernel) per
    (head, query block): max over the selected key blocks of
    sqrt((s_q^2 r_k^2 + s_k^2 r_q^2) / 12) * r_q * r_k with block RMS r and
    int8 scale s."""
    B, H, Lq, D = q.shape
    nqb, nkb = -(-Lq // 880), -(-k.shape[2] // 880)
    rq = np.sqrt((q.reshape(B, H, nqb, -1).astype(np.float64) ** 2).mean(-1))
    rk = np.sqrt((k.reshape(B, H, nkb, -1).astype(np.float64) ** 2).mean(-1))
    out = np.zeros((H, nqb))
    for h in range(H):
        for qb in range(nqb):
            b = sel[0, h, qb, :cnt[0, h, qb]]
            e = np.sqrt((qs[0, h, qb] ** 2 * rk[0, h, b] ** 2 + ks[0, h, b] ** 2 * rq[0, h, qb] ** 2) / 12)
            out[h, qb] = float((e * rq[0, h, qb] * rk[0, h, b]).max())
    return out


@pytest.mark.parametrize("name,min_fraction", [("cfg2", 0.45), ("cfg3", 0.25)])
def test_auto_int8_blocks_within_half_the_bar(name, min_fraction):
    w = workloads.config2() if name == "cfg2" else workloads.config3(heads=24)
    q, k, v = (t.float().numpy() for t in (w.q, w.k, w.v))
    sel, cnt, *_ = orc.rcsa_select(q, k, 880, w.budget)
    qc, qs = orc.quantize_blocks(q, 880)
    kc, ks = orc.quantize_blocks(k, 880)
    pred = predicted_error(q, k, qs, ks, sel, cnt)
    chosen = pred <= rcsa.DEFAULT_INT8_TOLERANCE
    assert chosen.mean() >= min_fraction
    exact = orc.block_sparse_attention(q, k, v, sel, cnt, 880, 880, rows=ROWS)
    int8 = orc.block_sparse_attention(q, k, v, sel, cnt, 880, 880, rows=ROWS, q_codes=qc, q_scales=qs,
                                      k_codes=kc, k_scales=ks)
    rounded = torch.from_numpy(int8.astype(np.float32)).bfloat16().double().numpy()
    for h, qb in zip(*np.nonzero(chosen)):
        r = qb * 880 + ROWS
        err = np.abs(rounded[0, h, r] - exact[0, h, r])
        assert err.max() < 1e-2, (h, qb, pred[h, qb], err.max())
