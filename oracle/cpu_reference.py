"""The reference's PyTorch CPU path for the RCSA layer -- TEST/BASELINE ONLY.

Used by ``bench.py`` as the timed CPU baseline (``cpu_baseline`` and
``--impl reference``) because the reference package itself is not present on
the GPU host.  It performs the reference's own operations, in its own float32
arithmetic and with torch's multi-threaded CPU kernels:

* pooled selection: block means over contiguous frame blocks,
  ``F.normalize``, ``matmul`` of pooled Q and K
  (``proposed/qk_uncertainty_tangent_attention.py:1011-1023``), stable
  descending ``argsort`` over the historical blocks (``:978-980``), then the
  block-causal current blocks;
* attention: the reference's explicit softmax over the allowed keys
  (``proposed/matrix_jit_spatial_acceleration.py:836-858``) -- bf16-rounded
  q/k/v upcast to float32, ``softmax(q k^T / sqrt(d)) v``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rcsa_layer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block: int, budget: int,
               heads: list[int] | None = None) -> torch.Tensor:
    """One RCSA layer call on CPU for the given heads; returns float32 output."""
    b, h, lq, d = q.shape
    lk = k.shape[2]
    nqb, nkb = lq // block, lk // block
    nhist = nkb - nqb
    keep = min(budget, nhist)
    hs = list(range(h)) if heads is None else heads
    out = torch.zeros(b, len(hs), lq, d)
    for oi, hi in enumerate(hs):
        qh = q[:, hi].float()
        kh = k[:, hi].float()
        vh = v[:, hi].float()
        qn = F.normalize(qh.reshape(b, nqb, block, d).mean(dim=2), dim=-1)
        kn = F.normalize(kh.reshape(b, nkb, block, d).mean(dim=2), dim=-1)
        score = torch.matmul(qn, kn.transpose(-2, -1))
        order = torch.argsort(score[..., :nhist], dim=-1, descending=True, stable=True)[..., :keep]
        for i in range(nqb):
            blocks = order[0, i].tolist() + list(range(nhist, nhist + i + 1))
            keys = torch.cat([torch.arange(bk * block, (bk + 1) * block) for bk in blocks])
            logits = qh[0, i * block:(i + 1) * block] @ kh[0, keys].T / math.sqrt(d)
            w = torch.softmax(logits, dim=-1)
            out[0, oi, i * block:(i + 1) * block] = w @ vh[0, keys]
    return out
