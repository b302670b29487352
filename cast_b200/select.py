"""Full-layer pooled-QK selection (TABA ``select``) on B200.

``TABASelector.select`` keeps the signature and result of
``MatrixTrajectoryAdaptiveBudgetAttentionCompiler.select``
(``proposed/qk_uncertainty_tangent_attention.py:988-1082``): pooled block
means over the ``(tt,th,tw)`` visual tiling (``_tile_visual_tensor``,
``proposed/reciprocal_joint_attention.py:64-103``), cosine scores, a ``+1e6``
bonus on the Manhattan-<=1 block stencil, a stable descending order truncated
to ``max(row_degrees)``.  The per-row degrees come from the compiler's
geometry step (``compile``), which stays host-side; set them with
:meth:`set_row_degrees` or copy them from a compiled reference instance.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from .rcsa import Workspace, _need_cuda, _stream


@dataclass
class SelectionReport:
    """Subset of ``QKUncertaintyTangentSelectionReport`` computed on device."""

    batch_heads: int
    query_rows: int
    budget_min: int
    budget_max: int
    budget_total: int


class TABASelector:
    def __init__(self, block_shape: tuple[int, int, int] = (4, 4, 8)):
        self._block_shape = tuple(int(x) for x in block_shape)
        self._row_degrees: torch.Tensor | None = None
        self._num_blocks: int | None = None
        self._ws = Workspace()

    def set_row_degrees(self, row_degrees: torch.Tensor, block_shape=None) -> None:
        if block_shape is not None:
            self._block_shape = tuple(int(x) for x in block_shape)
        rd = torch.as_tensor(row_degrees).to(torch.int64)
        if rd.ndim != 1 or len(rd) == 0 or int(rd.min()) <= 0:
            raise ValueError("row degrees must be a non-empty positive vector")
        self._row_degrees = rd.cpu()
        self._num_blocks = len(rd)

    @classmethod
    def from_reference(cls, compiler) -> "TABASelector":
        """Copies the compiled budget of a reference TABA compiler instance."""
        sel = cls(compiler._block_shape)
        sel.set_row_degrees(compiler._row_degrees)
        return sel

    def select(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        *,
        geometry_indices: torch.Tensor | None,
        geometry_counts: torch.Tensor | None,
        latent_hw: tuple[int, int],
        block_shape: tuple[int, int, int],
        return_scores: bool = False,
    ):
        del geometry_indices, geometry_counts
        if q.shape != k.shape or q.ndim != 4:
            raise ValueError("TABA requires equal B,H,L,D Q/K")
        if self._row_degrees is None:
            raise RuntimeError("TABA budgets were not compiled")
        if tuple(int(x) for x in block_shape) != self._block_shape:
            raise RuntimeError("TABA runtime block shape differs from compilation")
        q = q.to(torch.bfloat16).contiguous()
        k = k.to(torch.bfloat16).contiguous()
        _need_cuda("q", q, torch.bfloat16, 4)
        _need_cuda("k", k, torch.bfloat16, 4)
        b, h, length, d = q.shape
        hl, wl = (int(x) for x in latent_hw)
        if length % (hl * wl):
            raise ValueError("Q/K tokens do not define an integral temporal grid")
        t = length // (hl * wl)
        tt, th, tw = self._block_shape
        nblocks = math.ceil(t / tt) * math.ceil(hl / th) * math.ceil(wl / tw)
        if nblocks != self._num_blocks:
            raise RuntimeError("tiled Q/K count differs from compiled geometry")
        rd = self._row_degrees
        maxdeg = int(rd.max())
        dev = q.device
        rd_dev = rd.to(device=dev, dtype=torch.int32)
        sel = torch.empty(b, h, nblocks, maxdeg, dtype=torch.int32, device=dev)
        cnt = torch.empty(b, h, nblocks, dtype=torch.int32, device=dev)
        scores = torch.empty(b, h, nblocks, nblocks, dtype=torch.float64, device=dev) if return_scores else None
        lib = _lib.load()
        nbytes = lib.cast_taba_select_workspace_bytes(b, h, t, hl, wl, d, tt, th, tw)
        ws = self._ws.get(dev, nbytes)
        P = _lib.ptr
        _lib.call("cast_taba_select", P(q), P(k), b, h, t, hl, wl, d, tt, th, tw, P(rd_dev), maxdeg,
                  P(sel), P(cnt), P(scores), P(ws), ws.numel(), _stream(dev))
        report = SelectionReport(b * h, nblocks, int(rd.min()), maxdeg, int(rd.sum()))
        if return_scores:
            return sel, cnt, report, scores
        return sel, cnt, report
