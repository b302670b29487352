"""Compact-layout packing with the RoPE phase (B200 kernels).

Host side of ``cast_compact_pack`` / ``cast_compact_unpack`` for the compact
selection / attention path of the frame weave:

* :func:`pack` replaces, for one layer call, the RoPE rotation
  ``MatrixCurvaturePhaseFrameWeave._apply_compact_rope_phase`` of q and k
  (``proposed/matrix_curvature_phase_frame_weave.py:5565-5574``) and the
  packing in ``_compact_cwca_attention`` (:5677-5684) with the bf16 cast of
  the attention launch: one pass over q, k and v.
* :func:`unpack` replaces ``output_packed[:, token_to_packed]`` (:6095).
"""

from __future__ import annotations

import torch

from . import _lib
from .rcsa import _need_cuda, _stream


def layout_indices(block_indices: torch.Tensor) -> torch.Tensor:
    """The reference's ``compact_block_indices`` ([blocks, block_size] long,
    -1 padding) as the flat int32 slot -> token map the kernel takes."""
    return block_indices.reshape(-1).to(torch.int32).contiguous()


def phase_pairs(phase: torch.Tensor) -> torch.Tensor:
    """The reference's complex RoPE phase ``[L, Hp, D/2]`` (or ``[L, D/2]``)
    as contiguous float32 (re, im) pairs."""
    if phase.dim() == 2:
        phase = phase.unsqueeze(1)
    return torch.view_as_real(phase.to(torch.complex64)).contiguous()


def pack(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor,
         phase: torch.Tensor | None = None, out=None):
    """``q, k, v`` ``[B,L,H,128]`` (bf16 or fp32, token order) -> packed bf16
    ``[B,H,P,128]`` each: q and k rotated by ``phase`` (complex ``[L,Hp,64]``,
    Hp 1 or H; None: no rotation), gathered by ``block_indices`` (int32
    ``[P]`` or the reference's ``[blocks, block_size]``; -1 = padding, written
    as zeros)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _need_cuda(name, t, None, 4)
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("q, k and v must share dtype bf16 or float32")
    if not (q.shape == k.shape == v.shape):
        raise ValueError("q, k and v shapes differ")
    b, l, h, d = q.shape
    idx = block_indices if block_indices.dtype == torch.int32 and block_indices.dim() == 1 \
        else layout_indices(block_indices)
    _need_cuda("block_indices", idx, torch.int32, 1)
    p = idx.numel()
    ph, ph_heads = None, 1
    if phase is not None:
        ph = phase if phase.dtype == torch.float32 and phase.dim() == 4 else phase_pairs(phase)
        _need_cuda("phase", ph, torch.float32, 4)
        if ph.shape[0] != l or ph.shape[2] != d // 2 or ph.shape[1] not in (1, h):
            raise ValueError("phase must be [L, 1 or H, D/2]")
        ph_heads = ph.shape[1]
    if out is None:
        out = tuple(torch.empty(b, h, p, d, dtype=torch.bfloat16, device=q.device) for _ in range(3))
    P = _lib.ptr
    _lib.call("cast_compact_pack", P(q), P(k), P(v), 0 if q.dtype == torch.bfloat16 else 1, P(ph),
              ph_heads, P(idx), b, l, h, d, p, P(out[0]), P(out[1]), P(out[2]), _stream(q.device))
    return out


def unpack(packed: torch.Tensor, token_to_packed: torch.Tensor, out: torch.Tensor | None = None):
    """bf16 ``[B,H,P,D]`` -> ``[B,L,H,D]`` with ``out[:, t] = packed[:, :, token_to_packed[t]]``."""
    _need_cuda("packed", packed, torch.bfloat16, 4)
    ttp = token_to_packed if token_to_packed.dtype == torch.int32 else token_to_packed.to(torch.int32)
    ttp = ttp.contiguous()
    _need_cuda("token_to_packed", ttp, torch.int32, 1)
    b, h, p, d = packed.shape
    l = ttp.numel()
    if out is None:
        out = torch.empty(b, l, h, d, dtype=torch.bfloat16, device=packed.device)
    P = _lib.ptr
    _lib.call("cast_compact_unpack", P(packed), P(ttp), b, l, h, d, p, P(out), _stream(packed.device))
    return out
