"""Host side of Reconstruction-Coupled Sparse Attention (RCSA) on B200.

Mirrors the reference's operator seams:

* ``longcat_active`` / ``longcat_asymmetric`` -- drop-ins for
  ``MatrixJiTSpatialAcceleration._longcat_active``
  (``proposed/matrix_jit_spatial_acceleration.py:663-729``) and
  ``MatrixCausalFrameLayerRelay._longcat_asymmetric``
  (``proposed/matrix_curvature_phase_frame_weave.py:8847-8917``): same
  arguments, same bf16 ``[B,H,L,D]`` result.
* ``select_quant`` -- pooled-QK block scoring with the historical-budget +
  block-causal rule, fused with per-block symmetric int8 quantisation.
* ``rcsa_attention`` -- selection, quantisation and the int8/bf16 tcgen05
  block-sparse attention in one call.

Every function runs the CUDA kernels of ``libcast_b200.so`` on the current
CUDA stream; there is no CPU path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

import torch

from . import _lib

POLICIES = {"bf16": 0, "int8": 1, "auto": 2}
DEFAULT_INT8_TOLERANCE = 0.035
RULE_BUDGET_CAUSAL = 0


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(name: str, t: torch.Tensor, dtype: torch.dtype | None = None, ndim: int | None = None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the RCSA hot path has no CPU implementation)")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.ndim != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


@dataclass
class Selection:
    """Outputs of :func:`select_quant` (device tensors)."""

    indices: torch.Tensor          # int32 [B,H,nQb,maxdeg], -1 padded
    counts: torch.Tensor           # int32 [B,H,nQb]
    q_codes: torch.Tensor | None   # int8 [B,H,Lq,D]
    q_scales: torch.Tensor | None  # float32 [B,H,nQb]
    k_codes: torch.Tensor | None   # int8 [B,H,Lk,D]
    k_scales: torch.Tensor | None  # float32 [B,H,nKb]
    v_codes: torch.Tensor | None
    v_scales: torch.Tensor | None
    qk_mode: torch.Tensor | None   # uint8 [B,H,nQb]: 1 int8, 0 bf16
    pooled: torch.Tensor | None    # float64 [B,H,nQb+nKb,D]

    @property
    def max_degree(self) -> int:
        return int(self.indices.shape[-1])


class Workspace:
    """Caller-owned scratch buffer reused across calls (grown on demand)."""

    def __init__(self):
        self._buf: dict[torch.device, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int, zero: bool = False) -> torch.Tensor:
        """A buffer of at least ``nbytes``; ``zero``: zero-filled when (re)allocated."""
        buf = self._buf.get(device)
        if buf is None or buf.numel() < nbytes:
            alloc = torch.zeros if zero else torch.empty
            buf = alloc(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._buf[device] = buf
        return buf


_default_ws = Workspace()
# Attention workspaces hold arrival counters that every completed call leaves
# at zero, so they are zero-filled once and never shared with other kernels.
_attn_ws = Workspace()


def budget_count_hint(B: int, H: int, nqb: int, nkb: int, budget: int) -> np.ndarray:
    """Key blocks per (b, h, query block) under the historical-budget +
    block-causal rule: ``min(budget, nkb - nqb)`` history blocks plus current
    blocks ``0..i`` (host int32 ``[B,H,nQb]``, the attention's balance hint)."""
    keep = min(budget, nkb - nqb)
    per_qb = keep + 1 + np.arange(nqb, dtype=np.int32)
    return np.ascontiguousarray(np.broadcast_to(per_qb, (B, H, nqb)).astype(np.int32))


def _attention_workspace(b, h, lq, lk, q_block, k_block, max_degree, hint, device, workspace):
    nbytes = int(_lib.load().cast_rcsa_attention_workspace_bytes(
        b, h, lq, lk, q_block, k_block, max_degree, None if hint is None else hint.ctypes.data))
    if nbytes == 0:
        return None, 0
    return (workspace or _attn_ws).get(device, nbytes, zero=True), nbytes


def select_quant(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor | None = None,
    *,
    block_size: int,
    budget: int,
    policy: str = "auto",
    int8_tolerance: float = DEFAULT_INT8_TOLERANCE,
    quantize: bool = True,
    quantize_v: bool = False,
    return_pooled: bool = False,
    q_valid: torch.Tensor | None = None,
    k_valid: torch.Tensor | None = None,
    workspace: Workspace | None = None,
) -> Selection:
    """Pooled-QK block selection fused with per-block int8 quantisation.

    ``q``: bf16 ``[B,H,Lq,D]`` (current chunk); ``k``/``v``: bf16
    ``[B,H,Lk,D]`` with history blocks first and the chunk's own blocks last.
    Selection: per (b, h, query block i) the ``budget`` historical blocks of
    highest pooled cosine (``F.normalize(mean)`` dot product, as
    ``proposed/qk_uncertainty_tangent_attention.py:1021-1042``; ties to the
    lower index), then current blocks ``0..i``.
    ``q_valid`` / ``k_valid``: optional uint8 ``[Lq]`` / ``[Lk]`` token
    validity of the compact packing (the same for every (b, h)); invalid
    tokens count as zero in a block's sums and amax, leave its pooled-mean
    denominator and get code 0
    (``proposed/matrix_curvature_phase_frame_weave.py:5696-5699``).
    """
    if policy not in POLICIES:
        raise ValueError(f"policy must be one of {sorted(POLICIES)}")
    _need_cuda("q", q, torch.bfloat16, 4)
    _need_cuda("k", k, torch.bfloat16, 4)
    if v is not None:
        _need_cuda("v", v, torch.bfloat16, 4)
    b, h, lq, d = q.shape
    lk = k.shape[2]
    if k.shape[:2] != (b, h) or k.shape[3] != d:
        raise ValueError(f"k shape {tuple(k.shape)} incompatible with q {tuple(q.shape)}")
    if q_valid is not None:
        _need_cuda("q_valid", q_valid, torch.uint8, 1)
        if q_valid.numel() != lq:
            raise ValueError("q_valid must have Lq entries")
    if k_valid is not None:
        _need_cuda("k_valid", k_valid, torch.uint8, 1)
        if k_valid.numel() != lk:
            raise ValueError("k_valid must have Lk entries")
    nqb, nkb = -(-lq // block_size), -(-lk // block_size)
    keep = min(budget, nkb - nqb)
    dev = q.device
    idx = torch.empty(b, h, nqb, keep + nqb, dtype=torch.int32, device=dev)
    cnt = torch.empty(b, h, nqb, dtype=torch.int32, device=dev)
    qc = torch.empty_like(q, dtype=torch.int8) if quantize else None
    kc = torch.empty_like(k, dtype=torch.int8) if quantize else None
    qs = torch.empty(b, h, nqb, dtype=torch.float32, device=dev) if quantize else None
    ks = torch.empty(b, h, nkb, dtype=torch.float32, device=dev) if quantize else None
    vc = torch.empty_like(v, dtype=torch.int8) if (quantize_v and v is not None) else None
    vs = torch.empty(b, h, nkb, dtype=torch.float32, device=dev) if vc is not None else None
    mode = torch.empty(b, h, nqb, dtype=torch.uint8, device=dev) if quantize else None
    pooled = torch.empty(b, h, nqb + nkb, d, dtype=torch.float64, device=dev) if return_pooled else None
    lib = _lib.load()
    nbytes = lib.cast_rcsa_select_quant_workspace_bytes(b, h, lq, lk, d, block_size)
    ws = (workspace or _default_ws).get(dev, nbytes)
    P = _lib.ptr
    _lib.call(
        "cast_rcsa_select_quant", P(q), P(k), P(v) if vc is not None else None, P(q_valid), P(k_valid),
        b, h, lq, lk, d,
        block_size, budget, RULE_BUDGET_CAUSAL, P(idx), P(cnt), P(qc), P(qs), P(kc), P(ks), P(vc),
        P(vs), P(mode), POLICIES[policy], float(int8_tolerance), P(pooled), P(ws), ws.numel(),
        _stream(dev),
    )
    return Selection(idx, cnt, qc, qs, kc, ks, vc, vs, mode, pooled)


def block_sparse_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    indices: torch.Tensor,
    counts: torch.Tensor,
    *,
    q_block: int,
    k_block: int,
    key_valid: torch.Tensor | None = None,
    sm_scale: float | None = None,
    q_codes: torch.Tensor | None = None,
    q_scales: torch.Tensor | None = None,
    k_codes: torch.Tensor | None = None,
    k_scales: torch.Tensor | None = None,
    qk_mode: torch.Tensor | None = None,
    return_lse: bool = False,
    out: torch.Tensor | None = None,
    count_hint=None,
    balance: bool = True,
    workspace: Workspace | None = None,
):
    """Block-sparse attention over listed key blocks (tcgen05, sm_100a).

    ``O = softmax(Q K^T * sm_scale) V`` per query row over the keys of blocks
    ``indices[b,h,i,:counts[b,h,i]]`` with ``key_valid`` (uint8 ``[Lk]``)
    set.  ``sm_scale`` defaults to ``1/sqrt(D)`` as the reference launch does.
    With int8 codes/scales the QK^T product runs in int8 where ``qk_mode`` is 1.
    ``balance`` cuts the items that would run last into key-tile parts merged
    on the device (a zero-filled attention ``workspace``); ``count_hint``
    (host ints ``[B,H,nQb]``, default ``max_degree``) is the expected
    ``counts``, used only for that balance.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _need_cuda(name, t, torch.bfloat16, 4)
    _need_cuda("indices", indices, torch.int32, 4)
    _need_cuda("counts", counts, torch.int32, 3)
    if key_valid is not None:
        _need_cuda("key_valid", key_valid, torch.uint8, 1)
    b, h, lq, d = q.shape
    lk = k.shape[2]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty_like(q)
    lse = torch.empty(b, h, lq, dtype=torch.float32, device=q.device) if return_lse else None
    max_degree = int(indices.shape[-1])
    hint, ws, nbytes = None, None, 0
    if balance:
        if count_hint is not None:
            hint = np.ascontiguousarray(np.asarray(count_hint, dtype=np.int32).reshape(-1))
            if hint.size != b * h * (-(-lq // q_block)):
                raise ValueError("count_hint must have B*H*nQb entries")
        ws, nbytes = _attention_workspace(b, h, lq, lk, q_block, k_block, max_degree, hint,
                                          q.device, workspace)
    P = _lib.ptr
    _lib.call(
        "cast_rcsa_attention", P(q), P(k), P(v), P(q_codes), P(q_scales), P(k_codes), P(k_scales),
        P(qk_mode), P(indices), P(counts), max_degree, P(key_valid), b, h, lq, lk, d,
        q_block, k_block, float(sm_scale), P(out), P(lse),
        None if hint is None else hint.ctypes.data, P(ws), nbytes, _stream(q.device),
    )
    return (out, lse) if return_lse else out


def longcat_active(q, k, v, indices, counts, valid, block_size):
    """Drop-in for ``MatrixJiTSpatialAcceleration._longcat_active``.

    Same arguments and result as the reference launch of the block-sparse
    kernel (``proposed/matrix_jit_spatial_acceleration.py:663-729``): bf16
    ``[B,H,L,D]`` q/k/v, int32 block indices/counts, a ``[nBlocks,S]`` key
    validity mask, square blocks of ``block_size``, ``sm_scale = 1/sqrt(D)``.
    """
    q = q.to(torch.bfloat16).contiguous()
    k = k.to(torch.bfloat16).contiguous()
    v = v.to(torch.bfloat16).contiguous()
    indices = indices.to(torch.int32).contiguous()
    counts = counts.to(torch.int32).contiguous()
    key_valid = valid.reshape(-1).to(torch.uint8).contiguous()
    return block_sparse_attention(q, k, v, indices, counts, q_block=block_size,
                                  k_block=block_size, key_valid=key_valid)


def longcat_asymmetric(q, k, v, indices, counts, key_valid, *, query_block_size, key_block_size):
    """Drop-in for ``MatrixCausalFrameLayerRelay._longcat_asymmetric``
    (``proposed/matrix_curvature_phase_frame_weave.py:8847-8917``)."""
    q = q.to(torch.bfloat16).contiguous()
    k = k.to(torch.bfloat16).contiguous()
    v = v.to(torch.bfloat16).contiguous()
    if q.shape[2] % query_block_size or k.shape[2] % key_block_size:
        raise RuntimeError("asymmetric sparse storage is not block aligned")
    return block_sparse_attention(
        q, k, v, indices.to(torch.int32).contiguous(), counts.to(torch.int32).contiguous(),
        q_block=query_block_size, k_block=key_block_size,
        key_valid=key_valid.reshape(-1).to(torch.uint8).contiguous(),
    )


def rcsa_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    block_size: int,
    budget: int,
    policy: str = "auto",
    int8_tolerance: float = DEFAULT_INT8_TOLERANCE,
    sm_scale: float | None = None,
    workspace: Workspace | None = None,
):
    """Full RCSA step: select + quantise, then block-sparse attention.

    Returns ``(out bf16 [B,H,Lq,D], Selection)``.  ``policy`` picks the QK^T
    precision per (b, h, query block): ``"int8"`` everywhere, ``"bf16"``
    everywhere, or ``"auto"`` (int8 where the predicted logit error of the
    int8 product, times the logit spread, stays below ``int8_tolerance``).
    """
    sel = select_quant(q, k, None, block_size=block_size, budget=budget, policy=policy,
                       int8_tolerance=int8_tolerance, quantize=policy != "bf16",
                       workspace=workspace)
    b, h, lq, _ = q.shape
    nqb, nkb = -(-lq // block_size), -(-k.shape[2] // block_size)
    out = block_sparse_attention(
        q, k, v, sel.indices, sel.counts, q_block=block_size, k_block=block_size,
        sm_scale=sm_scale, q_codes=sel.q_codes, q_scales=sel.q_scales, k_codes=sel.k_codes,
        k_scales=sel.k_scales, qk_mode=sel.qk_mode,
        count_hint=budget_count_hint(b, h, nqb, nkb, budget),
    )
    return out, sel


class RCSAPlan:
    """Preallocated RCSA layer call for a fixed problem shape.

    Holds every output and scratch buffer (indices, counts, int8 codes, scales,
    precision modes, workspace, attention output), so repeated calls allocate
    nothing and can be captured in a CUDA graph (:meth:`capture`).  This is the
    B200 counterpart of the reference's cached per-shape workspaces.
    """

    def __init__(self, B: int, H: int, Lq: int, Lk: int, D: int, *, block_size: int,
                 budget: int, policy: str = "auto",
                 int8_tolerance: float = DEFAULT_INT8_TOLERANCE, device=None):
        if policy not in POLICIES:
            raise ValueError(f"policy must be one of {sorted(POLICIES)}")
        dev = torch.device(device if device is not None else "cuda")
        self.shape = (B, H, Lq, Lk, D)
        self.block_size, self.budget, self.policy = block_size, budget, policy
        self.int8_tolerance = float(int8_tolerance)
        nqb, nkb = -(-Lq // block_size), -(-Lk // block_size)
        keep = min(budget, nkb - nqb)
        quant = policy != "bf16"
        self.indices = torch.empty(B, H, nqb, keep + nqb, dtype=torch.int32, device=dev)
        self.counts = torch.empty(B, H, nqb, dtype=torch.int32, device=dev)
        self.q_codes = torch.empty(B, H, Lq, D, dtype=torch.int8, device=dev) if quant else None
        self.k_codes = torch.empty(B, H, Lk, D, dtype=torch.int8, device=dev) if quant else None
        self.q_scales = torch.empty(B, H, nqb, dtype=torch.float32, device=dev) if quant else None
        self.k_scales = torch.empty(B, H, nkb, dtype=torch.float32, device=dev) if quant else None
        self.qk_mode = torch.empty(B, H, nqb, dtype=torch.uint8, device=dev) if quant else None
        self.out = torch.empty(B, H, Lq, D, dtype=torch.bfloat16, device=dev)
        nbytes = _lib.load().cast_rcsa_select_quant_workspace_bytes(B, H, Lq, Lk, D, block_size)
        self.workspace = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
        # attention: expected counts of the rule (balance hint) and its own
        # zero-filled workspace of arrival counters and partial results
        self.count_hint = budget_count_hint(B, H, nqb, nkb, budget)
        with torch.cuda.device(dev):
            nbytes = int(_lib.load().cast_rcsa_attention_workspace_bytes(
                B, H, Lq, Lk, block_size, block_size, keep + nqb, self.count_hint.ctypes.data))
        self.attn_workspace = (torch.zeros(nbytes, dtype=torch.uint8, device=dev)
                               if nbytes else None)
        self.sm_scale = 1.0 / math.sqrt(D)
        self.device = dev

    def select(self, q: torch.Tensor, k: torch.Tensor) -> None:
        B, H, Lq, Lk, D = self.shape
        if tuple(q.shape) != (B, H, Lq, D) or tuple(k.shape) != (B, H, Lk, D):
            raise ValueError("q/k shapes differ from the plan")
        _need_cuda("q", q, torch.bfloat16, 4)
        _need_cuda("k", k, torch.bfloat16, 4)
        P = _lib.ptr
        _lib.call(
            "cast_rcsa_select_quant", P(q), P(k), None, None, None, B, H, Lq, Lk, D, self.block_size,
            self.budget, RULE_BUDGET_CAUSAL, P(self.indices), P(self.counts), P(self.q_codes),
            P(self.q_scales), P(self.k_codes), P(self.k_scales), None, None, P(self.qk_mode),
            POLICIES[self.policy], self.int8_tolerance, None, P(self.workspace),
            self.workspace.numel(), _stream(self.device),
        )

    def attend(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               out: torch.Tensor | None = None, peers=None) -> torch.Tensor:
        """Attention with the last selection; into ``out`` (bf16 ``[B,H,Lq,D]``)
        when given, else into the plan's own output buffer.  ``peers``: the
        fused all-gather's arguments ``(n_peers, peer_out, peer_flag,
        done_ticket, calls)`` (see :class:`cast_b200.distributed.PeerGather`),
        which store every output row into the peers' gathered buffers too."""
        B, H, Lq, Lk, D = self.shape
        _need_cuda("v", v, torch.bfloat16, 4)
        if out is None:
            out = self.out
        elif tuple(out.shape) != (B, H, Lq, D):
            raise ValueError("out shape differs from the plan")
        else:
            _need_cuda("out", out, torch.bfloat16, 4)
        P = _lib.ptr
        args = (P(q), P(k), P(v), P(self.q_codes), P(self.q_scales),
                P(self.k_codes), P(self.k_scales), P(self.qk_mode), P(self.indices), P(self.counts),
                int(self.indices.shape[-1]), None, B, H, Lq, Lk, D, self.block_size, self.block_size,
                float(self.sm_scale), P(out), None, self.count_hint.ctypes.data,
                P(self.attn_workspace),
                0 if self.attn_workspace is None else self.attn_workspace.numel())
        if peers is None:
            _lib.call("cast_rcsa_attention", *args, _stream(self.device))
        else:
            _lib.call("cast_rcsa_attention_peers", *args, *peers, _stream(self.device))
        return out

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        self.select(q, k)
        return self.attend(q, k, v)

    def selection(self) -> Selection:
        return Selection(self.indices, self.counts, self.q_codes, self.q_scales, self.k_codes,
                         self.k_scales, None, None, self.qk_mode, None)

    def check(self) -> None:
        """Waits for the plan's stream and raises :class:`cast_b200._lib.CastError`
        if a kernel reported a device-side error (a bounded wait that gave up,
        an index out of range) since the last check; the outputs of such a
        call are not valid."""
        _lib.check_device(_stream(self.device), "RCSAPlan")

    def capture(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, parts: str = "all",
                out: torch.Tensor | None = None):
        """CUDA graph of one call on these input buffers (``parts``: all,
        select or attend; the attention writes ``out`` when given).  Replaying
        it recomputes from the buffers' current contents."""
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._run_parts(q, k, v, parts, out)  # warm the launch paths on this stream
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(g, stream=s):
            self._run_parts(q, k, v, parts, out)
        return g

    def _run_parts(self, q, k, v, parts, out=None):
        if parts in ("all", "select"):
            self.select(q, k)
        if parts in ("all", "attend"):
            self.attend(q, k, v, out)


class RCSAHostPlan:
    """An RCSA layer call whose inputs and output live in pinned host memory.

    The heads are split into ``groups`` contiguous groups, each with its own
    :class:`RCSAPlan`.  Group g's Q and K cross to the device on one copy
    stream, its selection runs on the caller's stream once they are in, and
    its attention once its values are in; its device-to-host copy runs on a
    second copy stream once its attention is done -- so the copies of one
    group overlap the compute of another, and the two copy directions overlap
    each other.

    Values: with ``v_selected`` (the default) only the value blocks some
    query block of the head selected cross the link (the attention reads no
    others): the call reads each group's selection back as soon as it is
    made and copies the union of its blocks, one copy per run of consecutive
    blocks (runs ``value_gap`` or fewer blocks apart merged); the other blocks of the device buffer keep earlier contents,
    which are finite (the buffer starts zeroed), so the masked rows a key
    tile reads past its block's end contribute exact zeros.  Without it the
    whole value tensor is copied before the selection.

    The call returns with the output copy ordered before anything the caller
    enqueues next on its stream; ``last_h2d_bytes`` / ``last_d2h_bytes`` are
    the bytes it moved.  Batch size 1 (a head slice of ``[1,H,L,D]`` is
    contiguous).
    """

    def __init__(self, B: int, H: int, Lq: int, Lk: int, D: int, *, block_size: int,
                 budget: int, policy: str = "auto", groups: int = 4,
                 int8_tolerance: float = DEFAULT_INT8_TOLERANCE, device=None,
                 v_selected: bool = True, value_gap: int = 2, copy_streams: int = 1):
        if B != 1:
            raise ValueError("RCSAHostPlan takes batch size 1 (contiguous head slices)")
        dev = torch.device(device if device is not None else "cuda")
        groups = max(1, min(int(groups), H))
        bounds = [H * g // groups for g in range(groups + 1)]
        self.heads = [(bounds[g], bounds[g + 1]) for g in range(groups)]
        self.plans = [RCSAPlan(B, h1 - h0, Lq, Lk, D, block_size=block_size, budget=budget,
                               policy=policy, int8_tolerance=int8_tolerance, device=dev)
                      for h0, h1 in self.heads]
        self.q = torch.empty(B, H, Lq, D, dtype=torch.bfloat16, device=dev)
        self.k = torch.empty(B, H, Lk, D, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros(B, H, Lk, D, dtype=torch.bfloat16, device=dev)
        self.out = torch.empty(B, H, Lq, D, dtype=torch.bfloat16, device=dev)
        # host-to-device copy streams (more than one spreads the copies over
        # the device's copy engines)
        self.h2d_streams = [torch.cuda.Stream(dev) for _ in range(max(1, int(copy_streams)))]
        self.h2d = self.h2d_streams[0]
        self.d2h = torch.cuda.Stream(dev)
        self.shape = (B, H, Lq, Lk, D)
        self.block_size = block_size
        self.device = dev
        self.v_selected = bool(v_selected)
        self.value_gap = max(0, int(value_gap))
        # each group's selection, read back into pinned memory
        self._sel_host = [(torch.empty(p.indices.shape, dtype=torch.int32).pin_memory(),
                           torch.empty(p.counts.shape, dtype=torch.int32).pin_memory())
                          for p in self.plans]
        self.last_h2d_bytes = self.last_d2h_bytes = 0

    def _value_runs(self, g: int):
        """Runs ``(head, first key row, last key row + 1)`` of the value blocks
        group g's selection reads, consecutive blocks merged, and so are runs
        at most ``value_gap`` unselected blocks apart (one larger copy costs
        less than two small ones across a short gap)."""
        idx, cnt = (t.numpy() for t in self._sel_host[g])
        h0 = self.heads[g][0]
        Lk, bs = self.shape[3], self.block_size
        nkb = -(-Lk // bs)
        runs = []
        for h in range(idx.shape[1]):
            # the attention skips entries outside [0, nkb) the same way
            blocks = sorted({int(b) for qb in range(idx.shape[2])
                             for b in idx[0, h, qb, :max(0, int(cnt[0, h, qb]))] if 0 <= b < nkb})
            start = prev = None
            for b in blocks + [None]:
                if b is not None and prev is not None and b <= prev + 1 + self.value_gap:
                    prev = b
                    continue
                if start is not None:
                    runs.append((h0 + h, start * bs, min(Lk, (prev + 1) * bs)))
                start = prev = b
        return runs

    def __call__(self, hq: torch.Tensor, hk: torch.Tensor, hv: torch.Tensor,
                 hout: torch.Tensor, check: bool = True) -> torch.Tensor:
        """``hq``/``hk``/``hv``/``hout``: pinned host bf16 tensors of the plan's
        shapes; the attention output lands in ``hout``.  With ``check`` (the
        default) the call waits for the output copy, so ``hout`` is ready on
        return, and raises :class:`cast_b200._lib.CastError` if a kernel
        reported a device-side error; without it the call only enqueues, and
        the output copy is ordered before anything the caller enqueues next on
        its stream."""
        B, H, Lq, Lk, D = self.shape
        for name, t, L in (("q", hq, Lq), ("k", hk, Lk), ("v", hv, Lk), ("out", hout, Lq)):
            if t.is_cuda or t.dtype != torch.bfloat16 or tuple(t.shape) != (B, H, L, D):
                raise ValueError(f"{name} must be a host bf16 tensor of shape {(B, H, L, D)}")
            if not t.is_pinned():
                raise ValueError(f"{name} must be in pinned host memory")
        cur = torch.cuda.current_stream(self.device)
        # the previous call's compute and copies are done with the buffers
        for st in self.h2d_streams:
            st.wait_stream(cur)
        self.d2h.wait_stream(cur)
        row_bytes = D * 2
        h2d = 0
        n_cs = len(self.h2d_streams)
        ready = []
        for g, (h0, h1) in enumerate(self.heads):
            pairs = ((self.q, hq), (self.k, hk)) + (() if self.v_selected else ((self.v, hv),))
            evs = []
            for i, (dst, src) in enumerate(pairs):
                st = self.h2d_streams[(g + i) % n_cs]
                with torch.cuda.stream(st):
                    dst[:, h0:h1].copy_(src[:, h0:h1], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(st)
                evs.append(ev)
                h2d += dst[:, h0:h1].numel() * 2
            ready.append(evs)
        picked = []
        for g, (plan, evs) in enumerate(zip(self.plans, ready)):
            h0, h1 = self.heads[g]
            for ev in evs:
                cur.wait_event(ev)
            plan.select(self.q[:, h0:h1], self.k[:, h0:h1])
            if self.v_selected:
                idx, cnt = self._sel_host[g]
                idx.copy_(plan.indices, non_blocking=True)
                cnt.copy_(plan.counts, non_blocking=True)
                sel = torch.cuda.Event()
                sel.record(cur)
                picked.append(sel)
        for g, plan in enumerate(self.plans):
            h0, h1 = self.heads[g]
            if self.v_selected:
                picked[g].synchronize()
                for i, (h, r0, r1) in enumerate(self._value_runs(g)):
                    with torch.cuda.stream(self.h2d_streams[i % n_cs]):
                        self.v[0, h, r0:r1].copy_(hv[0, h, r0:r1], non_blocking=True)
                    h2d += (r1 - r0) * row_bytes
                for st in self.h2d_streams:
                    vin = torch.cuda.Event()
                    vin.record(st)
                    cur.wait_event(vin)
            plan.attend(self.q[:, h0:h1], self.k[:, h0:h1], self.v[:, h0:h1], out=self.out[:, h0:h1])
            done = torch.cuda.Event()
            done.record(cur)
            self.d2h.wait_event(done)
            with torch.cuda.stream(self.d2h):
                hout[:, h0:h1].copy_(self.out[:, h0:h1], non_blocking=True)
        self.last_h2d_bytes = h2d
        self.last_d2h_bytes = hout.numel() * 2
        cur.wait_stream(self.d2h)
        if check:
            _lib.check_device(cur.cuda_stream, "RCSAHostPlan")
        return hout
