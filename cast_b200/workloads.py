"""Seeded synthetic inputs for the five RCSA/PAR workloads.

There is no public dataset on this path; every input is drawn from a CPU
``torch.Generator`` so the same tensors are produced on any host, then moved
to the requested device.  Shapes and distributions follow the benchmark
configurations of the hot path:

* ``config1`` -- CPU plumbing: B=1, H=4, D=64, 64-token frames (8x8 grid),
  8 history + 2 current frames, budget 4, fp32 N(0,1), seed 0 (Q, K, V drawn
  in that order over all 10 frames).
* ``config2`` -- one Matrix-shaped DiT layer: H=24, D=128, 880-token frames
  (22x40), 32 history + 4 current frames, budget 8, bf16 N(0,1)*s_h with
  s_h ~ U(0.5, 2) per head, seed 1.
* ``config3`` -- long history: 128 history frames, budget 16, queries on
  anchor frames 0 and 3 only, historical K drift ``+0.1*f*u_h`` with a fixed
  unit vector ``u_h`` per head, seed 2.
* ``config4`` -- PAR: residual bf16 ``[1, 1+4, 880, 3072]`` ~ N(0, 0.02)
  (one memory frame then four current frames), anchors 0 and 3, seed 3.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class RCSAWorkload:
    name: str
    q: torch.Tensor  # [B,H,Lq,D] packed queries (current chunk)
    k: torch.Tensor  # [B,H,Lk,D] packed keys: history blocks then current blocks
    v: torch.Tensor  # [B,H,Lk,D]
    block_size: int
    budget: int
    latent_hw: tuple[int, int]
    head_scale: torch.Tensor | None = None
    meta: dict = field(default_factory=dict)

    @property
    def n_query_blocks(self) -> int:
        return self.q.shape[2] // self.block_size

    @property
    def n_key_blocks(self) -> int:
        return self.k.shape[2] // self.block_size


def config1(device: str | torch.device = "cpu") -> RCSAWorkload:
    g = torch.Generator().manual_seed(0)
    b, h, d, f, hist, cur = 1, 4, 64, 64, 8, 2
    total = (hist + cur) * f
    q_all = torch.randn(b, h, total, d, generator=g)
    k = torch.randn(b, h, total, d, generator=g)
    v = torch.randn(b, h, total, d, generator=g)
    q = q_all[:, :, hist * f:].contiguous()
    return RCSAWorkload(
        "config1", q.to(device), k.to(device), v.to(device), f, 4, (8, 8),
        meta={"q_full": q_all.to(device), "history_frames": hist, "current_frames": cur},
    )


def _scaled(shape, scale, g, dtype):
    x = torch.randn(*shape, generator=g)
    return (x * scale.view(1, -1, 1, 1)).to(dtype)


def config2(device: str | torch.device = "cpu", heads: int = 24,
            history: int = 32, current: int = 4, seed: int = 1) -> RCSAWorkload:
    g = torch.Generator().manual_seed(seed)
    b, d, f = 1, 128, 880
    s = 0.5 + 1.5 * torch.rand(heads, generator=g)
    q = _scaled((b, heads, current * f, d), s, g, torch.bfloat16)
    k = _scaled((b, heads, (history + current) * f, d), s, g, torch.bfloat16)
    v = _scaled((b, heads, (history + current) * f, d), s, g, torch.bfloat16)
    return RCSAWorkload("config2", q.to(device), k.to(device), v.to(device), f, 8,
                        (22, 40), head_scale=s,
                        meta={"history_frames": history, "current_frames": current})


def config3(device: str | torch.device = "cpu", heads: int = 24,
            history: int = 128) -> RCSAWorkload:
    """Anchor-only queries (chunk frames 0 and 3) over a 128-frame history.

    Historical key frame ``f`` (0-based) is ``s_h*(N(0,1) + 0.1*f*u_h)``; only
    history drifts, the two anchor (current) key frames are ``s_h*N(0,1)``.
    """
    g = torch.Generator().manual_seed(2)
    b, d, f = 1, 128, 880
    anchors = (0, 3)
    s = 0.5 + 1.5 * torch.rand(heads, generator=g)
    u = torch.randn(heads, d, generator=g)
    u = u / u.norm(dim=1, keepdim=True)
    q = _scaled((b, heads, len(anchors) * f, d), s, g, torch.bfloat16)
    frames = list(range(history)) + [history + a for a in anchors]
    k = torch.randn(b, heads, len(frames) * f, d, generator=g)
    drift = torch.tensor(frames, dtype=torch.float32).repeat_interleave(f)
    drift[history * f:] = 0.0  # anchors: no drift term beyond noise
    k = k + 0.1 * drift.view(1, 1, -1, 1) * u.view(1, heads, 1, d)
    k = (k * s.view(1, -1, 1, 1)).to(torch.bfloat16)
    v = _scaled((b, heads, len(frames) * f, d), s, g, torch.bfloat16)
    return RCSAWorkload("config3", q.to(device), k.to(device), v.to(device), f, 16,
                        (22, 40), head_scale=s,
                        meta={"history_frames": history, "anchors": anchors})


@dataclass
class PARWorkload:
    name: str
    full_residual: torch.Tensor  # [1, M+T, HW, C]
    active_frames: list[int]     # global frame ids (memory frames first)
    memory_length: int
    height: int
    width: int

    @property
    def active_residual(self) -> torch.Tensor:
        return self.full_residual[:, self.active_frames].contiguous()


def config4(device: str | torch.device = "cpu", channels: int = 3072,
            seed: int = 3) -> PARWorkload:
    g = torch.Generator().manual_seed(seed)
    m, t, hw = 1, 4, 880
    full = (torch.randn(1, m + t, hw, channels, generator=g) * 0.02).to(torch.bfloat16)
    return PARWorkload("config4", full.to(device), [0, m + 0, m + 3], m, 22, 40)


def par_motion(device: str | torch.device = "cpu", channels: int = 64,
               seed: int = 7) -> PARWorkload:
    """Frames that are shifted crops of one pattern (exercises the phase path)."""
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(1, channels, 22 + 16, 40 + 16, generator=g) * 0.02
    frames = []
    for t in range(5):
        crop = base[:, :, 8 + t // 2:8 + t // 2 + 22, 8 + t:8 + t + 40]
        frames.append(crop.permute(0, 2, 3, 1).reshape(1, 880, channels))
    full = torch.stack(frames, 1).to(torch.bfloat16)
    return PARWorkload("par_motion", full.to(device), [0, 1, 4], 1, 22, 40)


@dataclass
class CompactCase:
    q: torch.Tensor            # bf16 [1, L, H, 128], token order
    k: torch.Tensor
    v: torch.Tensor
    coords: torch.Tensor       # long [L, 3]: compact frame, row, column
    freqs: torch.Tensor        # complex64 [positions, 64] or [H, positions, 64]
    memory_length: int
    memory_latent_idx: list[int]
    predict_latent_idx: tuple[int, int]
    block_id: torch.Tensor     # long [L]: compact block of each token
    n_blocks: int
    block_size: int


def compact_case(per_head_phase: bool = False, heads: int = 2, frames: int = 3,
                 hw: tuple[int, int] = (4, 8), cell: tuple[int, int, int] = (1, 3, 8),
                 memory_frames: int = 1, seed: int = 5) -> CompactCase:
    """A small compact layout in the frame weave's conventions (memory frames
    first, block cells of (tt, th, tw) that may be ragged, so some packed
    slots are padding), with seeded q/k/v and a seeded unit-modulus RoPE
    frequency table."""
    g = torch.Generator().manual_seed(seed)
    h0, w0 = hw
    n = frames * h0 * w0
    q, k, v = (torch.randn(1, n, heads, 128, generator=g).bfloat16() for _ in range(3))
    tok = torch.arange(n)
    t, sp = tok // (h0 * w0), tok % (h0 * w0)
    hh, ww = sp // w0, sp % w0
    coords = torch.stack([t, hh, ww], dim=1)
    shape = (heads, 1024, 64) if per_head_phase else (1024, 64)
    angles = torch.rand(shape, generator=g) * (2 * math.pi)
    freqs = torch.polar(torch.ones(shape), angles)
    tt, th, tw = cell
    nh, nw = -(-h0 // th), -(-w0 // tw)
    mem_cells = -(-memory_frames // tt)
    tcell = torch.where(t < memory_frames, t // tt, mem_cells + (t - memory_frames) // tt)
    block_id = tcell * nh * nw + (hh // th) * nw + ww // tw
    n_blocks = (mem_cells + -(-(frames - memory_frames) // tt)) * nh * nw
    return CompactCase(q, k, v, coords, freqs, memory_frames, [5 + i for i in range(memory_frames)],
                       (7, 7 + frames - memory_frames), block_id, n_blocks, tt * th * tw)


@dataclass
class SwapCase:
    score: torch.Tensor          # float32 [B, H, Q, K], local entries lowered by 1e6
    pooled_value: torch.Tensor   # float32 [B, H, K, D]
    selected: torch.Tensor       # long [B, H, Q, S]: local keys, then the best others
    counts: torch.Tensor         # long [B, H, Q]
    local: torch.Tensor          # bool [Q, K]
    memory_blocks: int
    spatial_shape: tuple[int, int]
    exact_frames: tuple[int, ...]
    temporal_group_size: int
    current_boundary: int
    transport: dict | None


def swap_case(*, heads: int = 3, memory_blocks: int = 6, cells: int = 4,
              spatial_shape: tuple[int, int] = (2, 4), dim: int = 64, width: int = 10,
              exact_frames: tuple[int, ...] = (0, 3), transport: bool = False,
              ragged: bool = True, temporal_group_size: int = 1, seed: int = 11) -> SwapCase:
    """Pooled block scores and values in the layout the swap router reads at
    its call site: memory blocks first, then ``cells`` temporal cells of
    ``nh x nw`` current blocks; each current row's local stencil is the
    current blocks of its own cell, each memory row's its own block.  The
    selection holds every local key then the best-scoring others (ragged
    counts when ``ragged``).  With ``transport`` a seeded FC-PASM endpoint
    sketch (22x40 latent, 11x10 windows, stride 8, padding (4, 5), 2x2
    transport pooling) is attached for every skipped anchor pair."""
    g = torch.Generator().manual_seed(seed)
    nh, nw = spatial_shape
    sp = nh * nw
    Q = K = memory_blocks + cells * sp
    raw = torch.randn(1, heads, Q, K, generator=g) * 2.0
    local = torch.zeros(Q, K, dtype=torch.bool)
    for m in range(memory_blocks):
        local[m, m] = True
    for c in range(cells):
        rows = slice(memory_blocks + c * sp, memory_blocks + (c + 1) * sp)
        local[rows, rows] = True
    forced = raw + local[None, None].float() * 1e6
    order = torch.argsort(forced, dim=-1, descending=True, stable=True)
    selected = order[..., :width].clone()
    n_local = local.sum(-1)
    if ragged:
        extra = torch.randint(0, 3, (1, heads, Q), generator=g)
        counts = torch.clamp(torch.full((1, heads, Q), width) - extra, min=0)
        counts = torch.maximum(counts, n_local[None, None] + 1)
    else:
        counts = torch.full((1, heads, Q), width)
    pad = torch.gather(selected, -1, (counts - 1)[..., None])
    slot = torch.arange(width)[None, None, None]
    selected = torch.where(slot < counts[..., None], selected, pad)
    value = torch.randn(1, heads, K, dim, generator=g)
    tr = None
    if transport:
        patches, fh, fw = 18, 6, 3
        pairs = {}
        for left, right in zip(exact_frames, exact_frames[1:]):
            if right - left > 1:
                theta = (torch.rand(patches, fh, fw, generator=g) * 2 - 1) * math.pi
                aff = torch.sigmoid(torch.randn(patches, fh, fw, generator=g) + 1.0)
                pairs[(int(left), int(right))] = {"theta": theta, "affinity": aff,
                                                  "mean_affinity": aff.mean()}
        tr = {"tile_grid": (3, 6), "output_shape": (22, 40), "transport_shape": (6, 5),
              "window_shape": (11, 10), "stride": (8, 8), "padding": (4, 5), "pairs": pairs,
              "attention_spatial_h": nh, "attention_spatial_w": nw}
    return SwapCase(raw - local[None, None].float() * 1e6, value, selected, counts, local,
                    memory_blocks, (nh, nw), tuple(exact_frames), temporal_group_size, 4, tr)
