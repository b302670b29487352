"""Multi-GPU partitioning of the RCSA layer: one process per GPU.

Selection, quantisation and attention are independent per (batch, head)
(selected blocks ``[B,H,...]``, per-(head, block) scales, per-head softmax),
so the layer splits without any exchange on its data path:

* rollout sharding: independent rollouts (BASELINE config 5 runs 8) go one
  per GPU; no collective at all (weak scaling);
* head sharding: the H heads of one layer call are split into contiguous
  ranges, one per GPU, and the bf16 head outputs are gathered on every GPU
  (the only exchange a layer needs, 2.7 MB per GPU for config 2 at 8 GPUs):
  by default with plain peer stores over NVLink into IPC-shared buffers
  (:class:`PeerGather`), else with NCCL's all-gather.

The reference runs on one device and has no collective; this module is the
B200 partitioning around its per-head arithmetic.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .rcsa import RCSAPlan


def head_range(heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous head range ``[lo, hi)`` of ``rank``; heads must divide evenly
    so every rank does the same work and the gathered layout is plain."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if heads % world:
        raise ValueError(f"{heads} heads do not split evenly over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


def gather_heads(out_local: torch.Tensor, world: int, group=None,
                 gathered: torch.Tensor | None = None) -> torch.Tensor:
    """All-gathers ``[B, H/world, L, D]`` head outputs into ``[B, H, L, D]``.

    Rank ``r``'s heads land at ``[r*H/world, (r+1)*H/world)``.  The gather
    buffer is ``[world*B, H/world, L, D]`` (rank-major, the concatenated form
    every backend accepts).  With ``B == 1`` it already has the memory layout
    of ``[1, H, L, D]`` and is returned as a view; otherwise one permute copy
    restores head order.  ``gathered`` may be passed preallocated.
    """
    if out_local.ndim != 4:
        raise ValueError("expected [B, H_local, L, D]")
    out_local = out_local.contiguous()
    b, hl, length, d = out_local.shape
    if gathered is None:
        gathered = torch.empty((world * b, hl, length, d), dtype=out_local.dtype,
                               device=out_local.device)
    if world == 1:
        gathered.copy_(out_local)
    else:
        dist.all_gather_into_tensor(gathered, out_local, group=group)
    if b == 1:
        return gathered.view(1, world * hl, length, d)
    return gathered.view(world, b, hl, length, d).permute(1, 0, 2, 3, 4).reshape(b, world * hl, length, d)


class _DeviceArray:
    """A borrowed device buffer seen by ``torch.as_tensor`` (no ownership)."""

    def __init__(self, address: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (address, False),
                                         "version": 3, "strides": None}


class PeerGather:
    """The gathered head buffers of a head-sharded layer, written directly by
    every rank's attention (``cast_rcsa_attention_peers``): each rank owns one
    device buffer, shared with the others through CUDA IPC (no multicast),
    holding two gathered outputs ``[2][world*B][H/world][Lq][D]`` bf16 (the
    calls alternate between them, so a peer never writes the output its
    owner may still be reading), then the flag word each peer raises when its
    rows have landed, the attention's CTA ticket and the call counter.

    Every rank must make the same number of calls; :meth:`close` (collective)
    releases the buffers before the process group goes away."""

    def __init__(self, B: int, heads_local: int, Lq: int, D: int, *, device: torch.device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError("the fused gather runs on 2 to 8 ranks")
        self.device = torch.device(device)
        self.shape = (B, heads_local, Lq, D)
        slot = B * heads_local * Lq * D * 2
        self.slot_bytes = slot
        buf = 2 * self.world * slot
        self.flag_off = (buf + 255) // 256 * 256
        total = self.flag_off + 256
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        with torch.cuda.device(self.device):
            _lib.call("cast_peer_alloc", total, ctypes.byref(own), ctypes.byref(handle))
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        bases = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                p = ctypes.c_void_p()
                _lib.call("cast_peer_open", ctypes.byref(hb), ctypes.byref(p))
                self._opened.append(p.value)
                bases.append(p.value)
        others = [r for r in range(self.world) if r != self.rank]
        self._peer_out = [(ctypes.c_void_p * len(others))(
            *[bases[r] + (par * self.world + self.rank) * slot for r in others]) for par in (0, 1)]
        self._peer_flag = (ctypes.c_void_p * len(others))(
            *[bases[r] + self.flag_off + 4 * self.rank for r in others])
        self.flags = self._own + self.flag_off  # uint32 [8]: the peers' call numbers
        self.ticket = self.flags + 32
        self.calls = self.flags + 36
        self.gathered = torch.as_tensor(
            _DeviceArray(self._own, (2, self.world * B, heads_local, Lq, D), "<i2"),
            device=self.device).view(torch.bfloat16)
        self.calls_made = 0
        # one copy stream per peer for send() (made here: never during a capture)
        self._send_streams = [torch.cuda.Stream(self.device) for _ in range(self.world - 1)]

    def slot(self, parity: int) -> torch.Tensor:
        """This rank's ``[B, H/world, Lq, D]`` slot of gathered buffer ``parity``."""
        B = self.shape[0]
        return self.gathered[parity, self.rank * B:(self.rank + 1) * B]

    def peers(self, parity: int):
        """``cast_rcsa_attention_peers``'s gather arguments for buffer ``parity``."""
        return (self.world - 1, ctypes.cast(self._peer_out[parity], ctypes.c_void_p),
                ctypes.cast(self._peer_flag, ctypes.c_void_p), self.ticket, self.calls)

    def push(self, parity: int) -> None:
        """This rank's slot of gathered buffer ``parity`` into every peer's
        buffer (``cast_peer_push``, a launch after the attention)."""
        n, out, flag, ticket, calls = self.peers(parity)
        _lib.call("cast_peer_push", self.slot(parity).data_ptr(), self.slot_bytes, n, out, flag, ticket,
                  calls, torch.cuda.current_stream(self.device).cuda_stream)

    def send(self, parity: int) -> None:
        """This rank's slot of gathered buffer ``parity`` into every peer's
        buffer on the copy engines (``cast_peer_send``: one copy and its flag
        per peer, each on its own stream forked from the caller's stream and
        joined back), leaving the SMs to the caller's kernels."""
        cur = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(cur)
        src = self.slot(parity).data_ptr()
        outs, flags = self._peer_out[parity], self._peer_flag
        for j, st in enumerate(self._send_streams):
            st.wait_event(start)
            _lib.call("cast_peer_send", outs[j], src, self.slot_bytes, flags[j], self.calls, st.cuda_stream)
            done = torch.cuda.Event()
            done.record(st)
            cur.wait_event(done)

    def wait(self) -> None:
        """Orders the stream after every peer's rows of this call."""
        _lib.call("cast_peer_wait", self.flags, self.world, self.rank, self.calls,
                  torch.cuda.current_stream(self.device).cuda_stream)

    def heads(self, parity: int) -> torch.Tensor:
        """Gathered buffer ``parity`` as ``[B, H, Lq, D]`` in head order."""
        B, hl, lq, d = self.shape
        g = self.gathered[parity]
        if B == 1:
            return g.view(1, self.world * hl, lq, d)
        return g.view(self.world, B, hl, lq, d).permute(1, 0, 2, 3, 4).reshape(B, self.world * hl, lq, d)

    def close(self) -> None:
        """Collective: every rank stops using the peers' buffers, then frees its own."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("cast_peer_close", ctypes.c_void_p(p))
        self._opened = []
        dist.barrier(group=self.group)
        self.gathered = None
        with torch.cuda.device(self.device):
            _lib.call("cast_peer_free", ctypes.c_void_p(self._own))
        self._own = None


class HeadShardedRCSA:
    """One RCSA layer call split by heads over the ranks of a process group.

    Each rank holds a preallocated :class:`RCSAPlan` for its head range and a
    gather buffer, so a call allocates nothing on the device.  ``gather``:
    ``"nccl"`` (NCCL's all-gather after the attention), ``"peer"`` (one
    streaming launch writes this rank's heads into every peer's buffer over
    NVLink, :meth:`PeerGather.push`) or ``"fused"`` (the attention's epilogue
    stores every row into the peers' buffers as it is produced) or ``"ce"``
    (the copy engines move this rank's heads into every peer after the
    attention, :meth:`PeerGather.send`).
    """

    def __init__(self, B: int, H: int, Lq: int, Lk: int, D: int, *, block_size: int, budget: int,
                 policy: str = "auto", device: torch.device, group=None, gather: str = "peer"):
        if gather not in ("nccl", "peer", "fused", "ce"):
            raise ValueError("gather must be 'nccl', 'peer', 'fused' or 'ce'")
        self.gather = gather
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.group = group
        self.lo, self.hi = head_range(H, self.world, self.rank)
        self.plan = RCSAPlan(B, self.hi - self.lo, Lq, Lk, D, block_size=block_size,
                             budget=budget, policy=policy, device=device)
        self.peer = (PeerGather(B, self.hi - self.lo, Lq, D, device=device, group=group)
                     if gather != "nccl" and self.world > 1 else None)
        self.gathered = None if self.peer else torch.empty(
            (self.world * B, self.hi - self.lo, Lq, D), dtype=torch.bfloat16, device=device)

    def local_heads(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's head slice of a full ``[B, H, L, D]`` tensor."""
        return x[:, self.lo:self.hi].contiguous()

    def __call__(self, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor):
        """``q/k/v_local``: this rank's heads; returns all heads' outputs.
        With the fused gather the result is a view of one of the two gathered
        buffers, valid until the call after next."""
        if self.peer is None:
            out = self.plan(q_local, k_local, v_local)
            return gather_heads(out, self.world, self.group, self.gathered)
        par = self.peer.calls_made & 1
        self.plan.select(q_local, k_local)
        if self.gather == "fused":  # the attention's epilogue stores into the peers too
            self.plan.attend(q_local, k_local, v_local, out=self.peer.slot(par), peers=self.peer.peers(par))
        else:  # the attention, then the copy into the peers (SMs or copy engines)
            self.plan.attend(q_local, k_local, v_local, out=self.peer.slot(par))
            if self.gather == "ce":
                self.peer.send(par)
            else:
                self.peer.push(par)
        self.peer.wait()
        self.peer.calls_made += 1
        return self.peer.heads(par)

    def close(self) -> None:
        """Collective with the fused gather: releases the peer buffers."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None
