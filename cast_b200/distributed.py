"""Multi-GPU partitioning of the RCSA layer: one process per GPU.

Selection, quantisation and attention are independent per (batch, head)
(selected blocks ``[B,H,...]``, per-(head, block) scales, per-head softmax),
so the layer splits without any exchange on its data path:

* rollout sharding: independent rollouts (BASELINE config 5 runs 8) go one
  per GPU; no collective at all (weak scaling);
* head sharding: the H heads of one layer call are split into contiguous
  ranges, one per GPU, and the bf16 head outputs are all-gathered (the only
  exchange a layer needs, 2.7 MB per GPU for config 2 at 8 GPUs).

The reference runs on one device and has no collective; this module is the
B200 partitioning around its per-head arithmetic.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

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


class HeadShardedRCSA:
    """One RCSA layer call split by heads over the ranks of a process group.

    Each rank holds a preallocated :class:`RCSAPlan` for its head range and a
    gather buffer, so a call allocates nothing on the device.
    """

    def __init__(self, B: int, H: int, Lq: int, Lk: int, D: int, *, block_size: int, budget: int,
                 policy: str = "auto", device: torch.device, group=None):
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.group = group
        self.lo, self.hi = head_range(H, self.world, self.rank)
        self.plan = RCSAPlan(B, self.hi - self.lo, Lq, Lk, D, block_size=block_size,
                             budget=budget, policy=policy, device=device)
        self.gathered = torch.empty((self.world * B, self.hi - self.lo, Lq, D),
                                    dtype=torch.bfloat16, device=device)

    def local_heads(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's head slice of a full ``[B, H, L, D]`` tensor."""
        return x[:, self.lo:self.hi].contiguous()

    def __call__(self, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor):
        """``q/k/v_local``: this rank's heads; returns all heads' outputs."""
        out = self.plan(q_local, k_local, v_local)
        return gather_heads(out, self.world, self.group, self.gathered)
