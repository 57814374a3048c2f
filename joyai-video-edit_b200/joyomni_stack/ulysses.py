"""Ulysses sequence parallelism for the MMDiT block stack.

The reference runs the whole denoiser on one GPU and has no sequence
parallelism (nothing in deploy/ calls torch.distributed); this module is the
new multi-GPU layer for BASELINE config 5.  Each of the P ranks owns a
contiguous shard of the chunk's image tokens and of its text tokens and runs
every per-token operator (norm, modulation, FP8 GEMMs, QK-norm + RoPE) on its
shard with no communication.  Attention needs every token for a head, so
q/k/v are exchanged sequence-sharded -> head-sharded with one all-to-all
before attention, and the attention output is exchanged back after it
(NCCL over NVLink on the GPU box; gloo works for the CPU tests).

Token order after the exchange is [img_0, txt_0, img_1, txt_1, ...] (rank
order).  Non-causal attention without masks is invariant to the order of its
keys, and each rank gets its own queries back in its own order, so the order
never has to be undone.  Shards may differ in size by one token (uneven split
sizes), so no padding or masking is needed.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch


def split_sizes(n: int, parts: int) -> List[int]:
    """Contiguous split of n items into `parts` shards differing by at most one."""
    base, rem = divmod(n, parts)
    return [base + (1 if r < rem else 0) for r in range(parts)]


def shard_range(n: int, parts: int, rank: int):
    sizes = split_sizes(n, parts)
    start = sum(sizes[:rank])
    return start, start + sizes[rank]


@dataclass
class SeqParallel:
    """Process-group view of one Ulysses group (P ranks, heads % P == 0)."""

    group: Optional[object]
    world: int
    rank: int
    img_tokens: int
    txt_tokens: int
    heads: int

    @classmethod
    def create(cls, img_tokens: int, txt_tokens: int, heads: int, group=None) -> "SeqParallel":
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            world, rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            world, rank = 1, 0
        if heads % world:
            raise ValueError(f"heads ({heads}) must be divisible by the Ulysses degree ({world})")
        if img_tokens < world:
            raise ValueError(f"every rank needs at least one image token ({img_tokens} < {world})")
        return cls(group, world, rank, img_tokens, txt_tokens, heads)

    # -- shard bookkeeping ---------------------------------------------------
    @property
    def img_range(self):
        return shard_range(self.img_tokens, self.world, self.rank)

    @property
    def txt_range(self):
        return shard_range(self.txt_tokens, self.world, self.rank)

    def shard_len(self, r: int) -> int:
        return split_sizes(self.img_tokens, self.world)[r] + split_sizes(self.txt_tokens, self.world)[r]

    @property
    def local_len(self) -> int:
        return self.shard_len(self.rank)

    @property
    def total_len(self) -> int:
        return self.img_tokens + self.txt_tokens

    @property
    def local_heads(self) -> int:
        return self.heads // self.world

    def gathered_img_segments(self):
        """(start, length) of every rank's image tokens in the gathered order."""
        segs, off = [], 0
        isz = split_sizes(self.img_tokens, self.world)
        for r in range(self.world):
            segs.append((off, isz[r]))
            off += self.shard_len(r)
        return segs

    def gathered_segment_starts(self):
        """First row of every rank's tokens in the gathered order, then the
        total: rank k owns rows starts[k] .. starts[k + 1] (the segment table of
        the attention epilogue that stores each output row on its owner)."""
        starts, off = [], 0
        for r in range(self.world):
            starts.append(off)
            off += self.shard_len(r)
        return starts + [off]

    # -- exchanges -------------------------------------------------------------
    def seq_to_heads(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[L_local, H, Dh] (this rank's tokens, all heads) -> [L_total, H/P, Dh]
        (all tokens, this rank's heads), written into `out` when given (it must be
        contiguous; e.g. the tail of a preallocated [cache | current] KV buffer)."""
        L, H, Dh = x.shape
        P = self.world
        if out is None:
            out = torch.empty((self.total_len, H // P, Dh), dtype=x.dtype, device=x.device)
        if P == 1:
            out.copy_(x)
            return out
        send = x.view(L, P, H // P, Dh).transpose(0, 1).contiguous()          # [P, L, H/P, Dh]
        import torch.distributed as dist
        dist.all_to_all_single(out.view(self.total_len, -1), send.view(P * L, -1),
                               output_split_sizes=[self.shard_len(r) for r in range(P)],
                               input_split_sizes=[L] * P, group=self.group)
        return out

    def heads_to_seq(self, y: torch.Tensor) -> torch.Tensor:
        """[L_total, H/P, Dh] -> [L_local, H, Dh] (inverse of seq_to_heads)."""
        Lt, Hp, Dh = y.shape
        P = self.world
        if P == 1:
            return y
        L = self.local_len
        recv = torch.empty((P, L, Hp, Dh), dtype=y.dtype, device=y.device)
        import torch.distributed as dist
        dist.all_to_all_single(recv.view(P * L, -1), y.contiguous().view(Lt, -1),
                               output_split_sizes=[L] * P,
                               input_split_sizes=[self.shard_len(r) for r in range(P)], group=self.group)
        return recv.transpose(0, 1).reshape(L, P * Hp, Dh)
