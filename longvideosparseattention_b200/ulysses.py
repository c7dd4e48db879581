"""Ulysses context parallelism for the LVSA kernel (heads shard naturally).

Each rank holds a contiguous token shard [B, S_r, H, D] of q/k/v (shard sizes
may be uneven) and the full text K/V.  One all_to_all_single moves the packed
q/k/v from "my tokens, all heads" to "all tokens, my H/w heads"; every rank
then runs the world = 1 pattern on its heads; a second all_to_all_single
returns the output to the token-sharded layout.  Text query rows (dense) are
computed for the local heads and all-gathered.

Parity target: the world = 1 output of the reference (identical mask on every
rank).  The reference's own multi-GPU mode -- sequence shards plus a SUM
all_reduce of the anchor K/V (lvsa/lvsa_processor.py:643-706) with boundary
guard frames (lvsa/sparse_attention.py:107-129) -- has a different pattern
and is not what this path reproduces.

Layout choice: the packed send buffer is [w][B, S_r, 3, H/w, D], so what a
rank receives is [B, S, 3, H/w, D] (B = 1: one contiguous block) and q, k, v
are strided views handed to the kernel without another copy.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def shard_sizes(total: int, world: int) -> List[int]:
    """Contiguous token shards, the first ``total % world`` one token longer."""
    base, rem = divmod(total, world)
    return [base + (1 if r < rem else 0) for r in range(world)]


def _heads(H: int, world: int) -> int:
    if H % world:
        raise ValueError(f"Ulysses needs heads ({H}) divisible by world ({world})")
    return H // world


def pack_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, world: int) -> torch.Tensor:
    """[B, S_r, H, D] x3 -> contiguous [w, B, S_r, 3, H/w, D]."""
    B, S, H, D = q.shape
    Hl = _heads(H, world)
    x = torch.stack([q, k, v], dim=2)                      # [B, S_r, 3, H, D]
    x = x.view(B, S, 3, world, Hl, D).permute(3, 0, 1, 2, 4, 5)
    return x.contiguous()


def unpack_received(recv: torch.Tensor, sizes: Sequence[int], B: int, Hl: int, D: int):
    """Received flat buffer -> q, k, v [B, S, Hl, D] (views when B == 1)."""
    S = sum(sizes)
    if B == 1:
        x = recv.view(1, S, 3, Hl, D)
    else:
        parts, off = [], 0
        for s in sizes:
            n = B * s * 3 * Hl * D
            parts.append(recv[off:off + n].view(B, s, 3, Hl, D))
            off += n
        x = torch.cat(parts, dim=1)
    return x[:, :, 0], x[:, :, 1], x[:, :, 2]


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sizes: Sequence[int],
                      local_attention: Callable, text_q: Optional[torch.Tensor] = None,
                      text_k: Optional[torch.Tensor] = None, text_v: Optional[torch.Tensor] = None,
                      group=None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Head-parallel LVSA over ``group``.

    q/k/v: this rank's token shard [B, sizes[rank], H, D] (GQA: the kv heads
    must also divide by world).  ``local_attention(q, k, v, tq, tk, tv)`` runs
    the world = 1 pattern on full-sequence, local-head tensors and returns
    (out, text_out).  Returns (out shard [B, S_r, H, D], text_out [B, Nt, H, D]).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, S_r, H, D = q.shape
    if S_r != sizes[rank]:
        raise AssertionError(f"rank {rank} holds {S_r} tokens, expected {sizes[rank]}")
    if k.shape[2] != H:
        raise NotImplementedError("Ulysses path expects kv_heads == heads")
    Hl = _heads(H, world)
    send = pack_qkv(q, k, v, world).view(-1)
    unit = B * 3 * Hl * D
    in_splits = [S_r * unit] * world
    out_splits = [s * unit for s in sizes]
    recv = torch.empty(sum(out_splits), dtype=q.dtype, device=q.device)
    dist.all_to_all_single(recv, send, out_splits, in_splits, group=group)
    qf, kf, vf = unpack_received(recv, sizes, B, Hl, D)

    hs = slice(rank * Hl, (rank + 1) * Hl)
    tq = text_q[:, :, hs] if text_q is not None else None
    tk = text_k[:, :, hs] if text_k is not None else None
    tv = text_v[:, :, hs] if text_v is not None else None
    out_full, tout = local_attention(qf, kf, vf, tq, tk, tv)   # [B, S, Hl, D]

    # return path: chunk i = my heads for rank i's tokens
    if B == 1:
        send_o = out_full.contiguous().view(-1)
    else:
        send_o = torch.cat([c.contiguous().view(-1) for c in torch.split(out_full, list(sizes), dim=1)])
    o_unit = B * Hl * D
    recv_o = torch.empty(world * S_r * o_unit, dtype=out_full.dtype, device=q.device)
    dist.all_to_all_single(recv_o, send_o, [S_r * o_unit] * world, [s * o_unit for s in sizes],
                           group=group)
    out = recv_o.view(world, B, S_r, Hl, D).permute(1, 2, 0, 3, 4).reshape(B, S_r, H, D)

    text_out = None
    if tout is not None:
        gathered = [torch.empty_like(tout) for _ in range(world)]
        dist.all_gather(gathered, tout.contiguous(), group=group)
        text_out = torch.cat(gathered, dim=2)
    return out, text_out


def kernel_local_attention(metadata, scale: Optional[float] = None) -> Callable:
    """The default local step: the sm_100a kernel with the world = 1 mask."""
    from .block_sparse import block_sparse_attention

    def run(q, k, v, tq, tk, tv):
        nt = 0 if tk is None else int(tk.shape[1])
        mask = metadata.block_mask(q.device, nt)
        return block_sparse_attention(q, k, v, mask, tq, tk, tv, scale=scale)
    return run
