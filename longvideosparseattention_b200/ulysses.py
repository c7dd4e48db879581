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


def _default_chunks(Hl: int, world: int) -> int:
    # Measured on 2 B200s (cfg2): 1 group 18.6 ms/layer, 2 groups 19.6, 3 groups
    # 19.3 -- the NCCL kernels of the overlapped exchange take SMs from the
    # attention kernel and the head gathers add copies, so one exchange wins.
    return 1


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sizes: Sequence[int],
                      local_attention: Callable, text_q: Optional[torch.Tensor] = None,
                      text_k: Optional[torch.Tensor] = None, text_v: Optional[torch.Tensor] = None,
                      group=None, chunks: Optional[int] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Head-parallel LVSA over ``group``.

    q/k/v: this rank's token shard [B, sizes[rank], H, D] (GQA: the kv heads
    must also divide by world).  ``local_attention(q, k, v, tq, tk, tv)`` runs
    the world = 1 pattern on full-sequence, local-head tensors and returns
    (out, text_out).  Returns (out shard [B, S_r, H, D], text_out [B, Nt, H, D]).

    ``chunks`` splits this rank's heads into groups that are exchanged and
    computed one after another: the all-to-all of group c+1 and the return of
    group c-1 run on NCCL's stream while the kernel computes group c (default:
    one group, see ``_default_chunks``).  Results do not depend on it.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, S_r, H, D = q.shape
    if S_r != sizes[rank]:
        raise AssertionError(f"rank {rank} holds {S_r} tokens, expected {sizes[rank]}")
    if k.shape[2] != H:
        raise NotImplementedError("Ulysses path expects kv_heads == heads")
    Hl = _heads(H, world)
    n_chunks = chunks or _default_chunks(Hl, world)
    if Hl % n_chunks:
        raise ValueError(f"chunks ({n_chunks}) must divide the local head count ({Hl})")
    Hc = Hl // n_chunks

    def heads_of(c: int) -> torch.Tensor:
        # global head indices of group c on every rank: rank j's heads j*Hl + c*Hc ...
        idx = [j * Hl + c * Hc + i for j in range(world) for i in range(Hc)]
        return torch.tensor(idx, device=q.device)

    unit = B * 3 * Hc * D
    in_splits = [S_r * unit] * world
    out_splits = [s * unit for s in sizes]
    o_unit = B * Hc * D

    # Issue every forward exchange up front; NCCL runs them in order on its stream.
    fwd = []
    for c in range(n_chunks):
        hsel = heads_of(c) if n_chunks > 1 else None
        qc, kc, vc = ((x if hsel is None else x.index_select(2, hsel)) for x in (q, k, v))
        send = pack_qkv(qc, kc, vc, world).view(-1)
        recv = torch.empty(sum(out_splits), dtype=q.dtype, device=q.device)
        work = dist.all_to_all_single(recv, send, out_splits, in_splits, group=group, async_op=True)
        fwd.append((recv, send, work))

    back, touts = [], []
    for c in range(n_chunks):
        recv, _send, work = fwd[c]
        work.wait()
        qf, kf, vf = unpack_received(recv, sizes, B, Hc, D)
        hs = slice(rank * Hl + c * Hc, rank * Hl + (c + 1) * Hc)
        tq = text_q[:, :, hs] if text_q is not None else None
        tk = text_k[:, :, hs] if text_k is not None else None
        tv = text_v[:, :, hs] if text_v is not None else None
        out_full, tout = local_attention(qf, kf, vf, tq, tk, tv)   # [B, S, Hc, D]
        touts.append(tout)
        # return path: part j = these heads for rank j's tokens
        if B == 1:
            send_o = out_full.contiguous().view(-1)
        else:
            send_o = torch.cat([p.contiguous().view(-1) for p in torch.split(out_full, list(sizes), dim=1)])
        recv_o = torch.empty(world * S_r * o_unit, dtype=out_full.dtype, device=q.device)
        work_o = dist.all_to_all_single(recv_o, send_o, [S_r * o_unit] * world, [s * o_unit for s in sizes],
                                        group=group, async_op=True)
        back.append((recv_o, send_o, work_o))

    out = torch.empty(B, S_r, H, D, dtype=q.dtype, device=q.device)
    ov = out.view(B, S_r, world, n_chunks, Hc, D)
    for c, (recv_o, _send_o, work_o) in enumerate(back):
        work_o.wait()
        ov[:, :, :, c] = recv_o.view(world, B, S_r, Hc, D).permute(1, 2, 0, 3, 4)

    text_out = None
    if touts and touts[0] is not None:
        tloc = torch.cat(touts, dim=2).contiguous()              # [B, Nt, Hl, D], my heads
        gathered = [torch.empty_like(tloc) for _ in range(world)]
        dist.all_gather(gathered, tloc, group=group)
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
