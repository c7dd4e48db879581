"""Ulysses context parallelism for the LVSA kernel (heads shard naturally).

Each rank holds a contiguous token shard [B, S_r, H, D] of q/k/v (shard sizes
may be uneven) and the full text K/V.  One all_to_all_single moves the packed
q/k/v from "my tokens, all heads" to "all tokens, my heads"; every rank runs
the world = 1 pattern on its share; a second all_to_all_single returns the
output to the token-sharded layout.

Work partition (``make_schedule``).  When the GPU count divides the head
count, rank r owns heads [r H/w, (r+1) H/w), every tile row: the classic
Ulysses split.  Otherwise (12 heads on 8 GPUs) the work is the sequence of
(head, query-tile row) units in head-major order, each weighted by the number
of key tiles of its row (the kernel's cost), cut into w contiguous pieces of
equal weight at tile-row boundaries.  A rank then owns a run of whole heads
plus at most a partial head on either side; it receives q/k/v for the heads
it touches (a head shared by two ranks is sent to both) and launches the
kernel once per piece with the row range ``q_tiles=(t0, t1)``.  Grouped K/V
heads (Hkv < H) are supported: a rank receives the K/V heads of its query
heads, and pieces are split at K/V group boundaries so every launch maps its
query heads onto its K/V heads as SDPA's enable_gqa does.

Packing.  The send buffer for destination d is [B, S_r, nq_d + 2 nk_d, D]
(d's query heads, then its K heads, then its V heads); what a rank receives,
concatenated over sources, is [B, S, nq + 2 nk, D] (one contiguous block when
B = 1), and q, k, v are strided views of it handed to the kernel with no
unpack copy.  Both the pack and the return-path scatter are single launches
of the batched strided copy kernel (``lvsa_copy_segments``).  Text query rows
(dense) are computed by the rank whose piece holds them, written into a
zeroed [B, Nt, H, D] buffer and summed over ranks (each row has exactly one
writer, so the sum is exact).

Parity target: the world = 1 output of the reference (identical mask on every
rank).  The reference's own multi-GPU mode -- sequence shards plus a SUM
all_reduce of the anchor K/V (lvsa/lvsa_processor.py:643-706) with boundary
guard frames (lvsa/sparse_attention.py:107-129) -- has a different pattern;
``cp_mode.py`` reproduces that one.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .block_sparse import ATTN_BLOCK_Q, copy_segments


def shard_sizes(total: int, world: int) -> List[int]:
    """Contiguous token shards, the first ``total % world`` one token longer."""
    base, rem = divmod(total, world)
    return [base + (1 if r < rem else 0) for r in range(world)]


@dataclass(frozen=True)
class Piece:
    """Query heads [h0, h1) over tile-CSR rows [t0, t1)."""
    h0: int
    h1: int
    t0: int
    t1: int


@dataclass
class UlyssesSchedule:
    world: int
    heads: int
    kv_heads: int
    n_q_tiles: int
    pieces: List[List[Piece]]          # per rank
    q_heads: List[Tuple[int, int]]     # per rank: query heads [a, b) it receives
    kv_range: List[Tuple[int, int]]    # per rank: K/V heads [a, b) it receives

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads

    def cost(self, rank: int, costs: Sequence[float]) -> float:
        return sum((p.h1 - p.h0) * sum(costs[p.t0:p.t1]) for p in self.pieces[rank])


def _split_gqa(p: Piece, g: int) -> List[Piece]:
    """Split a head run so each part is one partial K/V group or whole groups."""
    if g == 1 or p.h1 - p.h0 == 1:
        return [p]
    out, h = [], p.h0
    a = -(-p.h0 // g) * g                        # first group boundary at or after h0
    if a > h:
        out.append(Piece(h, min(a, p.h1), p.t0, p.t1))
        h = min(a, p.h1)
    b = (p.h1 // g) * g                          # last group boundary at or before h1
    if b > h:
        out.append(Piece(h, b, p.t0, p.t1))
        h = b
    if h < p.h1:
        out.append(Piece(h, p.h1, p.t0, p.t1))
    return out


def make_schedule(heads: int, kv_heads: int, world: int, n_q_tiles: int,
                  costs: Optional[Sequence[float]] = None) -> UlyssesSchedule:
    """Partition heads x tile rows over ``world`` ranks (see the module doc).

    ``costs``: per tile-row weight (the row's key-tile count); uniform when
    None.  Whole heads per rank when ``world`` divides ``heads``."""
    if heads % kv_heads:
        raise ValueError(f"heads ({heads}) must be a multiple of kv_heads ({kv_heads})")
    g = heads // kv_heads
    nq = int(n_q_tiles)
    pieces: List[List[Piece]] = []
    if heads % world == 0:
        hl = heads // world
        for r in range(world):
            pieces.append(_split_gqa(Piece(r * hl, (r + 1) * hl, 0, nq), g))
    else:
        w = [float(c) for c in costs] if costs is not None else [1.0] * nq
        if len(w) != nq:
            raise ValueError(f"costs has {len(w)} rows, expected {nq}")
        w = [max(c, 0.0) + 1e-9 for c in w]     # empty rows still cost a launch slot
        row_prefix = [0.0]
        for c in w:
            row_prefix.append(row_prefix[-1] + c)
        per_head = row_prefix[-1]
        total = per_head * heads

        def cut(target: float) -> int:
            """Flattened unit index (head * nq + row) closest to cumulative weight ``target``."""
            h = min(int(target // per_head), heads - 1)
            rem = target - h * per_head
            lo, hi = 0, nq                        # smallest t with row_prefix[t] >= rem
            while lo < hi:
                mid = (lo + hi) // 2
                if row_prefix[mid] < rem:
                    lo = mid + 1
                else:
                    hi = mid
            t = lo
            if t > 0 and rem - row_prefix[t - 1] < row_prefix[t] - rem:
                t -= 1
            return h * nq + t
        bounds = [0] + [cut(total * r / world) for r in range(1, world)] + [heads * nq]
        for r in range(world):
            a, b = bounds[r], max(bounds[r], bounds[r + 1])
            ps: List[Piece] = []
            u = a
            while u < b:
                h, t = divmod(u, nq)
                if t == 0 and b - u >= nq:        # whole heads
                    nh = (b - u) // nq
                    ps.append(Piece(h, h + nh, 0, nq))
                    u += nh * nq
                else:
                    e = min(b, (h + 1) * nq)
                    ps.append(Piece(h, h + 1, t, e - h * nq))
                    u = e
            pieces.append([x for p in ps for x in _split_gqa(p, g)])
    q_heads, kv_range = [], []
    for ps in pieces:
        if ps:
            a, b = min(p.h0 for p in ps), max(p.h1 for p in ps)
        else:
            a = b = 0
        q_heads.append((a, b))
        kv_range.append((a // g, -(-b // g)) if b > a else (0, 0))
    return UlyssesSchedule(world, heads, kv_heads, nq, pieces, q_heads, kv_range)


def tile_costs(mask) -> List[int]:
    """Per tile-row key-tile counts of a BlockMask (one synchronising read)."""
    ip = mask.tile_indptr[: mask.n_q_tiles + 1].cpu().tolist()
    return [ip[i + 1] - ip[i] for i in range(mask.n_q_tiles)]


def _video_rows(p: Piece, n_q_video_tiles: int, n_video: int) -> Tuple[int, int]:
    """Token rows [s, e) of the video segment a piece covers."""
    s = min(p.t0, n_q_video_tiles) * ATTN_BLOCK_Q
    e = min(min(p.t1, n_q_video_tiles) * ATTN_BLOCK_Q, n_video)
    return min(s, n_video), e


_SCHED_CACHE: Dict[tuple, UlyssesSchedule] = {}
_STREAMS: Dict[tuple, List[torch.cuda.Stream]] = {}


def _piece_streams(device: torch.device, n: int) -> List[torch.cuda.Stream]:
    key = (str(device), n)
    if key not in _STREAMS:
        _STREAMS[key] = [torch.cuda.Stream(device=device) for _ in range(n)]
    return _STREAMS[key]


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sizes: Sequence[int],
                      local_attention: Callable, text_q: Optional[torch.Tensor] = None,
                      text_k: Optional[torch.Tensor] = None, text_v: Optional[torch.Tensor] = None,
                      group=None, n_q_tiles: Optional[int] = None, costs: Optional[Sequence[float]] = None,
                      schedule: Optional[UlyssesSchedule] = None, timing: Optional[dict] = None
                      ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Head-parallel LVSA over ``group``.

    q [B, sizes[rank], H, D], k/v [B, sizes[rank], Hkv, D]: this rank's
    token shard.  ``local_attention(q, k, v, tq, tk, tv, q_tiles, out,
    text_out)`` runs the world = 1 pattern on full-sequence tensors of some
    heads (k/v: their K/V heads) for tile rows ``q_tiles = (t0, t1)`` and
    writes rows of ``out`` [B, S, h, D] / ``text_out`` [B, Nt, h, D] in
    place.  ``n_q_tiles`` / ``costs``: the mask's tile-row count and per-row
    weights (needed only when the GPU count does not divide the head count;
    default: uniform weights over ceil(S/128) + ceil(Nt/128) rows); or pass
    a prebuilt ``schedule``.  ``timing``: a dict that receives CUDA events
    (pack, exchange, attention, return) for the caller to read.

    Returns (out shard [B, S_r, H, D], text_out [B, Nt, H, D] or None).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, S_r, H, D = q.shape
    Hkv = k.shape[2]
    if S_r != sizes[rank]:
        raise AssertionError(f"rank {rank} holds {S_r} tokens, expected {sizes[rank]}")
    S = int(sum(sizes))
    Nt = 0 if text_k is None else int(text_k.shape[1])
    text_rows = text_q is not None and Nt > 0
    nqv = -(-S // ATTN_BLOCK_Q)
    if schedule is None:
        nq = n_q_tiles if n_q_tiles is not None else nqv + (-(-Nt // ATTN_BLOCK_Q) if text_rows else 0)
        key = (H, Hkv, world, nq, tuple(costs) if costs is not None else None)
        schedule = _SCHED_CACHE.get(key)
        if schedule is None:
            schedule = _SCHED_CACHE[key] = make_schedule(H, Hkv, world, nq, costs)
    sch = schedule
    g = H // Hkv
    dev, dt = q.device, q.dtype
    ev = (lambda name: timing.setdefault(name, torch.cuda.Event(enable_timing=True)).record()) \
        if (timing is not None and q.is_cuda) else (lambda name: None)

    # ---- pack: for destination d, [B, S_r, nq_d + 2 nk_d, D] of my tokens
    ev("start")
    widths = [(b - a) + 2 * (kb - ka) for (a, b), (ka, kb) in zip(sch.q_heads, sch.kv_range)]
    in_splits = [B * S_r * wd * D for wd in widths]
    send = torch.empty(sum(in_splits), dtype=dt, device=dev)
    segs, off = [], 0
    for d in range(world):
        (a, b), (ka, kb) = sch.q_heads[d], sch.kv_range[d]
        blk = send[off:off + in_splits[d]].view(B, S_r, widths[d], D)
        nqh, nkh = b - a, kb - ka
        segs += [(q[:, :, a:b], blk[:, :, :nqh]), (k[:, :, ka:kb], blk[:, :, nqh:nqh + nkh]),
                 (v[:, :, ka:kb], blk[:, :, nqh + nkh:])]
        off += in_splits[d]
    copy_segments(segs)
    ev("packed")

    my_w = widths[rank]
    out_splits = [B * s * my_w * D for s in sizes]
    recv = torch.empty(sum(out_splits), dtype=dt, device=dev)
    dist.all_to_all_single(recv, send, out_splits, in_splits, group=group)
    ev("exchanged")
    if B == 1:
        x = recv.view(1, S, my_w, D)
    else:
        parts, o2 = [], 0
        for n in out_splits:
            parts.append(recv[o2:o2 + n].view(B, -1, my_w, D))
            o2 += n
        x = torch.cat(parts, dim=1)
    (qa, qb), (ka, kb) = sch.q_heads[rank], sch.kv_range[rank]
    nqh, nkh = qb - qa, kb - ka
    qf, kf, vf = x[:, :, :nqh], x[:, :, nqh:nqh + nkh], x[:, :, nqh + nkh:]

    # ---- local attention, one launch per piece
    out_loc = torch.empty(B, S, max(nqh, 1), D, dtype=dt, device=dev)
    tout_loc = torch.zeros(B, Nt, max(nqh, 1), D, dtype=dt, device=dev) if text_rows else None
    pieces = sch.pieces[rank]
    # Several pieces (a partial head beside whole heads): launch them on
    # concurrent streams, so the CTAs of one fill the last wave of another.
    streams = _piece_streams(dev, len(pieces)) if (q.is_cuda and len(pieces) > 1) else None
    if streams:
        cur = torch.cuda.current_stream(dev)
        for st in streams:
            st.wait_stream(cur)
    for j, p in enumerate(pieces):
        hq = slice(p.h0 - qa, p.h1 - qa)
        hk = slice(p.h0 // g - ka, (p.h1 - 1) // g + 1 - ka)
        tq = text_q[:, :, p.h0:p.h1] if text_rows else None
        tk = text_k[:, :, p.h0 // g:(p.h1 - 1) // g + 1] if Nt else None
        tv = text_v[:, :, p.h0 // g:(p.h1 - 1) // g + 1] if Nt else None
        args = (qf[:, :, hq], kf[:, :, hk], vf[:, :, hk], tq, tk, tv, (p.t0, p.t1),
                out_loc[:, :, hq], tout_loc[:, :, hq] if text_rows else None)
        if streams:
            with torch.cuda.stream(streams[j]):
                local_attention(*args)
        else:
            local_attention(*args)
    if streams:
        for st in streams:
            cur.wait_stream(st)
        for t in (x, out_loc, tout_loc):
            if t is not None:
                for st in streams:
                    t.record_stream(st)
    ev("attended")

    # ---- return: the video rows of my pieces to their token owners
    starts = [sum(sizes[:j]) for j in range(world)]

    def segments_between(src_rank: int, dst_rank: int):
        """(piece, token rows [s, e)) of src_rank's pieces inside dst_rank's shard."""
        lo, hi = starts[dst_rank], starts[dst_rank] + sizes[dst_rank]
        res = []
        for p in sch.pieces[src_rank]:
            s, e = _video_rows(p, nqv, S)
            s, e = max(s, lo), min(e, hi)
            if e > s:
                res.append((p, s, e))
        return res

    send_o_splits, segs = [], []
    for d in range(world):
        n = sum(B * (e - s) * (p.h1 - p.h0) * D for p, s, e in segments_between(rank, d))
        send_o_splits.append(n)
    send_o = torch.empty(max(1, sum(send_o_splits)), dtype=dt, device=dev)
    off = 0
    for d in range(world):
        for p, s, e in segments_between(rank, d):
            nh = p.h1 - p.h0
            n = B * (e - s) * nh * D
            segs.append((out_loc[:, s:e, p.h0 - qa:p.h1 - qa], send_o[off:off + n].view(B, e - s, nh, D)))
            off += n
    copy_segments(segs)
    recv_o_splits = []
    for src in range(world):
        recv_o_splits.append(sum(B * (e - s) * (p.h1 - p.h0) * D for p, s, e in segments_between(src, rank)))
    recv_o = torch.empty(max(1, sum(recv_o_splits)), dtype=dt, device=dev)
    dist.all_to_all_single(recv_o[:sum(recv_o_splits)], send_o[:sum(send_o_splits)],
                           recv_o_splits, send_o_splits, group=group)
    ev("returned")
    out = torch.empty(B, S_r, H, D, dtype=dt, device=dev)
    segs, off = [], 0
    a0 = starts[rank]
    for src in range(world):
        for p, s, e in segments_between(src, rank):
            nh = p.h1 - p.h0
            n = B * (e - s) * nh * D
            segs.append((recv_o[off:off + n].view(B, e - s, nh, D), out[:, s - a0:e - a0, p.h0:p.h1]))
            off += n
    copy_segments(segs)

    text_out = None
    if text_rows:
        tglob = torch.zeros(B, Nt, H, D, dtype=dt, device=dev)
        if nqh:
            tglob[:, :, qa:qb] += tout_loc[:, :, :nqh]
        dist.all_reduce(tglob, op=dist.ReduceOp.SUM, group=group)
        text_out = tglob
    ev("done")
    return out, text_out


def kernel_local_attention(metadata, scale: Optional[float] = None) -> Callable:
    """The default local step: the sm_100a kernel with the world = 1 mask."""
    from .block_sparse import block_sparse_attention
    from .sparse_attention import mask_for

    def run(q, k, v, tq, tk, tv, q_tiles, out, text_out):
        nt = 0 if tk is None else int(tk.shape[1])
        mask = mask_for(metadata, q.device, nt)
        block_sparse_attention(q, k, v, mask, tq, tk, tv, scale=scale, out=out, text_out=text_out,
                               q_tiles=q_tiles)
    return run


def mask_local_attention(mask, scale: Optional[float] = None) -> Callable:
    """Local step over a prebuilt BlockMask (the benchmark's path)."""
    from .block_sparse import block_sparse_attention

    def run(q, k, v, tq, tk, tv, q_tiles, out, text_out):
        block_sparse_attention(q, k, v, mask, tq, tk, tv, scale=scale, out=out, text_out=text_out,
                               q_tiles=q_tiles)
    return run
