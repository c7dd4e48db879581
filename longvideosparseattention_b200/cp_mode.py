"""Reference-compatible context parallelism: the reference's own world > 1
semantics (sequence shards, global frames gathered by one all-reduce,
rank-local windows), on the sm_100a kernel.

Reference behaviour restated (lvsa/lvsa_processor.py:131-137, 454-601,
643-706; lvsa/sparse_attention.py:107-129, 389-402, 643-706):

* every rank holds a contiguous token shard [gts, gts + S_r) of the T x P grid;
* globals = keyframes + boundary guards (the frames within W of each shard
  boundary), identical on all ranks;
* each rank writes the global-frame tokens it owns into a zeroed buffer and
  one all_reduce(SUM) assembles every global frame on every rank;
* a video query of frame f attends [all global frames; text] plus the tokens
  of f's window frames that are not global and lie on this rank;
* a text query attends [this rank's video tokens; text].

B200 mapping: two launches of the block-sparse kernel per layer.  Video rows:
the video segment is the local shard (``token_offset`` = gts, tile CSR over
local tiles with frame bitsets window(f) minus globals), the dense second
segment is the all-reduced [globals; text] buffer.  Text rows: the video
segment again with the text as second segment, rows from ``first_q_tile``.
The all-reduce is NCCL over NVLink (``torch.distributed``), with the buffer
cached across layers.  The Ulysses path (``ulysses.py``) remains the faster
multi-GPU mode; this one reproduces the reference's outputs rank by rank.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np
import torch

from .block_sparse import ATTN_BLOCK_K, ATTN_BLOCK_Q, block_sparse_attention
from .sparse_attention import compute_boundary_guard_frames, compute_global_indices, get_window_bounds


@dataclass
class ShardMask:
    """Tile CSR of one launch over a sequence shard (the fields
    ``block_sparse_attention`` reads)."""
    total_frames: int
    num_patches: int
    frame_words: int
    n_video: int
    n_text: int
    n_q_video_tiles: int
    n_q_tiles: int
    n_k_video_tiles: int
    token_offset: int
    first_q_tile: int
    frame_bits: torch.Tensor
    tile_indptr: torch.Tensor
    tile_indices: torch.Tensor
    tile_flags: torch.Tensor
    block_q: int = ATTN_BLOCK_Q
    block_k: int = ATTN_BLOCK_K


@dataclass
class ShardPattern:
    """Per-rank, per-step structures of the reference's world > 1 path."""
    T: int
    P: int
    rank: int
    world: int
    global_token_start: int
    local_seq: int
    global_indices: List[int]
    n_text: int
    video: ShardMask            # video rows: local windows + dense [globals; text]
    text: Optional[ShardMask]   # text rows: local video + text (None without text)
    guards: List[int] = field(default_factory=list)


def _bits(rows: List[List[int]], T: int) -> np.ndarray:
    words = (T + 31) // 32
    out = np.zeros((T, words), dtype=np.uint32)
    for f, frames in enumerate(rows):
        for g in frames:
            out[f, g >> 5] |= np.uint32(1) << np.uint32(g & 31)
    return out


def _dense_cols(n_dense: int, nkv: int, BK: int) -> List[Tuple[int, int]]:
    nt = -(-n_dense // BK)
    return [(nkv + j, 1 if (j + 1) * BK > n_dense else 0) for j in range(nt)]


def build_shard_pattern(T: int, P: int, W: int, n_first: int, kfi: Optional[int], offset: int,
                        rank: int, world: int, n_text: int = 0, expand: bool = True,
                        device: Optional[torch.device] = None,
                        global_indices: Optional[List[int]] = None) -> ShardPattern:
    """Host build (per rank and denoising step, like the reference's
    LVSAMetadata.build) of the two launches' tile CSRs.  ``global_indices``
    (keyframes and boundary guards, e.g. a reference LVSAMetadata's) replaces
    the global frames derived from n_first / kfi / offset."""
    total = T * P
    if total % world:
        raise AssertionError(f"total_seq={total} (T={T} x P={P}) must be divisible by world={world}.")
    S_r = total // world
    gts = rank * S_r
    guards = compute_boundary_guard_frames(T, S_r, P, world, W)
    if global_indices is not None:
        globals_ = sorted(set(int(g) for g in global_indices))
    else:
        globals_ = sorted(set(compute_global_indices(T, n_first, kfi, offset)) | set(guards))
    gset = set(globals_)
    # Frames a query frame attends inside the shard: its window minus globals.
    allowed = []
    for f in range(T):
        lo, hi = get_window_bounds(f, W, T, expand, gset, len(globals_))
        allowed.append([g for g in range(lo, hi + 1) if g not in gset])
    BQ, BK = ATTN_BLOCK_Q, ATTN_BLOCK_K
    nqv, nkv = -(-S_r // BQ), -(-S_r // BK)
    tok_frame = (gts + np.arange(S_r)) // P
    kt_lo = tok_frame[np.arange(nkv) * BK]
    kt_hi = tok_frame[np.minimum(np.arange(nkv) * BK + BK, S_r) - 1]
    kt_partial = (np.arange(nkv) + 1) * BK > S_r
    allow_mat = np.zeros((T, T + 1), dtype=np.int32)  # prefix counts of allowed frames per query frame
    for f in range(T):
        row = np.zeros(T, dtype=np.int32)
        row[allowed[f]] = 1
        allow_mat[f, 1:] = np.cumsum(row)
    n_dense = len(globals_) * P + n_text
    dense = _dense_cols(n_dense, nkv, BK)
    indptr, indices, flags = [0], [], []
    for qt in range(nqv):
        qf = sorted(set(tok_frame[qt * BQ:min(S_r, qt * BQ + BQ)].tolist()))
        cnt = allow_mat[qf][:, kt_hi + 1] - allow_mat[qf][:, kt_lo]     # [len(qf), nkv]
        width = kt_hi - kt_lo + 1
        active = (cnt > 0).any(axis=0)
        full = (cnt == width[None, :]).all(axis=0) & ~kt_partial
        for kt in np.nonzero(active)[0]:
            indices.append(int(kt))
            flags.append(0 if full[kt] else 1)
        for kt, fl in dense:
            indices.append(kt)
            flags.append(fl)
        indptr.append(len(indices))
    dev = device if device is not None else torch.device("cuda")

    def _mask(ip, ix, fl, n_dense_seg, nq, first):
        return ShardMask(T, P, (T + 31) // 32, S_r, n_dense_seg, nqv, nq, nkv, gts, first,
                         torch.from_numpy(_bits(allowed, T)).to(dev),
                         torch.tensor(ip, dtype=torch.int32, device=dev),
                         torch.tensor(ix if ix else [0], dtype=torch.int32, device=dev),
                         torch.tensor(fl if fl else [0], dtype=torch.uint8, device=dev))
    # The dense segment's rows exist for the geometry check but are never run
    # (no text queries in this launch): their CSR rows are empty.
    n_phantom = -(-n_dense // BQ) if n_dense else 0
    indptr += [indptr[-1]] * n_phantom
    video = _mask(indptr, indices, flags, n_dense, nqv + n_phantom, 0)
    text = None
    if n_text > 0:
        nqt = -(-n_text // BQ)
        ip, ix, fl = [0] * (nqv + 1), [], []
        tcols = _dense_cols(n_text, nkv, BK)
        for _ in range(nqt):
            for kt in range(nkv):
                ix.append(kt)
                fl.append(1 if kt_partial[kt] else 0)
            for kt, f in tcols:
                ix.append(kt)
                fl.append(f)
            ip.append(len(ix))
        text = _mask(ip, ix, fl, n_text, nqv + nqt, nqv)
    return ShardPattern(T, P, rank, world, gts, S_r, globals_, n_text, video, text, guards)


class GlobalKV:
    """The [2, B, G*P + n_text, Hkv, D] buffer of global-frame K/V (+ text),
    reused across layers: ``fill`` zeroes it and writes the global-frame
    tokens this rank owns, ``all_reduce(SUM)`` over the group assembles every
    global frame on every rank (lvsa/lvsa_processor.py:643-706), ``finish``
    copies the replicated text into the tail."""

    def __init__(self) -> None:
        self.buf: Optional[torch.Tensor] = None

    def fill(self, key: torch.Tensor, value: torch.Tensor, pat: ShardPattern) -> torch.Tensor:
        B, S_r, Hkv, D = key.shape
        P, gts, G = pat.P, pat.global_token_start, len(pat.global_indices)
        shape = (2, B, G * P + pat.n_text, Hkv, D)
        if (self.buf is None or tuple(self.buf.shape) != shape or self.buf.dtype != key.dtype
                or self.buf.device != key.device):
            self.buf = torch.empty(shape, dtype=key.dtype, device=key.device)
        buf = self.buf
        buf.zero_()
        for gi, gf in enumerate(pat.global_indices):
            s, e = max(gf * P, gts), min((gf + 1) * P, gts + S_r)
            if s >= e:
                continue  # owned by other ranks
            dst = slice(gi * P + (s - gf * P), gi * P + (e - gf * P))
            buf[0, :, dst] = key[:, s - gts:e - gts]
            buf[1, :, dst] = value[:, s - gts:e - gts]
        return buf

    def finish(self, pat: ShardPattern, text_k: Optional[torch.Tensor], text_v: Optional[torch.Tensor]
               ) -> Tuple[torch.Tensor, torch.Tensor]:
        G = len(pat.global_indices) * pat.P
        if pat.n_text:
            self.buf[0, :, G:] = text_k
            self.buf[1, :, G:] = text_v
        return self.buf[0], self.buf[1]


def cp_attend(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, pat: ShardPattern,
              k_dense: torch.Tensor, v_dense: torch.Tensor, text_q: Optional[torch.Tensor] = None,
              text_k: Optional[torch.Tensor] = None, text_v: Optional[torch.Tensor] = None
              ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """The two launches of one rank, given the assembled [globals; text] K/V."""
    out, _ = block_sparse_attention(query, key, value, pat.video, None, k_dense, v_dense)
    text_out = None
    if text_q is not None and pat.text is not None:
        # Text rows only (first_q_tile skips the video rows, so `query` is not written).
        _, text_out = block_sparse_attention(query, key, value, pat.text, text_q, text_k, text_v, out=query)
    return out, text_out


def cp_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, pat: ShardPattern,
                 kv: GlobalKV, text_q: Optional[torch.Tensor] = None, text_k: Optional[torch.Tensor] = None,
                 text_v: Optional[torch.Tensor] = None, group=None
                 ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """One layer of the reference's world > 1 attention on this rank:
    (out [B, S_r, H, D], text_out or None)."""
    import torch.distributed as dist
    nt = 0 if text_k is None else int(text_k.shape[1])
    if nt != pat.n_text:
        raise AssertionError(f"text length {nt} does not match the shard pattern ({pat.n_text})")
    buf = kv.fill(key, value, pat)
    if pat.world > 1:
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    kg, vg = kv.finish(pat, text_k, text_v)
    return cp_attend(query, key, value, pat, kg, vg, text_q, text_k, text_v)
