"""CPU restatement of LVSA's sparse-attention path (test oracle).

TEST INFRASTRUCTURE ONLY -- imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``; never by the shipped package.

Reference: JiusiServe/LongVideoSparseAttention v1.2.0.  Every function below
names the reference lines it restates.  The frame-level pattern functions are
plain Python integer arithmetic (the reference's own algorithm, restated);
the attention arithmetic is numpy float32 matmuls with a float64 softmax
normaliser, mirroring the reference's per-frame SDPA loop
(``lvsa/sparse_attention.py:643-706``).

Parity pinning: this module is checked against golden vectors produced by
importing the unmodified reference (``tests/golden/make_golden.py``) and
against the reference test-suite's known answers (``tests/test_oracle.py``).

The tile-level CSR (``tile_csr``) has no reference counterpart; it is the
deterministic expansion of the reference's frame sets to (block_q x block_k)
tiles, defined as:

* video tile (qb, kb) is active iff some valid query token t in
  [qb*BQ, min(Nv,(qb+1)*BQ)) and key token u in [kb*BK, min(Nv,(kb+1)*BK))
  satisfy frame(u) in attended(frame(t));
* its flag bit 0 ("needs in-tile mask") is set unless every such (t, u) pair
  is allowed and (kb+1)*BK <= Nv;
* text tiles (text tokens are their own segment, tiled from 0) are appended
  after the video tiles, always active; flag set iff the tile runs past the
  end of its segment.  Text query rows are dense over every video and text
  tile.  Columns within a row are strictly ascending.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Set, Tuple

import numpy as np

# --------------------------------------------------------------------------
# Frame-level pattern (reference: lvsa/sparse_attention.py)
# --------------------------------------------------------------------------


def adaptive_window_bounds(f: int, W: int, T: int) -> Tuple[int, int]:
    """Constant-width window shifted inside [0, T-1].  lvsa/sparse_attention.py:40-47."""
    lo = max(0, min(f - W, T - 1 - 2 * W))
    hi = min(T - 1, max(f + W, 2 * W))
    return lo, hi


def expanded_window_bounds(f: int, W: int, T: int, global_set: Set[int],
                           global_count: int) -> Tuple[int, int]:
    """Grow the adaptive window, left then right, until it holds
    min(2W+1, T-|G|) non-global frames.  lvsa/sparse_attention.py:50-86."""
    lo, hi = adaptive_window_bounds(f, W, T)
    need = min(2 * W + 1, T - global_count)
    have = sum(1 for x in range(lo, hi + 1) if x not in global_set)
    while have < need:
        grew = False
        if lo > 0:
            lo -= 1
            grew = True
            if lo not in global_set:
                have += 1
        if have >= need:
            break
        if hi < T - 1:
            hi += 1
            grew = True
            if hi not in global_set:
                have += 1
        if not grew:
            break
    return lo, hi


def get_window_bounds(f: int, W: int, T: int, expand: bool, global_set: Set[int],
                      global_count: int) -> Tuple[int, int]:
    """W == 0 gives the empty range (f, f-1).  lvsa/sparse_attention.py:89-104."""
    if W == 0:
        return f, f - 1
    if expand:
        return expanded_window_bounds(f, W, T, global_set, global_count)
    return adaptive_window_bounds(f, W, T)


def compute_boundary_guard_frames(total_frames: int, local_seq: int, num_patches: int,
                                  world: int, window_size: int) -> List[int]:
    """Frames within +-W of every rank split.  lvsa/sparse_attention.py:107-129."""
    out: Set[int] = set()
    for r in range(1, world):
        bf = (r * local_seq) // num_patches
        out.update(range(max(0, bf - window_size), min(total_frames, bf + window_size + 1)))
    return sorted(out)


def compute_auto_kfi(total_frames: int, window_size: int, n_first_frames: int,
                     reference_frames: int = 21, sparsity_scale: float = 1.0) -> int:
    """max(strict, closed-form fallback) keyframe interval.
    lvsa/sparse_attention.py:132-195."""
    T = total_frames
    scaled_ref = max(n_first_frames + 1, int(reference_frames * sparsity_scale))
    if T <= scaled_ref:
        return 1
    target = min(scaled_ref, T)
    target_g = max(n_first_frames, target - min(2 * window_size + 1, T))
    strict = 1
    for kfi in range(T, 0, -1):
        s = set(range(min(n_first_frames, T)))
        s.update(range(0, T, kfi))
        if len(s) >= target_g:
            strict = kfi
            break
    mandatory = 2 * window_size + n_first_frames
    fb = math.ceil(max(T - mandatory, scaled_ref - mandatory) / max(scaled_ref - mandatory, 1))
    return max(strict, fb)


def compute_global_indices(total_frames: int, n_first_frames: int,
                           key_frame_interval: Optional[int], offset: int = 0) -> List[int]:
    """First frames plus ceil(T/kfi) keyframes at (offset + i*kfi) mod T.
    lvsa/sparse_attention.py:198-216."""
    g = set(range(min(n_first_frames, total_frames)))
    if key_frame_interval is not None and key_frame_interval > 0:
        for i in range(math.ceil(total_frames / key_frame_interval)):
            g.add((offset + i * key_frame_interval) % total_frames)
    return sorted(g)


def frame_pattern(T: int, P: int, W: int, n_first: int, kfi: Optional[int],
                  offset: int = 0, expand: bool = True, rank: int = 0, world: int = 1,
                  boundary_guards: Optional[Sequence[int]] = None) -> Dict:
    """All frame-level structures of ``LVSAMetadata.build``.

    lvsa/sparse_attention.py:335-484 (build), :510-547 (attended indices),
    :550-635 (frame CSR).  Returned arrays use the reference dtypes.
    """
    total = T * P
    assert total % world == 0, f"total_seq={total} must be divisible by world={world}"
    local = total // world
    gts = rank * local
    g = sorted(set(compute_global_indices(T, n_first, kfi, offset)) | set(boundary_guards or []))
    gs = set(g)
    gc = len(g)
    first, last = gts // P, (gts + local - 1) // P

    local_frames = []
    for f in range(first, last + 1):
        local_frames.append((f, max(f * P, gts) - gts, min((f + 1) * P, gts + local) - gts))

    bounds = np.zeros((T, 2), dtype=np.int32)
    for f in range(T):
        bounds[f] = get_window_bounds(f, W, T, expand, gs, gc)

    window_ctx: Dict[int, List[Tuple[int, int]]] = {}
    for f, _, _ in local_frames:
        lo, hi = bounds[f]
        parts = []
        for wf in range(int(lo), int(hi) + 1):
            if wf in gs:
                continue
            s, e = max(wf * P, gts), min((wf + 1) * P, gts + local)
            if s < e:
                parts.append((s - gts, e - gts))
        window_ctx[f] = parts

    gmask = np.zeros(T, dtype=np.int8)
    gmask[g] = 1

    attended: List[List[int]] = []
    for f in range(T):
        lo, hi = int(bounds[f, 0]), int(bounds[f, 1])
        attended.append(sorted(gs | set(range(lo, hi + 1))))

    # [T_local, C] padded with the row's last entry (lvsa/sparse_attention.py:540-545)
    loc = [attended[f] for f in range(first, last + 1)]
    C = max(len(a) for a in loc)
    att_idx = np.empty((len(loc), C), dtype=np.int32)
    for i, a in enumerate(loc):
        att_idx[i, :len(a)] = a
        att_idx[i, len(a):] = a[-1]

    # frame CSR over compacted frames (lvsa/sparse_attention.py:562-607)
    MB = -(-local // P)
    per_q = []
    for qi in range(MB):
        f = first + qi
        lo, hi = int(bounds[f, 0]), int(bounds[f, 1])
        s = set(g)
        for wf in range(lo, hi + 1):
            if wf in gs:
                continue
            if max(wf * P, gts) < min((wf + 1) * P, gts + local):
                s.add(wf)
        per_q.append(s)
    compact = sorted(set().union(*per_q)) if per_q else []
    to_c = {f: i for i, f in enumerate(compact)}
    indptr = [0]
    indices: List[int] = []
    for s in per_q:
        indices.extend(sorted(to_c[f] for f in s))
        indptr.append(len(indices))

    return dict(
        T=T, P=P, W=W, local_seq=local, global_token_start=gts,
        global_indices=g, global_set=gs, local_frames=local_frames, window_ctx=window_ctx,
        global_frame_mask=gmask, window_bounds=bounds, attended=attended,
        attended_indices=att_idx, attended_C=C,
        fi_indptr=np.asarray(indptr, dtype=np.int32),
        fi_indices=np.asarray(indices, dtype=np.int32),
        fi_MB=MB, fi_M=MB * P, fi_compact_n=len(compact), fi_N=len(compact) * P,
    )


# --------------------------------------------------------------------------
# Tile-level CSR (expansion of the frame sets; definition in the module doc)
# --------------------------------------------------------------------------


def tile_csr(attended: Sequence[Sequence[int]], T: int, P: int, n_video: int,
             n_text: int = 0, block_q: int = 128, block_k: int = 128):
    """Return (indptr int32, indices int32, flags uint8, n_q_video, n_k_video)."""
    BQ, BK = block_q, block_k
    nqv, nkv = -(-n_video // BQ), -(-n_video // BK)
    nqt, nkt = -(-n_text // BQ), -(-n_text // BK)
    att_sets = [set(a) for a in attended]
    text_cols = [(nkv + j, 1 if (j + 1) * BK > n_text else 0) for j in range(nkt)]
    indptr = [0]
    indices: List[int] = []
    flags: List[int] = []
    for qb in range(nqv):
        t0, t1 = qb * BQ, min(n_video, (qb + 1) * BQ)
        qf = range(t0 // P, (t1 - 1) // P + 1)
        union = set().union(*(att_sets[f] for f in qf))
        inter = set.intersection(*(att_sets[f] for f in qf))
        tiles = set()
        for f in union:
            tiles.update(range((f * P) // BK, (min(n_video, (f + 1) * P) - 1) // BK + 1))
        for kb in sorted(tiles):
            u0, u1 = kb * BK, min(n_video, (kb + 1) * BK)
            full = (kb + 1) * BK <= n_video and all(
                f in inter for f in range(u0 // P, (u1 - 1) // P + 1))
            indices.append(kb)
            flags.append(0 if full else 1)
        for kb, fl in text_cols:
            indices.append(kb)
            flags.append(fl)
        indptr.append(len(indices))
    for _ in range(nqt):
        for kb in range(nkv):
            indices.append(kb)
            flags.append(1 if (kb + 1) * BK > n_video else 0)
        for kb, fl in text_cols:
            indices.append(kb)
            flags.append(fl)
        indptr.append(len(indices))
    return (np.asarray(indptr, dtype=np.int32), np.asarray(indices, dtype=np.int32),
            np.asarray(flags, dtype=np.uint8), nqv, nkv)


def flop_counts(attended, T, P, n_video, n_text, H, D, block_q=128, block_k=128):
    """(FLOP_tiles, FLOP_exact): 4*D*H per (query, key) pair; tiles counted at
    their clipped area for video x video, text terms exact."""
    indptr, indices, _, nqv, nkv = tile_csr(attended, T, P, n_video, 0, block_q, block_k)
    area = 0
    for qb in range(nqv):
        rows = min(n_video, (qb + 1) * block_q) - qb * block_q
        for kb in indices[indptr[qb]:indptr[qb + 1]]:
            area += rows * (min(n_video, (int(kb) + 1) * block_k) - int(kb) * block_k)
    text = n_video * n_text + n_text * (n_video + n_text)
    exact = sum(P * len(attended[f]) * P for f in range(T))
    c = 4 * D * H
    return c * (area + text), c * (exact + text)


# --------------------------------------------------------------------------
# Attention arithmetic (reference: lvsa_sdpa + the processor's text handling)
# --------------------------------------------------------------------------


def _softmax_av(q, k, v, scale):
    """q [n,D], k [m,D], v [m,D] float32 -> [n,D] float32 (float64 normaliser)."""
    s = (q @ k.T) * np.float32(scale)
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s.astype(np.float64))
    out = (p.astype(np.float32) @ v).astype(np.float64) / p.sum(axis=1, keepdims=True)
    return out.astype(np.float32)


def attention(q, k, v, pattern: Dict, text_q=None, text_k=None, text_v=None,
              scale: Optional[float] = None, frames: Optional[Sequence[int]] = None,
              heads: Optional[Sequence[int]] = None, text_rows: bool = True):
    """Block-sparse LVSA attention on host arrays laid out [B, S, H, D].

    Video query frame f attends to every token of attended(f) (globals plus
    its window; lvsa/sparse_attention.py:674-704) and to all text tokens
    (text K/V appended to the global K/V, lvsa/lvsa_processor.py:545-549).
    Text queries attend densely to video + text (lvsa/lvsa_processor.py:584-591).
    GQA maps query head h to key head h // (H / Hkv), as SDPA's enable_gqa.

    ``frames`` restricts the computed video rows (others are left NaN);
    ``heads`` restricts the heads likewise.  Returns (out_video, out_text).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    B, Nv, H, D = q.shape
    Hkv = k.shape[2]
    grp = H // Hkv
    P = pattern["P"]
    T = pattern["T"]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    has_text = text_k is not None and text_k.shape[1] > 0
    if has_text:
        tk = np.asarray(text_k, dtype=np.float32)
        tv = np.asarray(text_v, dtype=np.float32)
    out = np.full(q.shape, np.nan, dtype=np.float32)
    heads = list(range(H)) if heads is None else list(heads)
    frames = list(range(T)) if frames is None else list(frames)
    for f in frames:
        idx = np.concatenate([np.arange(g * P, (g + 1) * P) for g in pattern["attended"][f]])
        for b in range(B):
            for h in heads:
                kh = h // grp
                kk, vv = k[b, idx, kh], v[b, idx, kh]
                if has_text:
                    kk = np.concatenate([kk, tk[b, :, kh]])
                    vv = np.concatenate([vv, tv[b, :, kh]])
                out[b, f * P:(f + 1) * P, h] = _softmax_av(q[b, f * P:(f + 1) * P, h], kk, vv, scale)
    out_text = None
    if text_q is not None and text_rows and text_q.shape[1] > 0:
        tq = np.asarray(text_q, dtype=np.float32)
        out_text = np.full(tq.shape, np.nan, dtype=np.float32)
        for b in range(B):
            for h in heads:
                kh = h // grp
                kk = np.concatenate([k[b, :, kh], tk[b, :, kh]])
                vv = np.concatenate([v[b, :, kh], tv[b, :, kh]])
                out_text[b, :, h] = _softmax_av(tq[b, :, h], kk, vv, scale)
    return out, out_text


def attention_torch_cpu(q, k, v, pattern: Dict, text_k=None, text_v=None,
                        frames: Optional[Sequence[int]] = None):
    """The reference's own CPU arithmetic for the video rows: per query frame,
    concatenate the anchor and window K/V (plus text) and call torch's fp32
    scaled_dot_product_attention -- lvsa/sparse_attention.py:674-704 with the
    text K/V appended as lvsa/lvsa_processor.py:545-549.  Multithreaded by
    torch; used as the timed CPU baseline.  Inputs: torch CPU [B, S, H, D]."""
    import torch
    import torch.nn.functional as F
    P = pattern["P"]
    B, N, H, D = q.shape
    gqa = k.shape[2] != H
    gidx = pattern["global_indices"]
    ar = torch.arange(P)
    gtok = (torch.tensor(gidx)[:, None] * P + ar[None, :]).reshape(-1)
    kg, vg = k[:, gtok], v[:, gtok]
    if text_k is not None and text_k.shape[1] > 0:
        kg, vg = torch.cat([kg, text_k], 1), torch.cat([vg, text_v], 1)
    out = torch.empty_like(q)
    for f in (range(pattern["T"]) if frames is None else frames):
        lo, hi = (int(x) for x in pattern["window_bounds"][f])
        win = [w for w in range(lo, hi + 1) if w not in pattern["global_set"]]
        kc = torch.cat([kg] + [k[:, w * P:(w + 1) * P] for w in win], 1)
        vc = torch.cat([vg] + [v[:, w * P:(w + 1) * P] for w in win], 1)
        o = F.scaled_dot_product_attention(q[:, f * P:(f + 1) * P].transpose(1, 2), kc.transpose(1, 2),
                                           vc.transpose(1, 2), enable_gqa=gqa)
        out[:, f * P:(f + 1) * P] = o.transpose(1, 2)
    return out


# ---------------------------------------------------------------------------
# QK prologue (the adapters' norm + rotary embedding), fp32, torch on CPU.
def norm_rope(x, norm, weight=None, bias=None, eps=1e-6, cos=None, sin=None, rope_offset=0):
    """x [B, S, H, D] -> fp32.  norm: None | "rms_row" (RMSNorm over the H*D
    row, Wan's norm_q/norm_k, lvsa/adapters/wan.py:48-67) | "rms_head"
    (per-head RMSNorm, lvsa/adapters/hunyuan_video.py:71-103) | "layer_head"
    (per-head LayerNorm, lvsa/adapters/cogvideox.py:88-117); then the
    interleaved-pair rotation of lvsa/rope.py:10-28 with cos/sin given as pair
    angle tables [S_tab, D/2] or [B, S_tab, D/2], rows rope_offset + s."""
    import torch
    B, S, H, D = x.shape
    f = x.float()
    if norm == "rms_row":
        r = f.reshape(B, S, H * D)
        r = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps)
        if weight is not None:
            r = r * weight.float()
        f = r.reshape(B, S, H, D)
    elif norm == "rms_head":
        f = f * torch.rsqrt(f.pow(2).mean(-1, keepdim=True) + eps)
        if weight is not None:
            f = f * weight.float()
    elif norm == "layer_head":
        mu = f.mean(-1, keepdim=True)
        f = (f - mu) * torch.rsqrt((f - mu).pow(2).mean(-1, keepdim=True) + eps)
        if weight is not None:
            f = f * weight.float()
        if bias is not None:
            f = f + bias.float()
    if cos is not None:
        c = cos.float()[..., rope_offset:rope_offset + S, :]
        s = sin.float()[..., rope_offset:rope_offset + S, :]
        c = c.unsqueeze(-2) if c.dim() == 3 else c[None, :, None, :]
        s = s.unsqueeze(-2) if s.dim() == 3 else s[None, :, None, :]
        x0, x1 = f[..., 0::2], f[..., 1::2]
        out = torch.empty_like(f)
        out[..., 0::2] = x0 * c - x1 * s
        out[..., 1::2] = x0 * s + x1 * c
        f = out
    return f


# ---------------------------------------------------------------------------
# Reference context parallelism (world > 1): one rank's output.
def attention_cp(q, k, v, k_full, v_full, T, P, W, n_first, kfi, offset, rank, world, expand=True,
                 text_q=None, text_k=None, text_v=None, scale=None):
    """The reference's sequence-sharded LVSA on rank ``rank`` of ``world``.

    q/k/v [B, S_r, H(kv), D] are this rank's tokens; k_full/v_full [B, T*P,
    Hkv, D] the whole sequence, from which the global frames are taken (what
    ``_build_global_kv``'s all_reduce assembles, lvsa/lvsa_processor.py:
    643-706).  Globals = user keyframes + boundary guards
    (lvsa/lvsa_processor.py:131-137, lvsa/sparse_attention.py:107-129).
    Video rows of local frame f attend [global frames; text] + the parts of
    f's window frames (globals excluded) that are on this rank
    (lvsa/sparse_attention.py:389-402, 643-706, processor :545-549); text rows
    attend [this rank's video keys; text] (processor :586-591).
    Returns (out [B, S_r, H, D], text_out or None), float32."""
    B, S_r, H, D = q.shape
    Hkv = k.shape[2]
    rep = H // Hkv
    sc = scale if scale is not None else 1.0 / np.sqrt(D)
    guards = compute_boundary_guard_frames(T, T * P // world, P, world, W)
    fp = frame_pattern(T, P, W, n_first, kfi, offset, expand, rank, world, boundary_guards=guards)
    g = [int(x) for x in np.nonzero(fp["global_frame_mask"])[0]]
    gidx = np.concatenate([np.arange(f * P, (f + 1) * P) for f in g]) if g else np.zeros(0, dtype=np.int64)
    out = np.zeros((B, S_r, H, D), dtype=np.float32)
    for b in range(B):
        kg, vg = k_full[b][gidx], v_full[b][gidx]
        if text_k is not None:
            kg, vg = np.concatenate([kg, text_k[b]]), np.concatenate([vg, text_v[b]])
        for f, s, e in fp["local_frames"]:
            parts = fp["window_ctx"][f]
            kc = np.concatenate([kg] + [k[b][ps:pe] for ps, pe in parts])
            vc = np.concatenate([vg] + [v[b][ps:pe] for ps, pe in parts])
            for h in range(H):
                out[b, s:e, h] = _softmax_av(q[b, s:e, h].astype(np.float32), kc[:, h // rep].astype(np.float32),
                                             vc[:, h // rep].astype(np.float32), sc)
    tout = None
    if text_q is not None:
        nt = text_q.shape[1]
        tout = np.zeros((B, nt, H, D), dtype=np.float32)
        for b in range(B):
            kc, vc = np.concatenate([k[b], text_k[b]]), np.concatenate([v[b], text_v[b]])
            for h in range(H):
                tout[b, :, h] = _softmax_av(text_q[b, :, h].astype(np.float32), kc[:, h // rep].astype(np.float32),
                                            vc[:, h // rep].astype(np.float32), sc)
    return out, tout
