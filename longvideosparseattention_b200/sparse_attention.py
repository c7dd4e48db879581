"""Drop-in for the reference module ``lvsa/sparse_attention.py``.

Same names, signatures and error behaviour as the reference:

* pattern helpers (``adaptive_window_bounds`` ... ``compute_global_indices``),
  pure host integer arithmetic, restated from lvsa/sparse_attention.py:40-216;
* ``LVSAMetadata`` with every reference field (lvsa/sparse_attention.py:286-333)
  built on the host (vectorised) by ``LVSAMetadata.build``; its GPU form -- the
  tile CSR the kernel consumes -- comes from the GPU mask builder via
  ``LVSAMetadata.block_mask(device, n_text)`` and is cached per device;
* ``lvsa_sdpa`` / ``sparse_windowed_attention`` run the sm_100a block-sparse
  kernel for every backend name: there is one kernel and no CPU path.
"""

from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Set, Tuple

import torch

from .block_sparse import ATTN_BLOCK_K, ATTN_BLOCK_Q, BlockMask, block_sparse_attention, build_block_mask

# --------------------------------------------------------------------------
# Pattern helpers
# --------------------------------------------------------------------------


def adaptive_window_bounds(f: int, W: int, T: int) -> Tuple[int, int]:
    """Window of constant width min(2W+1, T) shifted to stay inside [0, T-1]
    (lvsa/sparse_attention.py:40-47)."""
    return max(0, min(f - W, T - 1 - 2 * W)), min(T - 1, max(f + W, 2 * W))


def expanded_window_bounds(f: int, W: int, T: int, global_set: Set[int],
                           global_count: int) -> Tuple[int, int]:
    """Adaptive window widened alternately left then right until it covers
    min(2W+1, T - global_count) non-anchor frames (lvsa/sparse_attention.py:50-86)."""
    lo, hi = adaptive_window_bounds(f, W, T)
    target = min(2 * W + 1, T - global_count)
    covered = sum(x not in global_set for x in range(lo, hi + 1))
    while covered < target:
        moved = False
        if lo > 0:
            lo -= 1
            moved = True
            covered += lo not in global_set
        if covered >= target:
            break
        if hi < T - 1:
            hi += 1
            moved = True
            covered += hi not in global_set
        if not moved:
            break
    return lo, hi


def get_window_bounds(f: int, W: int, T: int, expand: bool, global_set: Set[int],
                      global_count: int) -> Tuple[int, int]:
    """(f, f-1) -- an empty range -- when W == 0 (lvsa/sparse_attention.py:89-104)."""
    if W == 0:
        return (f, f - 1)
    return (expanded_window_bounds(f, W, T, global_set, global_count) if expand
            else adaptive_window_bounds(f, W, T))


def compute_boundary_guard_frames(total_frames: int, local_seq: int, num_patches: int,
                                  world: int, window_size: int) -> List[int]:
    """Frames within W of each context-parallel token split
    (lvsa/sparse_attention.py:107-129)."""
    guards: Set[int] = set()
    for r in range(1, world):
        bf = (r * local_seq) // num_patches
        guards.update(range(max(0, bf - window_size), min(total_frames, bf + window_size + 1)))
    return sorted(guards)


def compute_auto_kfi(total_frames: int, window_size: int, n_first_frames: int,
                     reference_frames: int = 21, sparsity_scale: float = 1.0) -> int:
    """Keyframe interval targeting ``reference_frames * sparsity_scale``
    attended frames: max(strict, closed-form fallback)
    (lvsa/sparse_attention.py:132-195)."""
    T = total_frames
    budget = max(n_first_frames + 1, int(reference_frames * sparsity_scale))
    if T <= budget:
        return 1
    want_globals = max(n_first_frames, min(budget, T) - min(2 * window_size + 1, T))
    strict = 1
    for kfi in range(T, 0, -1):
        if len(set(range(min(n_first_frames, T))) | set(range(0, T, kfi))) >= want_globals:
            strict = kfi
            break
    mandatory = 2 * window_size + n_first_frames
    fallback = math.ceil(max(T - mandatory, budget - mandatory) / max(budget - mandatory, 1))
    return max(strict, fallback)


def compute_global_indices(total_frames: int, n_first_frames: int,
                           key_frame_interval: Optional[int], offset: int = 0) -> List[int]:
    """Sorted anchors: the first frames and ceil(T/kfi) keyframes at
    (offset + i*kfi) mod T (lvsa/sparse_attention.py:198-216)."""
    anchors = set(range(min(n_first_frames, total_frames)))
    if key_frame_interval is not None and key_frame_interval > 0:
        n = -(-total_frames // key_frame_interval)
        anchors.update((offset + i * key_frame_interval) % total_frames for i in range(n))
    return sorted(anchors)


def print_attention_mask_compact(total_frames: int, window_size: int, global_set: Set[int],
                                 expand_window: bool, file=None) -> None:
    """One character per key frame: G anchor, W window, X both, . skipped
    (lvsa/sparse_attention.py:219-278)."""
    T, W = total_frames, window_size
    pad = len(str(T - 1)) if T > 1 else 1
    print(" " * (pad + 2) + "".join(str(k % 10) if k % 5 == 0 else " " for k in range(T)), file=file)
    counts = []
    for f in range(T):
        lo, hi = get_window_bounds(f, W, T, expand_window, global_set, len(global_set))
        win = set(range(lo, hi + 1)) if lo <= hi else set()
        row = "".join("X" if (k in global_set and k in win) else "G" if k in global_set
                      else "W" if k in win else "." for k in range(T))
        counts.append(len(global_set | win))
        print(f"{f:>{pad}} |{row}| {counts[-1]}", file=file)
    if counts:
        print(f"G=global W=window X=both .=skip  min={min(counts)} max={max(counts)} "
              f"avg={sum(counts) / len(counts):.1f}/{T}", file=file)


# --------------------------------------------------------------------------
# LVSAMetadata
# --------------------------------------------------------------------------


@dataclass
class LVSAMetadata:
    """All index structures of one pattern; field names and dtypes as the
    reference dataclass (lvsa/sparse_attention.py:286-333)."""

    total_latent_frames: int
    num_patches: int
    window_size: int
    n_first_frames: int
    key_frame_interval: Optional[int]
    expand_window: bool
    rank: int
    world: int
    local_seq: int
    global_token_start: int
    global_indices: List[int]
    global_set: Set[int]
    local_frames: List[Tuple[int, int, int]]
    window_ctx: Dict[int, List[Tuple[int, int]]]
    global_frame_mask: torch.Tensor
    window_bounds: torch.Tensor
    attended_indices: torch.Tensor
    attended_C: int
    global_src_idx: torch.Tensor
    global_dst_idx: torch.Tensor
    local_src_idx: torch.Tensor
    local_dst_idx: torch.Tensor
    fi_indptr: torch.Tensor
    fi_indices: torch.Tensor
    fi_M: int
    fi_N: int
    fi_MB: int
    fi_compact_n: int
    fi_global_copies: List[Tuple[int, int]]
    fi_local_copies: List[Tuple[int, int]]
    keyframe_offset: int = 0
    boundary_guards: List[int] = field(default_factory=list)
    _block_masks: Dict[Any, BlockMask] = field(default_factory=dict, repr=False)

    @classmethod
    @torch.compiler.disable
    def build(cls, total_latent_frames: int, num_patches: int, window_size: int,
              n_first_frames: int, key_frame_interval: Optional[int], rank: int, world: int,
              expand_window: bool = True, keyframe_offset: int = 0,
              boundary_guards: Optional[List[int]] = None, reference_frames: int = 21,
              sparsity_scale: float = 1.0) -> "LVSAMetadata":
        T, P, W = total_latent_frames, num_patches, window_size
        total = T * P
        assert total % world == 0, (
            f"total_seq={total} (T={T} x P={P}) must be divisible by world={world}.")
        local = total // world
        gts = rank * local
        guards = list(boundary_guards or [])
        gidx = sorted(set(compute_global_indices(T, n_first_frames, key_frame_interval,
                                                 keyframe_offset)) | set(guards))
        gset = set(gidx)
        first, last = gts // P, (gts + local - 1) // P
        lo_hi = [get_window_bounds(f, W, T, expand_window, gset, len(gidx)) for f in range(T)]

        local_frames = [(f, max(f * P, gts) - gts, min((f + 1) * P, gts + local) - gts)
                        for f in range(first, last + 1)]

        def owned(wf):  # the part of frame wf inside this rank's token range
            s, e = max(wf * P, gts), min((wf + 1) * P, gts + local)
            return (s, e) if s < e else None

        window_ctx: Dict[int, List[Tuple[int, int]]] = {}
        for f, _, _ in local_frames:
            lo, hi = lo_hi[f]
            parts = []
            for wf in range(lo, hi + 1):
                if wf in gset:
                    continue
                o = owned(wf)
                if o:
                    parts.append((o[0] - gts, o[1] - gts))
            window_ctx[f] = parts

        gmask = torch.zeros(T, dtype=torch.int8)
        if gidx:
            gmask[torch.tensor(gidx)] = 1
        bounds = torch.tensor(lo_hi, dtype=torch.int32).reshape(T, 2)

        ar = torch.arange(P, dtype=torch.long)
        g_t = torch.tensor(gidx, dtype=torch.long)
        global_src = (torch.arange(len(gidx))[:, None] * P + ar[None, :]).reshape(-1)
        global_dst = (g_t[:, None] * P + ar[None, :]).reshape(-1)
        lsrc, ldst = [], []
        for f in range(first, last + 1):
            if f in gset:
                continue
            o = owned(f)
            if o:
                lsrc.append(torch.arange(o[0] - gts, o[1] - gts))
                ldst.append(torch.arange(o[0], o[1]))
        local_src = torch.cat(lsrc) if lsrc else torch.empty(0, dtype=torch.long)
        local_dst = torch.cat(ldst) if ldst else torch.empty(0, dtype=torch.long)

        # [T_local, C] attended frames, padded with each row's last entry
        rows = []
        for f in range(first, last + 1):
            lo, hi = lo_hi[f]
            rows.append(sorted(gset | set(range(lo, hi + 1))))
        C = max(len(r) for r in rows)
        att = torch.tensor([r + [r[-1]] * (C - len(r)) for r in rows], dtype=torch.int32)

        # frame-level CSR over the compacted attended frames
        MB = -(-local // P)
        per_q = []
        for qi in range(MB):
            lo, hi = lo_hi[first + qi]
            s = set(gidx)
            s.update(wf for wf in range(lo, hi + 1) if wf not in gset and owned(wf))
            per_q.append(s)
        compact = sorted(set().union(*per_q))
        to_c = {f: i for i, f in enumerate(compact)}
        indptr, indices = [0], []
        for s in per_q:
            indices.extend(sorted(to_c[f] for f in s))
            indptr.append(len(indices))
        gpos = {g: i for i, g in enumerate(gidx)}
        gcopies, lcopies = [], []
        for ci, f in enumerate(compact):
            (gcopies.append((gpos[f] * P, ci * P)) if f in gset else lcopies.append((f * P - gts, ci * P)))
        fi_indptr = torch.tensor(indptr, dtype=torch.int32)
        fi_indices = torch.tensor(indices, dtype=torch.int32)
        assert fi_indptr[0] == 0, "CSR indptr must start at 0"
        assert len(fi_indptr) == MB + 1, f"CSR indptr length {len(fi_indptr)} != MB+1={MB + 1}"
        assert len(fi_indices) == int(fi_indptr[-1]), "CSR indices length != nnz"
        if compact:
            assert int(fi_indices.max()) < len(compact), "CSR index >= compact_n"
        assert len(gcopies) + len(lcopies) == len(compact), "copy instructions != compact_n"

        return cls(
            total_latent_frames=T, num_patches=P, window_size=W, n_first_frames=n_first_frames,
            key_frame_interval=key_frame_interval, expand_window=expand_window, rank=rank,
            world=world, local_seq=local, global_token_start=gts, global_indices=gidx,
            global_set=gset, local_frames=local_frames, window_ctx=window_ctx,
            global_frame_mask=gmask, window_bounds=bounds, attended_indices=att, attended_C=C,
            global_src_idx=global_src, global_dst_idx=global_dst, local_src_idx=local_src,
            local_dst_idx=local_dst, fi_indptr=fi_indptr, fi_indices=fi_indices,
            fi_M=MB * P, fi_N=len(compact) * P, fi_MB=MB, fi_compact_n=len(compact),
            fi_global_copies=gcopies, fi_local_copies=lcopies,
            keyframe_offset=keyframe_offset, boundary_guards=guards)

    def ensure_device(self, device: torch.device) -> None:
        """Move the tensor fields (not the frame CSR) to ``device``
        (lvsa/sparse_attention.py:486-504)."""
        for name in ("global_frame_mask", "window_bounds", "attended_indices", "global_src_idx",
                     "global_dst_idx", "local_src_idx", "local_dst_idx"):
            t = getattr(self, name)
            if t.device != device:
                object.__setattr__(self, name, t.to(device))

    def attended_frames(self, f: int) -> List[int]:
        lo, hi = (int(x) for x in self.window_bounds[f].tolist())
        return sorted(self.global_set | set(range(lo, hi + 1)))

    def block_mask(self, device: torch.device, n_text: int = 0, block_q: int = ATTN_BLOCK_Q,
                   block_k: int = ATTN_BLOCK_K) -> BlockMask:
        """GPU tile CSR of this pattern (world = 1 semantics), cached per device."""
        device = torch.device(device)
        key = (str(device), int(n_text), block_q, block_k)
        m = self._block_masks.get(key)
        if m is None:
            m = build_block_mask(self.total_latent_frames, self.num_patches, self.window_size,
                                 self.n_first_frames, self.key_frame_interval, self.keyframe_offset,
                                 self.expand_window, n_text, block_q, block_k,
                                 self.boundary_guards or None, device=device)
            self._block_masks[key] = m
        return m


def tile_flop_counts(meta: LVSAMetadata, n_text: int, heads: int, head_dim: int,
                     block_q: int = 128, block_k: int = 128) -> Tuple[int, int]:
    """(FLOP_tiles, FLOP_exact) of one layer: 4*D*H per attended (query, key)
    pair; video x video counted over active tiles at their clipped area,
    text terms exact."""
    T, P = meta.total_latent_frames, meta.num_patches
    Nv = T * P
    att = [meta.attended_frames(f) for f in range(T)]
    area = 0
    for qb in range(-(-Nv // block_q)):
        t0, t1 = qb * block_q, min(Nv, (qb + 1) * block_q)
        frames = set().union(*(att[f] for f in range(t0 // P, (t1 - 1) // P + 1)))
        tiles = set()
        for f in frames:
            tiles.update(range(f * P // block_k, (min(Nv, (f + 1) * P) - 1) // block_k + 1))
        area += (t1 - t0) * sum(min(Nv, (kb + 1) * block_k) - kb * block_k for kb in tiles)
    text = Nv * n_text + n_text * (Nv + n_text)
    exact = sum(P * P * len(a) for a in att)
    c = 4 * head_dim * heads
    return c * (area + text), c * (exact + text)


# --------------------------------------------------------------------------
# Attention entry points
# --------------------------------------------------------------------------


# Masks of metadata objects that carry no GPU mask of their own (the
# reference's LVSAMetadata), keyed by the pattern they describe.
_FOREIGN_MASKS: "OrderedDict[tuple, Any]" = OrderedDict()
_FOREIGN_CAP = 32


def pattern_key(metadata: Any) -> tuple:
    """The pattern an LVSAMetadata (this package's or the reference's,
    lvsa/sparse_attention.py:286-353) describes, from fields both carry:
    geometry, shard, and the global frame list.  The reference object stores
    neither the keyframe interval nor the offset, but its global_indices
    (keyframes, anchors and boundary guards) and W / expand_window determine
    every window bound (lvsa/sparse_attention.py:52-104), hence the whole
    pattern."""
    return (int(metadata.total_latent_frames), int(metadata.num_patches), int(metadata.window_size),
            bool(metadata.expand_window), tuple(int(g) for g in metadata.global_indices),
            int(metadata.rank), int(metadata.world))


def _cached(key: tuple, make):
    m = _FOREIGN_MASKS.get(key)
    if m is None:
        m = make()
        _FOREIGN_MASKS[key] = m
        while len(_FOREIGN_MASKS) > _FOREIGN_CAP:
            _FOREIGN_MASKS.popitem(last=False)
    else:
        _FOREIGN_MASKS.move_to_end(key)
    return m


def mask_for(metadata: Any, device: torch.device, n_text: int = 0) -> BlockMask:
    """World = 1 GPU mask for any LVSAMetadata: this package's (its own
    cache) or a foreign one such as the reference's, rebuilt on the GPU from
    ``pattern_key`` with the global frames passed as explicit globals (no
    anchors, no keyframe grid) and cached by pattern."""
    if isinstance(metadata, LVSAMetadata):
        return metadata.block_mask(device, n_text)
    T, P, W, expand, gidx, _, world = pattern_key(metadata)
    if world != 1:
        raise ValueError("mask_for: world = 1 metadata expected (shards go through shard_pattern_for)")
    device = torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return _cached(pattern_key(metadata) + ("mask", str(device), int(n_text)),
                   lambda: build_block_mask(T, P, W, 0, None, 0, expand, n_text,
                                            boundary_guards=list(gidx), device=device))


def shard_pattern_for(metadata: Any, device: torch.device, n_text: int = 0):
    """Sequence-shard (world > 1) launch pattern of a rank's metadata: the
    reference's own context-parallel semantics (``cp_mode``), with the
    metadata's global frames (keyframes + boundary guards) taken as given."""
    from .cp_mode import build_shard_pattern
    T, P, W, expand, gidx, rank, world = pattern_key(metadata)
    device = torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return _cached(pattern_key(metadata) + ("shard", str(device), int(n_text)),
                   lambda: build_shard_pattern(T, P, W, 0, None, 0, rank, world, n_text, expand,
                                               device=device, global_indices=list(gidx)))


def _text_part(k_global: Optional[torch.Tensor], metadata: LVSAMetadata) -> int:
    if k_global is None:
        return 0
    n = int(k_global.shape[1]) - len(metadata.global_indices) * metadata.num_patches
    if n < 0:
        raise AssertionError(
            f"k_global holds {k_global.shape[1]} tokens, fewer than the "
            f"{len(metadata.global_indices)} global frames x {metadata.num_patches} patches")
    return n


@torch.compiler.disable
def lvsa_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   metadata: LVSAMetadata, text_query: Optional[torch.Tensor] = None,
                   text_key: Optional[torch.Tensor] = None, text_value: Optional[torch.Tensor] = None,
                   scale: Optional[float] = None, return_lse: bool = False):
    """Video rows (sparse, plus all text) and optional text rows (dense) of one
    layer in a single kernel launch.  Full-sequence (world = 1) tensors;
    ``metadata`` is this package's LVSAMetadata or the reference's."""
    if metadata.world != 1:
        raise NotImplementedError(
            "lvsa_attention takes the full sequence; for context parallelism use "
            "longvideosparseattention_b200.ulysses (head-parallel all-to-all) or lvsa_sdpa with "
            "the rank's metadata and its gathered global K/V")
    nt = 0 if text_key is None else int(text_key.shape[1])
    mask = mask_for(metadata, query.device, nt)
    return block_sparse_attention(query, key, value, mask, text_query, text_key, text_value,
                                  scale=scale, return_lse=return_lse)


@torch.compiler.disable
def lvsa_sdpa(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, k_global: torch.Tensor,
              v_global: torch.Tensor, metadata: LVSAMetadata, attention_backend: Any = None) -> torch.Tensor:
    """Drop-in for lvsa_sdpa (lvsa/sparse_attention.py:643-706).

    ``metadata`` is this package's LVSAMetadata or the reference's own
    object (read through ``pattern_key``; its GPU mask is cached by pattern).
    query/key/value [B, S, H(kv), D]; k_global/v_global the gathered anchor
    K/V with any text K/V appended after them, as the processor builds them
    (lvsa/lvsa_processor.py:545-549).  At world = 1 the anchor K/V are read
    in place from ``key``/``value`` (identical there) and only the appended
    text part of k_global/v_global is used.  For a rank's shard (world > 1)
    the query, key and value are the local shard and k_global/v_global the
    all-reduced [globals; text] buffer, as in the reference: the video rows
    run as the video launch of the reference's context-parallel pattern.
    ``attention_backend`` is accepted and ignored.
    """
    if metadata.world > 1:
        nt = _text_part(k_global, metadata)
        pat = shard_pattern_for(metadata, query.device, nt)
        out, _ = block_sparse_attention(query, key, value, pat.video, None, k_global, v_global)
        return out
    nt = _text_part(k_global, metadata)
    tk = k_global[:, k_global.shape[1] - nt:] if nt else None
    tv = v_global[:, v_global.shape[1] - nt:] if nt else None
    out, _ = lvsa_attention(query, key, value, metadata, None, tk, tv)
    return out


def lvsa_flashinfer(query_padded: torch.Tensor, k_compact: torch.Tensor, v_compact: torch.Tensor,
                    fi_wrapper: Any, local_seq: int, fi_M: int) -> torch.Tensor:
    """Drop-in for lvsa_flashinfer (lvsa/sparse_attention.py:709-742).

    ``fi_wrapper`` is a planned ``bsr.LvsaBlockSparseWrapper`` (same plan
    arguments as the reference's flashinfer.BlockSparseAttentionWrapper:
    the frame CSR fi_indptr / fi_indices, M = fi_M, N = compact_n x P,
    R = C = P) or any object with that ``run(q, k, v)``.
    query_padded [B, M, H, D], k_compact / v_compact [B, compact_N, Hkv, D];
    returns [B, local_seq, H, D]."""
    from .bsr import LvsaBlockSparseWrapper
    if isinstance(fi_wrapper, LvsaBlockSparseWrapper):
        out = fi_wrapper.run(query_padded, k_compact, v_compact)       # one launch for the batch
    else:
        out = query_padded.new_empty(query_padded.shape[0], fi_M, *query_padded.shape[2:])
        for b in range(query_padded.shape[0]):
            out[b] = fi_wrapper.run(query_padded[b], k_compact[b], v_compact[b])
    return out[:, :local_seq]


def sparse_windowed_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                              k_global: torch.Tensor, v_global: torch.Tensor,
                              metadata: LVSAMetadata, backend: str = "sdpa", *,
                              k_compact: Optional[torch.Tensor] = None,
                              v_compact: Optional[torch.Tensor] = None, fi_wrapper: Optional[Any] = None,
                              attention_backend: Any = None) -> torch.Tensor:
    """Drop-in for the dispatcher (lvsa/sparse_attention.py:750-788).  Both
    backend names run the same kernel; "flashinfer" keeps the reference's
    argument assertion so callers fail the same way."""
    if backend == "flashinfer":
        assert k_compact is not None and v_compact is not None and fi_wrapper is not None, (
            "FlashInfer backend requires k_compact, v_compact, and fi_wrapper")
    return lvsa_sdpa(query, key, value, k_global, v_global, metadata, attention_backend)
