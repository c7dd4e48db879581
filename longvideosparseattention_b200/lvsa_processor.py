"""Drop-in for ``DistributedLVSAProcessor`` (lvsa/lvsa_processor.py:68-917).

Same constructor, attributes, per-step controls (``set_step``,
``set_window_size``, ``set_sparsity_scale``) and ``__call__`` contract as the
reference processor; the attention itself is one launch of the sm_100a
block-sparse kernel that computes both the sparse video rows (with every text
token attended) and the dense encoder/text rows, so the reference's global-KV
gather, K/V concatenation, FlashInfer plan / compact copy / LSE merge and the
separate dense encoder SDPA all disappear.

Multi-GPU: with ``world > 1`` the processor expects sequence-sharded hidden
states (as the reference).  ``cp_mode="ulysses"`` (default) runs Ulysses head
parallelism (``ulysses.ulysses_attention``) with the world = 1 pattern on
every rank; ``cp_mode="reference"`` reproduces the reference's own world > 1
pattern (boundary-guard anchors gathered by one all-reduce, rank-local
windows, ``cp_mode.cp_attention``).
"""

from __future__ import annotations

from typing import Any, List, Optional, Tuple

import torch
import torch.nn.functional as F

from .adapters.base import ModelAdapter
from .block_sparse import block_sparse_attention
from .sparse_attention import (LVSAMetadata, compute_auto_kfi, compute_boundary_guard_frames,
                               get_window_bounds, print_attention_mask_compact)


class DistributedLVSAProcessor:
    """Block-sparse LVSA attention processor (one instance shared by all blocks)."""

    _attention_backend = None
    _parallel_config = None

    def __init__(self, total_num_latent_frames: int, num_patches: int, window_size: int,
                 n_first_frames: int, key_frame_interval: Optional[int], rank: int, world: int,
                 expand_window: bool = True, adapter: Optional[ModelAdapter] = None,
                 sparsity_scale: float = 1.0, reference_frames: int = 21, cp_mode: str = "ulysses") -> None:
        if cp_mode not in ("ulysses", "reference"):
            raise ValueError(f"cp_mode must be 'ulysses' or 'reference', got {cp_mode!r}")
        self.cp_mode = cp_mode
        self._shard = None  # reference-mode shard pattern (per step, built lazily on the device)
        self._global_kv = None
        self.total_num_frames = total_num_latent_frames
        self.num_patches = num_patches
        self.window_size = window_size
        self.n_first_frames = n_first_frames
        self.rank = rank
        self.world = world
        self._expand_window = expand_window
        self._sparsity_scale = sparsity_scale
        self._reference_frames = reference_frames
        if adapter is None:
            from .adapters.wan import WanAdapter
            adapter = WanAdapter()
        self.adapter = adapter
        # lvsa/lvsa_processor.py:131-137.  cp_mode="reference" makes them
        # anchors (build_shard_pattern derives the same list); the Ulysses
        # path uses the world = 1 pattern, where they are not anchors.
        self._boundary_guards: List[int] = compute_boundary_guard_frames(
            total_num_latent_frames, total_num_latent_frames * num_patches // world,
            num_patches, world, window_size)
        self.key_frame_interval = key_frame_interval
        self._current_offset = 0
        assert (total_num_latent_frames * num_patches) % world == 0, (
            f"total_seq={total_num_latent_frames * num_patches} must be divisible by world={world}.")
        self._build(0)
        self._geometry_warned = False

    # ------------------------------------------------------------------ state
    def _build(self, offset: int) -> None:
        self._current_offset = offset
        self._metadata = LVSAMetadata.build(
            self.total_num_frames, self.num_patches, self.window_size, self.n_first_frames,
            self.key_frame_interval, 0, 1, expand_window=self._expand_window,
            keyframe_offset=offset, reference_frames=self._reference_frames,
            sparsity_scale=self._sparsity_scale)
        m = self._metadata
        self.local_seq = m.local_seq // self.world
        self.global_token_start = self.rank * self.local_seq
        self._global_indices = m.global_indices
        self._global_set = m.global_set
        self._window_bounds = m.window_bounds
        self._global_frame_mask = m.global_frame_mask
        self._attended_indices = m.attended_indices
        self._attended_C = m.attended_C
        self._fi_indptr = m.fi_indptr
        self._fi_indices = m.fi_indices
        self._fi_MB = m.fi_MB
        self._fi_compact_n = m.fi_compact_n
        self._block_mask = None  # GPU tile CSR, rebuilt lazily (reusing its buffers)
        self._shard = None

    def _rebuild_for_current_params(self, offset: int) -> None:
        """Recompute the pattern for the current window / kfi / offset
        (lvsa/lvsa_processor.py:362-405)."""
        old = self._block_mask
        self._build(offset)
        self._stale_mask = old

    def set_step(self, step_idx: int) -> None:
        """Rotate keyframes: offset = step % kfi (lvsa/lvsa_processor.py:317-331)."""
        if not self.key_frame_interval:
            return
        offset = step_idx % self.key_frame_interval
        if offset == self._current_offset:
            return
        self._rebuild_for_current_params(offset)

    def set_window_size(self, new_window_size: int) -> None:
        """Switch window size; kfi is re-derived for the budget (:288-315)."""
        if new_window_size == self.window_size:
            return
        self.window_size = new_window_size
        self.key_frame_interval = compute_auto_kfi(self.total_num_frames, self.window_size,
                                                   self.n_first_frames, self._reference_frames,
                                                   self._sparsity_scale)
        self._rebuild_for_current_params(self._current_offset)

    def set_sparsity_scale(self, new_sparsity_scale: float) -> None:
        """Change the attended-frame budget; kfi re-derived (:333-360)."""
        if new_sparsity_scale == self._sparsity_scale:
            return
        self._sparsity_scale = new_sparsity_scale
        self.key_frame_interval = compute_auto_kfi(self.total_num_frames, self.window_size,
                                                   self.n_first_frames, self._reference_frames,
                                                   self._sparsity_scale)
        self._rebuild_for_current_params(self._current_offset)

    def _get_window_bounds(self, f: int, W: int, T: int) -> Tuple[int, int]:
        return get_window_bounds(f, W, T, self._expand_window, self._global_set, len(self._global_indices))

    def _geometry_matches(self, local_seq: int) -> bool:
        """local_seq x world must equal T x P (lvsa/lvsa_processor.py:611-619)."""
        return self.num_patches > 0 and local_seq * self.world == self.total_num_frames * self.num_patches

    def print_attention_mask_compact(self) -> None:
        print_attention_mask_compact(self.total_num_frames, self.window_size, self._global_set,
                                     self._expand_window)

    def block_mask(self, device: torch.device, n_text: int):
        """GPU tile CSR of the current step (rebuilt into the previous buffers)."""
        bm = self._block_mask
        if bm is None or bm.device != torch.device(device) or bm.n_text != n_text:
            from .block_sparse import build_block_mask
            m = self._metadata
            reuse = getattr(self, "_stale_mask", None) or bm
            bm = build_block_mask(m.total_latent_frames, m.num_patches, m.window_size, m.n_first_frames,
                                  m.key_frame_interval, m.keyframe_offset, m.expand_window, n_text,
                                  device=device, reuse=reuse)
            self._block_mask, self._stale_mask = bm, None
        return bm

    # --------------------------------------------------------------- forward
    def _attend(self, query, key, value, enc_q, enc_k, enc_v):
        if self.world > 1 and self.cp_mode == "reference":
            from .cp_mode import GlobalKV, build_shard_pattern, cp_attention
            nt = 0 if enc_k is None else int(enc_k.shape[1])
            m = self._metadata
            if self._shard is None or self._shard.n_text != nt or self._shard.video.tile_indptr.device != query.device:
                self._shard = build_shard_pattern(m.total_latent_frames, m.num_patches, m.window_size,
                                                  m.n_first_frames, m.key_frame_interval, m.keyframe_offset,
                                                  self.rank, self.world, nt, m.expand_window, device=query.device)
            if self._global_kv is None:
                self._global_kv = GlobalKV()
            return cp_attention(query, key, value, self._shard, self._global_kv, enc_q, enc_k, enc_v)
        if self.world == 1:
            nt = 0 if enc_k is None else int(enc_k.shape[1])
            return block_sparse_attention(query, key, value, self.block_mask(query.device, nt),
                                          enc_q, enc_k, enc_v)
        from .ulysses import shard_sizes, tile_costs, ulysses_attention
        nt = 0 if enc_k is None else int(enc_k.shape[1])
        mask = self.block_mask(query.device, nt)

        def local(q, k, v, tq, tk, tv, q_tiles, out, text_out):
            block_sparse_attention(q, k, v, mask, tq, tk, tv, out=out, text_out=text_out, q_tiles=q_tiles)
        costs = None
        if query.shape[2] % self.world:
            # Head count not divisible by the GPU count: balance (head, tile row)
            # units by each row's key-tile count, read once per pattern.
            ck = (self._metadata.keyframe_offset, nt, query.device)
            if getattr(self, "_costs_key", None) != ck:
                self._costs, self._costs_key = tile_costs(mask), ck
            costs = self._costs
        sizes = shard_sizes(self.total_num_frames * self.num_patches, self.world)
        return ulysses_attention(query, key, value, sizes, local, enc_q, enc_k, enc_v,
                                 n_q_tiles=mask.n_q_tiles, costs=costs)

    @staticmethod
    def _dense(query, key, value):
        out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2),
                                             value.transpose(1, 2))
        return out.transpose(1, 2)

    def __call__(self, attn: Any, hidden_states: torch.Tensor,
                 encoder_hidden_states: Optional[torch.Tensor] = None,
                 attention_mask: Optional[torch.Tensor] = None, rotary_emb: Optional[Any] = None,
                 image_rotary_emb: Optional[Any] = None, **kwargs) -> Any:
        adapter = self.adapter
        if rotary_emb is None and image_rotary_emb is not None:
            rotary_emb = image_rotary_emb
        encoder_img = None
        if encoder_hidden_states is not None:
            encoder_hidden_states, encoder_img = adapter.split_encoder_for_cross_attn(attn, encoder_hidden_states)
        local_seq = hidden_states.shape[1]
        # Projections, QK norm and rotary embedding (fused into one pass per
        # tensor by the adapter where the prologue kernel applies).
        query, key, value = adapter.project_qkv(attn, hidden_states, encoder_hidden_states, rotary_emb,
                                                local_seq, self.rank, self.world)
        query_dtype = query.dtype
        enc_q = enc_k = enc_v = None
        enc_len = 0
        if encoder_hidden_states is not None:
            enc = adapter.extract_encoder_qkv(attn, encoder_hidden_states)
            if enc is not None:
                enc_q, enc_k, enc_v = enc
                enc_len = enc_q.shape[1]

        enc_out = None
        if self._geometry_matches(local_seq):
            out, enc_out = self._attend(query, key, value, enc_q, enc_k, enc_v)
        else:
            # Not a frame grid: the model's own dense attention (lvsa/lvsa_processor.py:554-582).
            if self.world > 1:
                raise NotImplementedError(
                    f"LVSA dense fallback under context parallelism is unsupported "
                    f"(geometry mismatch: local_seq={local_seq}, world={self.world}).")
            if not self._geometry_warned:
                self._geometry_warned = True
                if self.rank == 0:
                    print(f"[LVSA] WARNING geometry mismatch: runtime seq={local_seq} != "
                          f"T_lat*P={self.total_num_frames * self.num_patches}; using dense attention.",
                          flush=True)
            if enc_k is not None:
                out = self._dense(query, torch.cat([key, enc_k], 1), torch.cat([value, enc_v], 1))
                enc_out = self._dense(enc_q, torch.cat([key, enc_k], 1), torch.cat([value, enc_v], 1))
            else:
                out = self._dense(query, key, value)

        # Extra image-context cross-attention is added before the output
        # projection (lvsa/lvsa_processor.py:593-601).
        cross = adapter.cross_attention(attn, query, encoder_img, self._attention_backend)
        if cross is not None:
            out = out + cross.unflatten(2, (out.shape[2], -1)).to(out.dtype)
        hs = adapter.output_projection(attn, out, query_dtype)
        if enc_out is not None:
            return adapter.format_output(attn, hs, enc_out, enc_len, query_dtype)
        return hs


# Backwards-compatible alias (lvsa/lvsa_processor.py:916-917).
WanDistributedLVSAProcessor = DistributedLVSAProcessor
