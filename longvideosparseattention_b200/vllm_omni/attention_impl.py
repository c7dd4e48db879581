"""``LVSAAttentionImpl`` (interface of lvsa-vllm-omni/lvsa_vllm_omni/attention_impl.py:247-532).

``forward_cuda(q, k, v)`` receives the joint ``[video; text]`` sequence of a
layer.  It detects the frame geometry from the sequence length
(``seq_len = T_lat * P + text``), reads the step's pattern (rebuilt on the
GPU when T/P change or keyframes rotate), and runs the video rows (sparse, plus all text) and the
text rows (dense) in ONE launch of the sm_100a kernel.  Cross-attention and
non-frame sequences use the model's dense attention, as the reference does.
"""

from typing import Any, Optional

import torch
import torch.nn.functional as F

from ..block_sparse import block_sparse_attention
from ..sparse_attention import LVSAMetadata, compute_auto_kfi
from ..step_mask import SHARED
from . import step_tracker
from ._fallback import warn_fallback
from .config import LVSAConfig, candidate_patches_per_frame


def _reset_step_counter() -> None:
    """Called by ``step_tracker.reset()``: drop the shared call counter so a
    calibration does not carry over between generations."""
    step_tracker._global_tracker = None


class LVSAAttentionImpl:
    _total_instances = 0
    # Set by the block-level hooks: they run the sparse path themselves, so
    # the backend's own forward keeps to dense attention.
    _hook_active = False

    def __init__(self, num_heads: int, head_size: int, softmax_scale: float, causal: bool = False,
                 num_kv_heads: Optional[int] = None, prefix: str = "", qkv_layout: Optional[str] = None,
                 backend_kwargs: Optional[dict] = None, **extra_impl_args: Any) -> None:
        self.num_heads = num_heads
        self.head_size = head_size
        self.softmax_scale = softmax_scale
        self.num_kv_heads = num_kv_heads or num_heads
        self.qkv_layout = qkv_layout
        self.backend_kwargs = backend_kwargs or {}
        self.config = LVSAConfig.from_env()
        self._meta: Optional[LVSAMetadata] = None
        self._key = None
        LVSAAttentionImpl._total_instances += 1

    def forward(self, query, key, value, attn_metadata: Any = None):
        return self.forward_cuda(query, key, value, attn_metadata)

    def _dense_attention(self, query, key, value):
        out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2), value.transpose(1, 2),
                                             scale=self.softmax_scale,
                                             enable_gqa=key.shape[2] != query.shape[2])
        return out.transpose(1, 2)

    def _total_frames(self) -> Optional[int]:
        return self.config.total_latent_frames

    @staticmethod
    def detect_geometry(seq_len: int, total_frames: int):
        """(P, text_tokens) with 0 <= text < T*P, or (None, None)."""
        for p in candidate_patches_per_frame():
            video = total_frames * p
            text = seq_len - video
            if 0 <= text < video:
                return p, text
        return None, None

    def _mask(self, T: int, P: int, text: int, device: torch.device):
        """The step's GPU mask, one per pattern for all instances
        (``step_mask.SHARED``; rebuilt in place once per rotation, no host
        metadata build)."""
        cfg = self.config
        W, nf = cfg.latent_window_size, cfg.latent_n_first_frames
        kfi = cfg.latent_key_frame_interval
        if cfg.auto_keyframes:
            kfi = compute_auto_kfi(T, W, nf, cfg.reference_latent_frames, cfg.sparsity_scale)
        return SHARED.get(device, T, P, W, nf, kfi, cfg.expand_window, text, step_tracker.get_step(),
                          rotate=cfg.rotate_keyframes)

    def _metadata(self, T: int, P: int) -> LVSAMetadata:
        """Host LVSAMetadata of the current step (reference interface; the
        forward path uses ``_mask``)."""
        cfg = self.config
        W, nf = cfg.latent_window_size, cfg.latent_n_first_frames
        kfi = cfg.latent_key_frame_interval
        if cfg.auto_keyframes:
            kfi = compute_auto_kfi(T, W, nf, cfg.reference_latent_frames, cfg.sparsity_scale)
        off = step_tracker.get_step() % kfi if (cfg.rotate_keyframes and kfi > 0) else 0
        key = (T, P, W, nf, kfi, off)
        if self._meta is None or self._key != key:
            self._meta = LVSAMetadata.build(T, P, W, nf, kfi, 0, 1, expand_window=cfg.expand_window,
                                            keyframe_offset=off,
                                            reference_frames=cfg.reference_latent_frames,
                                            sparsity_scale=cfg.sparsity_scale)
            self._key = key
        return self._meta

    @torch.compiler.disable
    def forward_cuda(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                     attn_metadata: Any = None) -> torch.Tensor:
        if LVSAAttentionImpl._hook_active:
            return self._dense_attention(query, key, value)
        if query.shape[1] != key.shape[1]:
            return self._dense_attention(query, key, value)  # cross-attention
        T = self._total_frames()
        if T is None:
            warn_fallback("forward_cuda", "no_t_lat", query.shape[1])
            return self._dense_attention(query, key, value)
        P, text = self.detect_geometry(query.shape[1], T)
        if P is None:
            warn_fallback("forward_cuda", "geometry_detect", query.shape[1], {"T_lat": T})
            return self._dense_attention(query, key, value)
        mask = self._mask(T, P, text, query.device)
        nv = T * P
        tq = query[:, nv:] if text else None
        tk = key[:, nv:] if text else None
        tv = value[:, nv:] if text else None
        out = torch.empty_like(query)
        o_v = out[:, :nv]
        o_t = out[:, nv:] if text else None
        block_sparse_attention(query[:, :nv], key[:, :nv], value[:, :nv], mask, tq, tk, tv,
                               scale=self.softmax_scale, out=o_v, text_out=o_t)
        return out
