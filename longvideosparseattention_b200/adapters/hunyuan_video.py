"""HunyuanVideo-1.5 adapter (interface of lvsa/adapters/hunyuan_video.py:31-333).

Dual-stream joint attention: video tokens use ``to_q/to_k/to_v`` + per-head
RMSNorm ``norm_q/norm_k`` + 3-D RoPE (``image_rotary_emb``); text tokens use
``add_q_proj/add_k_proj/add_v_proj`` + ``norm_added_q/norm_added_k`` and no
RoPE; outputs go through ``to_out`` (video) and ``to_add_out`` (text) and the
block receives ``(video, text)``.
"""

from typing import Any

from .dual_stream import DualStreamAdapter


class HunyuanVideoAdapter(DualStreamAdapter):
    def patches_per_frame(self, height: int, width: int, pipe: Any) -> int:
        ps = getattr(pipe.transformer.config, "patch_size", 2)
        ps = int(ps[1]) if isinstance(ps, (list, tuple)) else int(ps)
        s = getattr(pipe, "vae_scale_factor_spatial", 16)
        return (height // (s * ps)) * (width // (s * ps))

    def latent_frames(self, num_frames: int, pipe: Any) -> int:
        return (num_frames - 1) // getattr(pipe, "vae_scale_factor_temporal", 4) + 1

    def reference_latent_frames(self, pipe: Any) -> int:
        n = getattr(pipe.transformer.config, "sample_n_frames", None)
        return self.latent_frames(n, pipe) if n is not None else 33  # 129 raw frames

    def extract_encoder_qkv(self, attn, encoder_hidden_states):
        if getattr(attn, "add_q_proj", None) is None or encoder_hidden_states is None:
            return None
        q = self._split_heads(attn, attn.add_q_proj(encoder_hidden_states))
        k = self._split_heads(attn, attn.add_k_proj(encoder_hidden_states))
        v = self._split_heads(attn, attn.add_v_proj(encoder_hidden_states))
        return (self._norm(getattr(attn, "norm_added_q", None), q),
                self._norm(getattr(attn, "norm_added_k", None), k), v)

    def format_output(self, attn, hidden_states, encoder_output, encoder_seq_len, query_dtype):
        if encoder_output is None or encoder_seq_len <= 0:
            return hidden_states
        enc = encoder_output.flatten(2, 3).to(query_dtype)
        if getattr(attn, "to_add_out", None) is not None:
            enc = attn.to_add_out(enc)
        return hidden_states, enc

    def install_processor(self, pipe: Any, processor: Any) -> int:
        blocks = pipe.transformer.transformer_blocks
        for blk in blocks:
            blk.attn.processor = processor
        return len(blocks)
