"""CogVideoX adapter (interface of lvsa/adapters/cogvideox.py:37-348).

Joint attention with shared weights: text and video tokens both go through
``to_q/to_k/to_v`` and per-head LayerNorm ``norm_q/norm_k`` (projection and
norm commute with concatenation, so the text stream is projected separately
and handed to the processor as encoder Q/K/V); RoPE only on video tokens; one
``to_out`` for both streams; the block receives ``(video, text)``.
"""

from typing import Any

from .dual_stream import DualStreamAdapter


class CogVideoXAdapter(DualStreamAdapter):
    def patches_per_frame(self, height: int, width: int, pipe: Any) -> int:
        ps = getattr(pipe.transformer.config, "patch_size", 2)
        ps = int(ps[-1]) if isinstance(ps, (list, tuple)) else int(ps)
        s = getattr(pipe, "vae_scale_factor_spatial", 8)
        return (height // (s * ps)) * (width // (s * ps))

    def latent_frames(self, num_frames: int, pipe: Any) -> int:
        t = (num_frames - 1) // getattr(pipe, "vae_scale_factor_temporal", 4) + 1
        pt = getattr(pipe.transformer.config, "patch_size_t", None)
        if pt is not None and pt > 1:
            t = -(-t // pt)  # CogVideoX-1.5: temporal patches
        return t

    def reference_latent_frames(self, pipe: Any) -> int:
        n = getattr(pipe.transformer.config, "sample_frames", None)
        return self.latent_frames(n, pipe) if n is not None else 13  # 49 raw frames

    def extract_encoder_qkv(self, attn, encoder_hidden_states):
        if encoder_hidden_states is None:
            return None
        q, k, v = self._video_projections(attn, encoder_hidden_states)  # shared weights
        return self._norm(getattr(attn, "norm_q", None), q), self._norm(getattr(attn, "norm_k", None), k), v

    def format_output(self, attn, hidden_states, encoder_output, encoder_seq_len, query_dtype):
        if encoder_output is None or encoder_seq_len <= 0:
            return hidden_states
        return hidden_states, self.output_projection(attn, encoder_output, query_dtype)

    def install_processor(self, pipe: Any, processor: Any) -> int:
        blocks = pipe.transformer.transformer_blocks
        for blk in blocks:
            blk.attn1.processor = processor
        return len(blocks)
