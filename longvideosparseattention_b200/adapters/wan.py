"""Wan 2.x adapter (interface of lvsa/adapters/wan.py:17-222).

Works on any attention module exposing the diffusers Wan attention fields:
``to_q/to_k/to_v`` (or a fused ``to_qkv``), ``norm_q/norm_k``, ``heads``,
``to_out`` (Linear, Dropout), and for image-to-video ``add_k_proj``,
``add_v_proj``, ``norm_added_k``.  diffusers itself is not required.
"""

from typing import Any, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from .base import ModelAdapter

IMAGE_TEXT_TOKENS = 512  # Wan I2V: the last 512 encoder tokens are text


def apply_rotary_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE on interleaved (even, odd) pairs of the last dim; cos/sin carry the
    pair angle in the even (cos) / odd (sin) slots, broadcast over heads."""
    xe, xo = x[..., 0::2].float(), x[..., 1::2].float()
    c, s = cos[..., 0::2].float(), sin[..., 1::2].float()
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    out[..., 0::2] = xe * c - xo * s
    out[..., 1::2] = xe * s + xo * c
    return out.to(x.dtype)


def slice_rotary(rotary_emb: Sequence[torch.Tensor], local_seq: int, rank: int, world: int):
    """Cut each table's full-sequence dimension to this rank's tokens."""
    full = local_seq * world
    out = []
    for t in rotary_emb:
        for d in range(t.dim()):
            if t.shape[d] == full:
                t = t.narrow(d, rank * local_seq, local_seq)
                break
        out.append(t)
    return type(rotary_emb)(out)


class WanAdapter(ModelAdapter):
    def __init__(self) -> None:
        from ..prologue import RopeTableCache
        self._rope_cache = RopeTableCache()

    def patches_per_frame(self, height: int, width: int, pipe: Any) -> int:
        ps = getattr(pipe.transformer.config, "patch_size", [1, 2, 2])
        ps = int(ps[1]) if isinstance(ps, (list, tuple)) else int(ps)
        s = pipe.vae_scale_factor_spatial
        return (height // (s * ps)) * (width // (s * ps))

    def latent_frames(self, num_frames: int, pipe: Any) -> int:
        return (num_frames - 1) // pipe.vae_scale_factor_temporal + 1

    def reference_latent_frames(self, pipe: Any) -> int:
        sf = getattr(pipe.transformer.config, "sample_frames", None)
        return self.latent_frames(sf, pipe) if sf is not None else 21

    @staticmethod
    def _heads(attn: Any, x: torch.Tensor) -> torch.Tensor:
        return x.unflatten(2, (attn.heads, -1))

    def extract_qkv(self, attn, hidden_states, encoder_hidden_states):
        if getattr(attn, "fused_projections", False) and hasattr(attn, "to_qkv"):
            q, k, v = attn.to_qkv(hidden_states).chunk(3, dim=-1)
        else:
            q, k, v = attn.to_q(hidden_states), attn.to_k(hidden_states), attn.to_v(hidden_states)
        q, k = attn.norm_q(q), attn.norm_k(k)
        return self._heads(attn, q), self._heads(attn, k), self._heads(attn, v)

    def split_encoder_for_cross_attn(self, attn, encoder_hidden_states):
        if getattr(attn, "add_k_proj", None) is not None:
            n_img = encoder_hidden_states.shape[1] - IMAGE_TEXT_TOKENS
            return encoder_hidden_states[:, n_img:], encoder_hidden_states[:, :n_img]
        return encoder_hidden_states, None

    def extract_cross_attn_kv(self, attn, encoder_hidden_states):
        if getattr(attn, "add_k_proj", None) is None:
            return None
        k = attn.norm_added_k(attn.add_k_proj(encoder_hidden_states))
        v = attn.add_v_proj(encoder_hidden_states)
        return self._heads(attn, k), self._heads(attn, v)

    def project_qkv(self, attn, hidden_states, encoder_hidden_states, rotary_emb, local_seq, rank, world):
        """Projections, then the RMSNorm over the H*D row and the rotation of
        q and k in one pass each (the fused prologue kernel) when it applies;
        otherwise ``extract_qkv`` + ``apply_rotary``."""
        from ..prologue import fused_prologue_ok, norm_spec, qk_norm_rope
        if not hidden_states.is_cuda:
            return super().project_qkv(attn, hidden_states, encoder_hidden_states, rotary_emb, local_seq, rank, world)
        if getattr(attn, "fused_projections", False) and hasattr(attn, "to_qkv"):
            q, k, v = attn.to_qkv(hidden_states).chunk(3, dim=-1)
        else:
            q, k, v = attn.to_q(hidden_states), attn.to_k(hidden_states), attn.to_v(hidden_states)
        q, k, v = self._heads(attn, q), self._heads(attn, k), self._heads(attn, v)
        dim = q.shape[-2] * q.shape[-1]
        sq = norm_spec(getattr(attn, "norm_q", None), False, dim, q.dtype)
        sk = norm_spec(getattr(attn, "norm_k", None), False, dim, k.dtype)
        tabs = None if rotary_emb is None else self._rope_cache.get(rotary_emb, local_seq, rank, world)
        if sq is not None and sk is not None and (rotary_emb is None or tabs is not None) and fused_prologue_ok(q, k):
            cs, sn, off = tabs if tabs is not None else (None, None, 0)
            qk_norm_rope(q, *sq, cos=cs, sin=sn, rope_offset=off)
            qk_norm_rope(k, *sk, cos=cs, sin=sn, rope_offset=off)
            return q, k, v
        q = self._heads(attn, attn.norm_q(q.flatten(2, 3)))
        k = self._heads(attn, attn.norm_k(k.flatten(2, 3)))
        q, k = self.apply_rotary(q, k, rotary_emb, local_seq, rank, world)
        return q, k, v

    def apply_rotary(self, query, key, rotary_emb, local_seq, rank, world):
        if rotary_emb is None:
            return query, key
        cos, sin = slice_rotary(tuple(rotary_emb), local_seq, rank, world)
        return apply_rotary_interleaved(query, cos, sin), apply_rotary_interleaved(key, cos, sin)

    def output_projection(self, attn, hidden_states, query_dtype):
        h = hidden_states.flatten(2, 3).to(query_dtype)
        h = attn.to_out[0](h)
        return attn.to_out[1](h)

    def cross_attention(self, attn, query, encoder_image, attention_backend):
        if encoder_image is None:
            return None
        kv = self.extract_cross_attn_kv(attn, encoder_image)
        if kv is None:
            return None
        k, v = kv
        # Dense image-context attention of the model itself (not the LVSA path).
        out = F.scaled_dot_product_attention(query.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        return out.transpose(1, 2).flatten(2, 3).type_as(query)

    def install_processor(self, pipe: Any, processor: Any) -> int:
        for block in pipe.transformer.blocks:
            block.attn1.processor = processor
        return len(pipe.transformer.blocks)
