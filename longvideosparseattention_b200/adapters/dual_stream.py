"""Shared parts of the HunyuanVideo and CogVideoX adapters.

Both models attend video and text tokens jointly with per-head QK norms and a
3-D rotary embedding on the video tokens only; the LVSA processor gets the
text stream as encoder Q/K/V (dense rows, attended by every video query).
Method meanings follow lvsa/adapters/base.py:19-239.
"""

from typing import Any, Optional, Sequence, Tuple

import torch

from .base import ModelAdapter
from .wan import apply_rotary_interleaved


def slice_rope(rotary_emb: Any, local_seq: int, rank: int, world: int) -> Any:
    """This rank's rows of a rotary table (a tensor or a (cos, sin) pair):
    the first dimension of size local_seq * world is cut; a table without one
    is returned unchanged (lvsa/rope.py:31-57 behaviour)."""
    if world <= 1 or rotary_emb is None:
        return rotary_emb

    def cut(t: torch.Tensor) -> torch.Tensor:
        for d in range(t.dim()):
            if t.shape[d] == local_seq * world:
                return t.narrow(d, rank * local_seq, local_seq).contiguous()
        return t
    if isinstance(rotary_emb, torch.Tensor):
        return cut(rotary_emb)
    return type(rotary_emb)(cut(t) for t in rotary_emb)


def _pair_tables(rotary_emb: Any) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    if isinstance(rotary_emb, (tuple, list)) and len(rotary_emb) == 2:
        return rotary_emb[0], rotary_emb[1]
    return None


class DualStreamAdapter(ModelAdapter):
    """Per-head QK norm (``norm_q``/``norm_k`` on [.., H, D]) + rotary on video."""

    def __init__(self) -> None:
        from ..prologue import RopeTableCache
        self._rope_cache = RopeTableCache()

    @staticmethod
    def _split_heads(attn: Any, x: torch.Tensor) -> torch.Tensor:
        return x.unflatten(-1, (attn.heads, x.shape[-1] // attn.heads))

    @staticmethod
    def _norm(module: Any, x: torch.Tensor) -> torch.Tensor:
        return x if module is None else module(x)

    def _video_projections(self, attn: Any, hidden_states: torch.Tensor):
        return (self._split_heads(attn, attn.to_q(hidden_states)), self._split_heads(attn, attn.to_k(hidden_states)),
                self._split_heads(attn, attn.to_v(hidden_states)))

    def extract_qkv(self, attn, hidden_states, encoder_hidden_states):
        q, k, v = self._video_projections(attn, hidden_states)
        return self._norm(getattr(attn, "norm_q", None), q), self._norm(getattr(attn, "norm_k", None), k), v

    def split_encoder_for_cross_attn(self, attn, encoder_hidden_states):
        return encoder_hidden_states, None  # joint attention: no separate image context

    def extract_cross_attn_kv(self, attn, encoder_hidden_states):
        return None

    def cross_attention(self, attn, query, encoder_image, attention_backend):
        return None

    def apply_rotary(self, query, key, rotary_emb, local_seq, rank, world):
        if rotary_emb is None:
            return query, key
        tabs = _pair_tables(slice_rope(rotary_emb, local_seq, rank, world))
        if tabs is None:
            raise TypeError("rotary embedding must be a (cos, sin) pair")
        cos, sin = tabs
        # [S, D] tables broadcast over batch and heads.
        if cos.dim() == 2:
            cos, sin = cos[None, :, None, :], sin[None, :, None, :]
        return apply_rotary_interleaved(query, cos, sin), apply_rotary_interleaved(key, cos, sin)

    def project_qkv(self, attn, hidden_states, encoder_hidden_states, rotary_emb, local_seq, rank, world):
        """Projections, then per-head norm and rotation of q and k in one pass
        each (fused prologue kernel) when it applies."""
        from ..prologue import fused_prologue_ok, norm_spec, qk_norm_rope
        if not hidden_states.is_cuda:
            return super().project_qkv(attn, hidden_states, encoder_hidden_states, rotary_emb, local_seq, rank, world)
        q, k, v = self._video_projections(attn, hidden_states)
        D = q.shape[-1]
        sq = norm_spec(getattr(attn, "norm_q", None), True, D, q.dtype)
        sk = norm_spec(getattr(attn, "norm_k", None), True, D, k.dtype)
        tabs = None if rotary_emb is None else self._rope_cache.get(rotary_emb, local_seq, rank, world)
        if (sq is not None and sk is not None and (rotary_emb is None or tabs is not None)
                and fused_prologue_ok(q, k) and q.stride(-2) % 8 == 0):
            cs, sn, off = tabs if tabs is not None else (None, None, 0)
            qk_norm_rope(q, *sq, cos=cs, sin=sn, rope_offset=off)
            qk_norm_rope(k, *sk, cos=cs, sin=sn, rope_offset=off)
            return q, k, v
        q, k = self._norm(getattr(attn, "norm_q", None), q), self._norm(getattr(attn, "norm_k", None), k)
        q, k = self.apply_rotary(q, k, rotary_emb, local_seq, rank, world)
        return q, k, v

    def output_projection(self, attn, hidden_states, query_dtype):
        h = hidden_states.flatten(2, 3).to(query_dtype)
        h = attn.to_out[0](h)
        return attn.to_out[1](h) if len(attn.to_out) > 1 else h
