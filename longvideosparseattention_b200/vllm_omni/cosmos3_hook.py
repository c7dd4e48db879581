"""Block-level LVSA hook for NVIDIA Cosmos 3's generation-stream attention
(interface of lvsa-vllm-omni/lvsa_vllm_omni/cosmos3_hook.py:56-219).

``Cosmos3CrossAttention.forward(hidden_states, k_und, v_und, freqs_cos,
freqs_sin)``: the generation tokens form the T_lat x P grid; the
understanding K/V arrive pre-computed and are attended by every generation
query, i.e. they are the kernel's second (always attended) key segment.
Grouped-query attention runs natively (K/V stay at the KV head count);
``LVSA_REPEAT_KV=1`` repeats them to the query heads instead, as the
reference's ablation switch does.  Under sequence parallelism or on
non-grid shapes the original dense forward runs."""

import os

import torch.nn.functional as F

from ..block_sparse import block_sparse_attention
from ._fallback import warn_fallback
from .config import LVSAConfig
from .hunyuan_hook import HunyuanLVSAState, _log_engagement_once, _maybe_log_mask


def install_cosmos3_lvsa_hook(total_latent_frames: int) -> None:
    from vllm_omni.diffusion.models.cosmos3.transformer_cosmos3 import (
        Cosmos3CrossAttention,
        _apply_rotary_pos_emb,
        _is_sp_active,
    )

    state = HunyuanLVSAState(LVSAConfig.from_env())
    repeat_kv = os.environ.get("LVSA_REPEAT_KV", "").lower() in ("1", "true", "yes")
    _orig_forward = Cosmos3CrossAttention.forward

    def _lvsa_forward(self, hidden_states, k_und, v_und, freqs_cos, freqs_sin):
        B, S_gen, _ = hidden_states.shape
        step_idx = state.tick(id(self), S_gen)
        if _is_sp_active():
            warn_fallback("cosmos3_hook", "sequence_parallel", S_gen, {"step": step_idx})
            return _orig_forward(self, hidden_states, k_und, v_und, freqs_cos, freqs_sin)
        if total_latent_frames <= 0 or S_gen % total_latent_frames:
            warn_fallback("cosmos3_hook", "geometry_mismatch", S_gen, {"step": step_idx, "T_lat": total_latent_frames})
            return _orig_forward(self, hidden_states, k_und, v_und, freqs_cos, freqs_sin)
        P = S_gen // total_latent_frames
        q = self.to_q(hidden_states).view(B, S_gen, self.num_heads_local, self.head_dim)
        k = self.to_k(hidden_states).view(B, S_gen, self.num_kv_heads_local, self.head_dim)
        v = self.to_v(hidden_states).view(B, S_gen, self.num_kv_heads_local, self.head_dim)
        q = F.rms_norm(q, (q.shape[-1],), self.norm_q.weight, self.norm_q.variance_epsilon)
        k = F.rms_norm(k, (k.shape[-1],), self.norm_k.weight, self.norm_k.variance_epsilon)
        q, k = _apply_rotary_pos_emb(q, k, freqs_cos, freqs_sin)
        _log_engagement_once(state, "cosmos3", total_latent_frames, P, S_gen, step_idx)
        _maybe_log_mask(state, step_idx, total_latent_frames)
        if repeat_kv and self.num_heads_local != self.num_kv_heads_local:
            rep = self.num_heads_local // self.num_kv_heads_local
            k, v = k.repeat_interleave(rep, dim=2), v.repeat_interleave(rep, dim=2)
            k_und, v_und = k_und.repeat_interleave(rep, dim=2), v_und.repeat_interleave(rep, dim=2)
        # Generation rows: sparse pattern + every understanding token (no text query rows).
        mask = state.get_mask(total_latent_frames, P, step_idx, q.device, int(k_und.shape[1]))
        out, _ = block_sparse_attention(q, k, v, mask, None, k_und, v_und)
        return self.to_out(out.reshape(B, S_gen, -1))

    Cosmos3CrossAttention.forward = _lvsa_forward
    from .attention_impl import LVSAAttentionImpl
    LVSAAttentionImpl._hook_active = True
    print(f"[LVSA-hook] Installed LVSA hook on Cosmos3CrossAttention (T_lat={total_latent_frames})")
