"""Block-level LVSA hook for vllm-omni's Wan self-attention (interface of
lvsa-vllm-omni/lvsa_vllm_omni/wan_hook.py:31-179): the patched ``forward``
projects, norms and rotates as the model does, then runs the sparse pattern
in one kernel launch; warmup shapes, sharded sequences (sequence
parallelism) and other non-grid inputs go to the original dense forward."""

from typing import Any, Optional

from ..block_sparse import block_sparse_attention
from ._fallback import warn_fallback
from .config import LVSAConfig
from .hunyuan_hook import HunyuanLVSAState, _distributed, _log_engagement_once, _maybe_log_mask


def install_wan_lvsa_hook(total_latent_frames: int) -> None:
    """Patch ``WanSelfAttention.forward`` (class level, before the model is
    instantiated)."""
    from vllm_omni.diffusion.models.wan2_2.wan2_2_transformer import WanSelfAttention
    from vllm_omni.diffusion.layers.rope import RotaryEmbeddingWan

    config = LVSAConfig.from_env()
    state = HunyuanLVSAState(config)
    wan_rope = RotaryEmbeddingWan(is_neox_style=False, half_head_dim=True)
    _orig_forward = WanSelfAttention.forward

    def _lvsa_forward(self, hidden_states, rotary_emb: Optional[tuple] = None, attn_metadata: Optional[Any] = None):
        seq = hidden_states.shape[1]
        step_idx = state.tick(id(self), seq)
        dist_on = _distributed()
        if not (total_latent_frames > 0 and seq % total_latent_frames == 0 and not dist_on):
            warn_fallback("wan_hook", "distributed_cp" if dist_on else "geometry_mismatch", seq,
                          {"T_lat": total_latent_frames, "full_seq": seq, "distributed": dist_on})
            return _orig_forward(self, hidden_states, rotary_emb, attn_metadata)
        P = seq // total_latent_frames
        qkv, _ = self.to_qkv(hidden_states)
        hd, nh, nkv = self.head_dim, self.num_heads, self.num_kv_heads
        q, k, v = qkv.split([nh * hd, nkv * hd, nkv * hd], dim=-1)
        q, k = self.norm_q(q), self.norm_k(k)  # RMSNorm over the flat row, before the head split
        q, k, v = q.unflatten(2, (nh, hd)), k.unflatten(2, (nkv, hd)), v.unflatten(2, (nkv, hd))
        if rotary_emb is not None:
            cos, sin = rotary_emb
            q, k = wan_rope(q, cos, sin), wan_rope(k, cos, sin)
        _log_engagement_once(state, "wan", total_latent_frames, P, seq, step_idx)
        _maybe_log_mask(state, step_idx, total_latent_frames)
        out, _ = block_sparse_attention(q, k, v, state.get_mask(total_latent_frames, P, step_idx, q.device, 0))
        out = self.to_out(out.flatten(2, 3).type_as(q))
        return self.dropout(out)

    WanSelfAttention.forward = _lvsa_forward
    from .attention_impl import LVSAAttentionImpl
    LVSAAttentionImpl._hook_active = True
    print(f"[LVSA-hook] Installed LVSA hook on WanSelfAttention (T_lat={total_latent_frames}, "
          f"sparsity_scale={config.sparsity_scale})", flush=True)
