"""Block-level LVSA hook for vllm-omni's HunyuanVideo-1.5 attention, and the
hook state shared with the Wan and Cosmos 3 hooks (interface of
lvsa-vllm-omni/lvsa_vllm_omni/hunyuan_hook.py:29-410).

The patched ``forward`` projects the video and encoder streams as the model
does and then runs both in ONE launch of the sm_100a kernel: video rows
sparse (plus every text token), text rows dense, where the reference runs the
global-K/V gather, the per-frame SDPA loop and a separate dense SDPA for the
text queries.  vllm-omni is imported only when a hook is installed.
"""

import os
from types import SimpleNamespace
from typing import Optional

import torch

from ..block_sparse import block_sparse_attention
from ..sparse_attention import LVSAMetadata, compute_auto_kfi, compute_global_indices, \
    print_attention_mask_compact
from ..observability import StepLogger
from ..step_mask import SHARED
from ._fallback import warn_fallback
from .config import LVSAConfig


def _mask_log_should_fire(spec: str, step_idx: int, last_step: int) -> bool:
    """``LVSA_MASK_LOG`` selector: '1' every step, 'once', 'N', 'N-M', 'N,M,K';
    never twice for one step, never for '' or '0' or an unparsable spec."""
    if not spec or spec == "0" or step_idx == last_step:
        return False
    if spec == "1":
        return True
    if spec == "once":
        return last_step == -1
    try:
        if "-" in spec:
            lo, hi = (int(x) for x in spec.split("-", 1))
            return lo <= step_idx <= hi
        return step_idx in {int(x) for x in spec.split(",") if x.strip()}
    except ValueError:
        return False


def _log_engagement_once(state, model, total_latent_frames, num_patches, seq_len, step_idx) -> None:
    """One line per generation confirming that the sparse path engaged."""
    if state._engaged_logged:
        return
    state._engaged_logged = True
    metadata = state.pattern_info(total_latent_frames, step_idx)
    kfi = metadata.key_frame_interval
    mode = "SPARSE" if kfi > 1 else "DENSE (T_lat <= ref)"
    print(f"[LVSA] engaged ({model}): T_lat={total_latent_frames} P={num_patches} seq_len={seq_len} "
          f"kfi={kfi} W={metadata.window_size} |G|={len(metadata.global_set)} -> {mode}", flush=True)


def _maybe_log_mask(state, step_idx: int, total_latent_frames: int) -> None:
    spec = os.environ.get("LVSA_MASK_LOG", "")
    if _mask_log_should_fire(spec, step_idx, state._mask_log_last_step):
        state._mask_log_last_step = step_idx
        metadata = state.pattern_info(total_latent_frames, step_idx)
        print(f"[LVSA-MASK] step={step_idx}  T_lat={total_latent_frames}  W={metadata.window_size}  "
              f"|G|={len(metadata.global_set)}  kfi={metadata.key_frame_interval}", flush=True)
        print_attention_mask_compact(total_latent_frames, metadata.window_size, metadata.global_set,
                                     metadata.expand_window)


def _distributed() -> bool:
    try:
        import torch.distributed as dist
        return dist.is_initialized() and dist.get_world_size() > 1
    except (ImportError, RuntimeError):
        return False


class HunyuanLVSAState:
    """State shared by every hooked attention block of a worker: the step
    counter (one step = n_blocks x CFG passes forwards; n_blocks calibrated on
    the first repeated block id; a new sequence length starts a new
    generation) and the per-step pattern cache.  Worker processes run one
    request loop on one thread, so it is not thread-local."""

    def __init__(self, config: LVSAConfig) -> None:
        self.config = config
        self._metadata: Optional[LVSAMetadata] = None
        self._cached_total_frames: Optional[int] = None
        self._cached_patches: Optional[int] = None
        self._cached_step = -1
        self._call_count = 0
        self._n_blocks: Optional[int] = None
        self._cfg_passes = max(1, int(os.environ.get("LVSA_CFG_PASSES", 2)))
        self._step = 0
        self._seen_ids: set = set()
        self._generation_seq_len: Optional[int] = None
        self._mask_log_last_step = -1
        self._engaged_logged = False
        self._logger = StepLogger()

    def tick(self, layer_id: int, seq_len: int) -> int:
        if self._generation_seq_len is not None and seq_len != self._generation_seq_len:
            self._call_count, self._step = 0, 0
            self._seen_ids.clear()
            self._engaged_logged = False
        self._generation_seq_len = seq_len
        self._call_count += 1
        if self._n_blocks is None:
            if layer_id in self._seen_ids:
                self._n_blocks = len(self._seen_ids)
                self._seen_ids.clear()
                print(f"[LVSA-hook] Step counter calibrated: n_blocks={self._n_blocks} "
                      f"cfg_passes={self._cfg_passes}")
            else:
                self._seen_ids.add(layer_id)
        if self._n_blocks is not None:
            new = max(self._step, (self._call_count - 1) // (self._n_blocks * self._cfg_passes))
            if new > self._step:
                self._logger.step_boundary(new)   # LVSA_MEM_LOG / LVSA_STEP_TIME_LOG
            self._step = new
        return self._step

    def key_frame_interval(self, total_latent_frames: int) -> Optional[int]:
        cfg = self.config
        kfi = cfg.latent_key_frame_interval
        if cfg.auto_keyframes:
            kfi = compute_auto_kfi(total_latent_frames, cfg.latent_window_size, cfg.latent_n_first_frames,
                                   reference_frames=cfg.reference_latent_frames,
                                   sparsity_scale=cfg.sparsity_scale)
        return kfi

    def pattern_info(self, total_latent_frames: int, step_idx: int) -> SimpleNamespace:
        """The fields the engagement and mask logs print (host arithmetic
        only: the global frame list, no metadata build)."""
        cfg = self.config
        kfi = self.key_frame_interval(total_latent_frames)
        off = step_idx % kfi if (cfg.rotate_keyframes and kfi and kfi > 0) else 0
        g = compute_global_indices(total_latent_frames, cfg.latent_n_first_frames, kfi, off)
        return SimpleNamespace(key_frame_interval=kfi, window_size=cfg.latent_window_size,
                               global_set=set(g), global_indices=g, expand_window=True)

    def get_mask(self, total_latent_frames: int, num_patches: int, step_idx: int, device: torch.device,
                 n_text: int = 0):
        """The step's GPU block mask, shared with every other hooked block and
        impl instance (``step_mask.SHARED``): built once per rotation into
        the same buffers, keyframe offset read on the GPU from the step."""
        cfg = self.config
        return SHARED.get(device, total_latent_frames, num_patches, cfg.latent_window_size,
                          cfg.latent_n_first_frames, self.key_frame_interval(total_latent_frames), True,
                          n_text, step_idx, rotate=cfg.rotate_keyframes)

    def get_metadata(self, total_latent_frames: int, num_patches: int, step_idx: int,
                     device: torch.device) -> LVSAMetadata:
        """Host LVSAMetadata of the step (reference interface; the forward
        path uses ``get_mask`` and never builds this)."""
        cfg = self.config
        if (self._metadata is None or self._cached_total_frames != total_latent_frames
                or self._cached_patches != num_patches or (cfg.rotate_keyframes and self._cached_step != step_idx)):
            W, nf, kfi = cfg.latent_window_size, cfg.latent_n_first_frames, cfg.latent_key_frame_interval
            if cfg.auto_keyframes:
                kfi = compute_auto_kfi(total_latent_frames, W, nf, reference_frames=cfg.reference_latent_frames,
                                       sparsity_scale=cfg.sparsity_scale)
            offset = step_idx % kfi if (cfg.rotate_keyframes and kfi and kfi > 0) else 0
            self._metadata = LVSAMetadata.build(total_latent_frames, num_patches, W, nf, kfi, 0, 1,
                                                expand_window=True, keyframe_offset=offset,
                                                reference_frames=cfg.reference_latent_frames,
                                                sparsity_scale=cfg.sparsity_scale)
            self._cached_total_frames, self._cached_patches, self._cached_step = (
                total_latent_frames, num_patches, step_idx)
        return self._metadata


def install_hunyuan_lvsa_hook(total_latent_frames: int) -> None:
    """Patch ``HunyuanVideo15Attention.forward`` (class level, before the
    model is instantiated)."""
    from vllm_omni.diffusion.models.hunyuan_video.hunyuan_video_15_transformer import (
        HunyuanVideo15Attention,
    )

    state = HunyuanLVSAState(LVSAConfig.from_env())
    _orig_forward = HunyuanVideo15Attention.forward

    def _lvsa_forward(self, hidden_states, encoder_hidden_states=None, attention_mask=None,
                      image_rotary_emb=None, hidden_states_mask=None):
        video_seq = hidden_states.shape[1]
        step_idx = state.tick(id(self), video_seq)
        dist_on = _distributed()
        if not (total_latent_frames > 0 and video_seq % total_latent_frames == 0
                and encoder_hidden_states is not None and not dist_on):
            reason = ("no_encoder" if encoder_hidden_states is None else
                      "distributed_cp" if dist_on else "geometry_mismatch")
            warn_fallback("hunyuan_hook", reason, video_seq, {"step": step_idx, "T_lat": total_latent_frames})
            return _orig_forward(self, hidden_states, encoder_hidden_states, attention_mask, image_rotary_emb,
                                 hidden_states_mask)
        P = video_seq // total_latent_frames
        hd = self.head_dim
        qkv, _ = self.to_qkv(hidden_states)
        nh, nkv = self.to_qkv.num_heads, self.to_qkv.num_kv_heads
        q, k, v = qkv.split([nh * hd, nkv * hd, nkv * hd], dim=-1)
        q, k, v = q.unflatten(-1, (nh, -1)), k.unflatten(-1, (nkv, -1)), v.unflatten(-1, (nkv, -1))
        q, k = self.norm_q(q), self.norm_k(k)
        if image_rotary_emb is not None:
            cos, sin = (t.to(q.dtype) for t in image_rotary_emb)
            q, k = self.rope(q, cos, sin), self.rope(k, cos, sin)
        eqkv, _ = self.add_kv_proj(encoder_hidden_states)
        enh, enkv = self.add_kv_proj.num_heads, self.add_kv_proj.num_kv_heads
        eq, ek, ev = eqkv.split([enh * hd, enkv * hd, enkv * hd], dim=-1)
        eq, ek, ev = eq.unflatten(-1, (enh, -1)), ek.unflatten(-1, (enkv, -1)), ev.unflatten(-1, (enkv, -1))
        eq, ek = self.norm_added_q(eq), self.norm_added_k(ek)
        _log_engagement_once(state, "hunyuan", total_latent_frames, P, video_seq, step_idx)
        _maybe_log_mask(state, step_idx, total_latent_frames)
        mask = state.get_mask(total_latent_frames, P, step_idx, q.device, int(ek.shape[1]))
        # Video rows sparse + every text token, text rows dense: one launch.
        out, enc_out = block_sparse_attention(q, k, v, mask, eq, ek, ev)
        hs = self.to_out[0](out.flatten(2, 3).to(q.dtype))
        enc = self.to_add_out(enc_out.flatten(2, 3).to(q.dtype))
        return hs, enc

    HunyuanVideo15Attention.forward = _lvsa_forward
    from .attention_impl import LVSAAttentionImpl
    LVSAAttentionImpl._hook_active = True
    print(f"[LVSA-hook] Installed LVSA hook on HunyuanVideo15Attention (T_lat={total_latent_frames})")
