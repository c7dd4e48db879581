"""Model adapter interface (mirror of lvsa/adapters/base.py:19-239).

An adapter turns a diffusion model's attention layer into the generic
pieces the LVSA processor needs: Q/K/V in ``[B, seq, H, D]`` (QK-normed),
optional encoder (text) Q/K/V for dual-stream models, RoPE, the output
projection and any extra cross-attention (e.g. image context).  Method names
and meanings follow the reference so existing adapters port unchanged.
"""

from abc import ABC, abstractmethod
from typing import Any, Optional, Tuple

import torch


class ModelAdapter(ABC):
    """Bridge between one model family's attention layer and the LVSA path."""

    # geometry ---------------------------------------------------------------
    @abstractmethod
    def patches_per_frame(self, height: int, width: int, pipe: Any) -> int:
        """Spatial tokens per latent frame."""

    @abstractmethod
    def latent_frames(self, num_frames: int, pipe: Any) -> int:
        """Raw video frames -> latent frames."""

    @abstractmethod
    def reference_latent_frames(self, pipe: Any) -> int:
        """Latent frame count the model was trained on."""

    # projections ------------------------------------------------------------
    @abstractmethod
    def extract_qkv(self, attn: Any, hidden_states: torch.Tensor,
                    encoder_hidden_states: Optional[torch.Tensor]
                    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Video Q, K, V as ``[B, seq, H, D]``, QK-normed."""

    @abstractmethod
    def extract_cross_attn_kv(self, attn: Any, encoder_hidden_states: torch.Tensor
                              ) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        """K, V of an extra cross-attention context, or None."""

    @abstractmethod
    def split_encoder_for_cross_attn(self, attn: Any, encoder_hidden_states: torch.Tensor
                                     ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """(text tokens for self-attention, image context or None)."""

    @abstractmethod
    def apply_rotary(self, query: torch.Tensor, key: torch.Tensor, rotary_emb: Any,
                     local_seq: int, rank: int, world: int
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
        """RoPE on video Q and K (sliced to this rank's tokens)."""

    def project_qkv(self, attn: Any, hidden_states: torch.Tensor,
                    encoder_hidden_states: Optional[torch.Tensor], rotary_emb: Any,
                    local_seq: int, rank: int, world: int
                    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Video Q, K, V ready for attention: what ``extract_qkv`` followed by
        ``apply_rotary`` returns.  Adapters whose QK norm and rotation the
        fused prologue kernel covers override this to run both in one pass."""
        q, k, v = self.extract_qkv(attn, hidden_states, encoder_hidden_states)
        q, k = self.apply_rotary(q, k, rotary_emb, local_seq, rank, world)
        return q, k, v

    @abstractmethod
    def output_projection(self, attn: Any, hidden_states: torch.Tensor,
                          query_dtype: torch.dtype) -> torch.Tensor:
        """``[B, seq, H, D]`` -> ``[B, seq, C]``."""

    def extract_encoder_qkv(self, attn: Any, encoder_hidden_states: torch.Tensor
                            ) -> Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        """Encoder Q, K, V for dual-stream models; None for single-stream."""
        return None

    def format_output(self, attn: Any, hidden_states: torch.Tensor,
                      encoder_output: Optional[torch.Tensor], encoder_seq_len: int,
                      query_dtype: torch.dtype) -> Any:
        """What the block's forward() expects (a tensor, or a tuple for dual-stream)."""
        return hidden_states

    @abstractmethod
    def cross_attention(self, attn: Any, query: torch.Tensor, encoder_image: Optional[torch.Tensor],
                        attention_backend: Any) -> Optional[torch.Tensor]:
        """Extra dense cross-attention output ``[B, seq, C]`` or None."""

    # pipeline integration ---------------------------------------------------
    def install_processor(self, pipe: Any, processor: Any) -> int:
        raise NotImplementedError

    def setup_context_parallel(self, transformer: Any, world: int) -> None:
        raise NotImplementedError

    def patch_rotary_for_cp(self, rank: int, world: int) -> None:
        raise NotImplementedError
