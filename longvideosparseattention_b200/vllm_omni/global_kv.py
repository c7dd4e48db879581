"""Anchor-frame K/V gather (mirror of lvsa-vllm-omni/lvsa_vllm_omni/global_kv.py:12-42).

The sm_100a kernel reads anchor frames in place, so the LVSA path never needs
this copy; it is kept for callers of the reference API."""

from typing import List, Tuple

import torch


def build_global_kv(key: torch.Tensor, value: torch.Tensor, global_indices: List[int],
                    num_patches: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Tokens of the anchor frames, ``[B, |G| * P, H, D]`` each."""
    if not global_indices:
        B, _, H, D = key.shape
        return key.new_empty(B, 0, H, D), value.new_empty(B, 0, H, D)
    g = torch.as_tensor(global_indices, dtype=torch.long, device=key.device)
    idx = (g[:, None] * num_patches + torch.arange(num_patches, device=key.device)[None, :]).reshape(-1)
    return key[:, idx], value[:, idx]
