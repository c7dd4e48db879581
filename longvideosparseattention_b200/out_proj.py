"""The attention output projection (``attn.to_out[0]``) on the hand-written
tcgen05 GEMM, reading the attention output in place.

The kernel writes O as [B, S, H, D] token-major, which is exactly the
K-major [B*S, H*D] operand the GEMM consumes: no transpose, no copy between
the two launches.  ``attention_out_projection`` is the fused layer tail the
adapters run (attention, then the projection) as two back-to-back launches
on one stream; replaces the torch Linear after LVSA attention
(lvsa/adapters/wan.py:121-131, lvsa/adapters/hunyuan_video.py:207-217).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native as N
from .block_sparse import _DTYPES, _stream_ptr, block_sparse_attention, error_word


def out_projection(o: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[..., S, H, D] (or [..., S, H*D]) attention output x weight^T + bias
    -> [..., S, out_features], same dtype (bf16 / f16).  ``o`` must have its
    H*D features contiguous per token."""
    if not o.is_cuda:
        raise RuntimeError("out_projection needs CUDA tensors (no CPU fallback)")
    if o.dtype not in _DTYPES or weight.dtype != o.dtype or (bias is not None and bias.dtype != o.dtype):
        raise ValueError("out_projection: o, weight and bias in one of bf16 / f16")
    K = weight.shape[1]
    if o.shape[-1] == K:
        lead = o.shape[:-1]
    elif o.dim() >= 3 and o.shape[-1] * o.shape[-2] == K:
        lead = o.shape[:-2]
    else:
        raise ValueError(f"out_projection: features of o {tuple(o.shape)} do not match weight {tuple(weight.shape)}")
    a = o.reshape(-1, K) if o.is_contiguous() else o.contiguous().reshape(-1, K)
    if a.stride(1) != 1:
        a = a.contiguous()
    w = weight if weight.stride(1) == 1 else weight.contiguous()
    Nout = weight.shape[0]
    y = out if out is not None else torch.empty(a.shape[0], Nout, dtype=o.dtype, device=o.device)
    args = N.LvsaOutProjArgs(a.data_ptr(), w.data_ptr(), bias.data_ptr() if bias is not None else None,
                             y.data_ptr(), a.stride(0), w.stride(0), y.stride(0), a.shape[0], Nout, K,
                             _DTYPES[o.dtype], error_word(o.device).data_ptr())
    with torch.cuda.device(o.device):
        st = N.load().lvsa_out_proj(ctypes.byref(args), _stream_ptr(o.device))
    N.check(st, "lvsa_out_proj")
    return y.view(*lead, Nout)


def attention_out_projection(q, k, v, mask, weight, bias=None, text_q=None, text_k=None, text_v=None,
                             text_weight=None, text_bias=None, scale=None):
    """LVSA attention followed by the output projection(s): the video rows
    through ``weight`` (to_out[0]) and, for dual-stream models, the text rows
    through ``text_weight`` (to_add_out).  Returns (video, text or None)."""
    o, to = block_sparse_attention(q, k, v, mask, text_q, text_k, text_v, scale=scale)
    y = out_projection(o, weight, bias)
    ty = None
    if to is not None and text_weight is not None:
        ty = out_projection(to, text_weight, text_bias)
    return y, ty
