"""Fused QK prologue: the adapters' QK norm + rotary embedding in one pass.

``qk_norm_rope`` replaces, for one of q / k, the pair of elementwise passes
the reference adapters run before attention:

* Wan (lvsa/adapters/wan.py:48-67, 103-119; lvsa/rope.py:10-28): RMSNorm over
  the whole H*D row (``norm="rms_row"``, weight [H*D]) + interleaved RoPE.
* HunyuanVideo (lvsa/adapters/hunyuan_video.py:71-103, 156-205): RMSNorm per
  head (``norm="rms_head"``, weight [D]) + RoPE on the video tokens.
* CogVideoX (lvsa/adapters/cogvideox.py:88-117, 169-217): LayerNorm per head
  (``norm="layer_head"``, weight and bias [D]) + RoPE on the video tokens.

RoPE tables follow the reference's layout: ``cos``/``sin`` broadcastable to
[B?, S, 1?, D] with the pair angle at even (cos) / odd (sin) positions; they
are reduced here to [B?, S, D/2] fp32 once per call (``rope_tables``).
Arithmetic is fp32 with one rounding to the storage type (the unfused path
rounds after the norm and again after the rotation).
"""

from __future__ import annotations

import ctypes
from typing import Any, Optional, Tuple

import torch

from . import _native as N
from .block_sparse import _stream_ptr

_NORMS = {None: N.LVSA_NORM_NONE, "none": N.LVSA_NORM_NONE, "rms_row": N.LVSA_NORM_RMS_ROW,
          "rms_head": N.LVSA_NORM_RMS_HEAD, "layer_head": N.LVSA_NORM_LAYER_HEAD}
_DT = {torch.bfloat16: N.LVSA_DTYPE_BF16, torch.float16: N.LVSA_DTYPE_F16, torch.float32: N.LVSA_DTYPE_F32}


def rope_tables(cos: torch.Tensor, sin: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Reference (cos, sin) tables, [S, D] or [B, S, 1, D] with the pair angle
    in the even (cos) / odd (sin) slots as lvsa/rope.py:22-23 reads them ->
    contiguous fp32 pair-angle tables [S, D/2] or [B, S, D/2]."""
    def red(t: torch.Tensor, even: bool) -> torch.Tensor:
        t = t[..., 0::2] if even else t[..., 1::2]
        if t.dim() == 4:          # [B, S, 1, D/2]: drop the head axis
            t = t[:, :, 0, :]
        if t.dim() == 3 and t.shape[0] == 1:
            t = t[0]
        if t.dim() not in (2, 3):
            raise ValueError(f"unsupported rotary table shape {tuple(t.shape)}")
        return t.float().contiguous()
    return red(cos, True), red(sin, False)


def qk_norm_rope(x: torch.Tensor, norm: Optional[str] = None, weight: Optional[torch.Tensor] = None,
                 bias: Optional[torch.Tensor] = None, eps: float = 1e-6,
                 cos: Optional[torch.Tensor] = None, sin: Optional[torch.Tensor] = None,
                 rope_offset: int = 0) -> torch.Tensor:
    """In place on x [B, S, H, D] (bf16/fp16, stride 1 over D); returns x.
    cos/sin: fp32 [S_tab, D/2] or [B, S_tab, D/2] pair-angle tables (see
    ``rope_tables``); token s of x uses table row rope_offset + s."""
    if not x.is_cuda:
        raise RuntimeError("qk_norm_rope needs a CUDA tensor (no CPU fallback)")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"qk_norm_rope: bf16/fp16 input expected, got {x.dtype}")
    if x.stride(-1) != 1:
        raise ValueError("qk_norm_rope: x must be contiguous over head_dim")
    B, S, H, D = x.shape
    nm = _NORMS[norm]
    wt = None
    if weight is not None:
        wt = weight.detach().contiguous()
        if wt.dtype not in _DT:
            wt = wt.float()
    bs = bias.detach().to(wt.dtype if wt is not None else torch.float32).contiguous() if bias is not None else None
    cs = sn = None
    stride_b = 0
    if cos is not None:
        cs, sn = cos.float().contiguous(), sin.float().contiguous()
        if cs.shape[-1] != D // 2:
            raise ValueError(f"rope tables must be [.., S, {D // 2}], got {tuple(cs.shape)}")
        stride_b = cs.stride(0) if cs.dim() == 3 and cs.shape[0] > 1 else 0
        if cs.shape[-2] < rope_offset + S:
            raise ValueError("rope tables shorter than rope_offset + seq")
    args = N.LvsaQkPrologue(
        N.LvsaTensor(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2)), _DT[x.dtype], B, S, H, D, nm,
        _DT[wt.dtype] if wt is not None else N.LVSA_DTYPE_F32,
        wt.data_ptr() if wt is not None else None, bs.data_ptr() if bs is not None else None, float(eps),
        cs.data_ptr() if cs is not None else None, sn.data_ptr() if sn is not None else None,
        stride_b, int(rope_offset))
    with torch.cuda.device(x.device):
        st = N.load().lvsa_qk_prologue(ctypes.byref(args), _stream_ptr(x.device))
    N.check(st, "lvsa_qk_prologue")
    return x


_NO_NORM = (None, None, None, 0.0)


def norm_spec(module: Any, per_head: bool, dim: int, dtype: torch.dtype):
    """(norm, weight, bias, eps) for a QK-norm module the prologue kernel can
    run over ``dim`` values (H*D for the row norm, D per head), or None if it
    cannot (the caller then keeps the module call).  Recognised: None /
    Identity (no norm), RMSNorm (torch.nn.RMSNorm, or a module named
    *RMSNorm with ``weight`` and ``eps``), LayerNorm over the last dim."""
    if module is None or isinstance(module, torch.nn.Identity):
        return _NO_NORM
    w = getattr(module, "weight", None)
    if w is not None and w.numel() != dim:
        return None
    if "RMSNorm" in type(module).__name__ and hasattr(module, "eps"):
        eps = module.eps if module.eps is not None else torch.finfo(dtype).eps
        return ("rms_head" if per_head else "rms_row"), w, None, float(eps)
    if isinstance(module, torch.nn.LayerNorm) and per_head and tuple(module.normalized_shape) == (dim,):
        return "layer_head", w, module.bias, float(module.eps)
    return None


def fused_prologue_ok(*tensors: torch.Tensor) -> bool:
    """The in-place kernel applies: CUDA bf16/fp16 tensors, no autograd."""
    return all(t.is_cuda and t.dtype in (torch.bfloat16, torch.float16) and t.stride(-1) == 1 and
               not (torch.is_grad_enabled() and t.requires_grad) for t in tensors)


class RopeTableCache:
    """Pair-angle tables of the last rotary embedding seen (every layer of a
    denoising step passes the same tensors), and where this rank's tokens
    start in them."""

    def __init__(self) -> None:
        self._key = None
        self._tables: Optional[Tuple[torch.Tensor, torch.Tensor]] = None

    def get(self, rotary_emb: Any, local_seq: int, rank: int, world: int):
        """(cos, sin, rope_offset) for a (cos, sin) rotary embedding, or None
        when its layout is not one the kernel reads."""
        if not isinstance(rotary_emb, (tuple, list)) or len(rotary_emb) != 2:
            return None
        cos, sin = rotary_emb
        if not (isinstance(cos, torch.Tensor) and isinstance(sin, torch.Tensor)) or not cos.is_cuda:
            return None
        key = (cos.data_ptr(), sin.data_ptr(), tuple(cos.shape), tuple(sin.shape), cos.device)
        if key != self._key:
            try:
                self._tables = rope_tables(cos, sin)
            except ValueError:
                return None
            self._key = key
        cs, sn = self._tables
        rows = cs.shape[-2]
        if rows == local_seq * world:
            return cs, sn, rank * local_seq
        if rows == local_seq:
            return cs, sn, 0
        return None
