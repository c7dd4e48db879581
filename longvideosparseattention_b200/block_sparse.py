"""Torch-facing wrappers over the C ABI: the GPU mask builder and the
block-sparse attention forward.

Both run on torch's current CUDA stream, allocate their outputs with torch
(caller-visible tensors) and never synchronise the host.  There is no CPU
path: a missing library or a non-CUDA tensor raises.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Dict, Optional, Sequence, Tuple

import torch

from . import _native as N
from .observability import nvtx_range

_ERR_WORDS: Dict[int, torch.Tensor] = {}

# Tile shape the attention kernel consumes: 128 query rows x 128 keys (one
# tcgen05 M=128 tile per CTA, S and P double-buffered in TMEM).  The mask
# builder accepts other shapes (multiples of 16 up to 256) for analysis.
ATTN_BLOCK_Q = 128
ATTN_BLOCK_K = 128


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 that kernels set to LVSA_ERR_DEVICE_TIMEOUT when a
    bounded wait expires.  Read it with ``check_device_errors``."""
    idx = torch.device(device).index or 0
    t = _ERR_WORDS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR_WORDS[idx] = t
    return t


def check_device_errors(device: torch.device, reset: bool = True) -> None:
    """Synchronising check of the device error word; raises LvsaError."""
    t = error_word(device)
    v = int(t.item())
    if reset and v:
        t.zero_()
    if v:
        raise N.LvsaError(v, "device")


@dataclass
class BlockMask:
    """GPU-resident pattern of one denoising step (output of lvsa_build_mask)."""

    total_frames: int
    num_patches: int
    window_size: int
    n_first_frames: int
    key_frame_interval: Optional[int]
    keyframe_offset: int
    expand_window: bool
    n_text: int
    block_q: int
    block_k: int
    n_video: int
    n_q_video_tiles: int
    n_q_tiles: int
    n_k_video_tiles: int
    n_k_tiles: int
    frame_words: int
    max_nnz: int
    global_frame_mask: torch.Tensor
    window_bounds: torch.Tensor
    frame_bits: torch.Tensor
    attended_indices: torch.Tensor
    frame_indptr: torch.Tensor
    frame_indices: torch.Tensor
    tile_indptr: torch.Tensor
    tile_indices: torch.Tensor
    tile_flags: torch.Tensor
    counters: torch.Tensor

    @property
    def device(self) -> torch.device:
        return self.tile_indptr.device

    def counts(self) -> Dict[str, int]:
        """(synchronising) tile nnz, attended C, frame nnz, compact_n."""
        c = self.counters.tolist()
        return dict(nnz=c[0], attended_C=c[1], frame_nnz=c[2], compact_n=c[3])

    def host_csr(self) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(synchronising) tile CSR on the host, trimmed to nnz."""
        nnz = int(self.counters[0].item())
        return (self.tile_indptr.cpu(), self.tile_indices[:nnz].cpu(), self.tile_flags[:nnz].cpu())


def mask_layout(total_frames: int, num_patches: int, window_size: int, n_first_frames: int,
                key_frame_interval: Optional[int], keyframe_offset: int = 0,
                expand_window: bool = True, n_text: int = 0, block_q: int = ATTN_BLOCK_Q,
                block_k: int = ATTN_BLOCK_K, boundary_guards: Optional[Sequence[int]] = None,
                device_step: Optional[torch.Tensor] = None):
    lib = N.load()
    guards = list(boundary_guards or [])
    garr = (ctypes.c_int32 * max(1, len(guards)))(*guards)
    pat = N.LvsaPattern(int(total_frames), int(num_patches), int(window_size), int(n_first_frames),
                        int(key_frame_interval or 0), int(keyframe_offset), int(bool(expand_window)),
                        int(n_text), int(block_q), int(block_k), len(guards),
                        ctypes.cast(garr, ctypes.POINTER(ctypes.c_int32)),
                        device_step.data_ptr() if device_step is not None else None)
    lay = N.LvsaMaskLayout()
    N.check(lib.lvsa_mask_layout(ctypes.byref(pat), ctypes.byref(lay)), "lvsa_mask_layout")
    return pat, lay, garr


def build_block_mask(total_frames: int, num_patches: int, window_size: int, n_first_frames: int,
                     key_frame_interval: Optional[int], keyframe_offset: int = 0,
                     expand_window: bool = True, n_text: int = 0, block_q: int = ATTN_BLOCK_Q,
                     block_k: int = ATTN_BLOCK_K, boundary_guards: Optional[Sequence[int]] = None,
                     device: Optional[torch.device] = None,
                     reuse: Optional[BlockMask] = None,
                     device_step: Optional[torch.Tensor] = None) -> BlockMask:
    """Build the step's pattern on the GPU (4 small kernels, no host sync).

    ``reuse``: a BlockMask of the same geometry whose buffers are overwritten
    (per-step keyframe rotation without reallocation).  ``device_step``: a
    one-element int32 CUDA tensor holding the step index; the builder reads
    it on the GPU (keyframe offset = step mod key_frame_interval) and
    ``keyframe_offset`` is ignored, so rotating is a device-side update of
    that word (graph-replayable)."""
    if device_step is not None and (not device_step.is_cuda or device_step.dtype != torch.int32):
        raise ValueError("device_step must be a CUDA int32 tensor")
    pat, lay, _keep = mask_layout(total_frames, num_patches, window_size, n_first_frames,
                                  key_frame_interval, keyframe_offset, expand_window, n_text,
                                  block_q, block_k, boundary_guards, device_step)
    device = torch.device(device) if device is not None else torch.device("cuda")
    if device.type != "cuda":
        raise RuntimeError("build_block_mask needs a CUDA device (no CPU fallback)")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    T = int(total_frames)
    same = (reuse is not None and reuse.device == device and reuse.total_frames == T
            and reuse.num_patches == num_patches and reuse.n_text == n_text
            and reuse.block_q == block_q and reuse.block_k == block_k and reuse.max_nnz >= lay.max_nnz)
    if same:
        bufs = reuse
        t = dict(global_frame_mask=reuse.global_frame_mask, window_bounds=reuse.window_bounds,
                 frame_bits=reuse.frame_bits, attended_indices=reuse.attended_indices,
                 frame_indptr=reuse.frame_indptr, frame_indices=reuse.frame_indices,
                 tile_indptr=reuse.tile_indptr, tile_indices=reuse.tile_indices,
                 tile_flags=reuse.tile_flags, counters=reuse.counters)
    else:
        kw = dict(device=device)
        t = dict(
            global_frame_mask=torch.empty(T, dtype=torch.int8, **kw),
            window_bounds=torch.empty(T, 2, dtype=torch.int32, **kw),
            frame_bits=torch.empty(T, lay.frame_words, dtype=torch.int32, **kw),
            attended_indices=torch.empty(T, T, dtype=torch.int32, **kw),
            frame_indptr=torch.empty(T + 1, dtype=torch.int32, **kw),
            frame_indices=torch.empty(T * T, dtype=torch.int32, **kw),
            tile_indptr=torch.empty(lay.n_q_tiles + 1, dtype=torch.int32, **kw),
            tile_indices=torch.empty(max(1, lay.max_nnz), dtype=torch.int32, **kw),
            tile_flags=torch.empty(max(1, lay.max_nnz), dtype=torch.uint8, **kw),
            counters=torch.zeros(4, dtype=torch.int32, **kw),
        )
    bufs_c = N.LvsaMaskBuffers(*[t[n].data_ptr() for n, _ in N.LvsaMaskBuffers._fields_])
    with torch.cuda.device(device), nvtx_range("lvsa_build_mask"):
        st = N.load().lvsa_build_mask(ctypes.byref(pat), ctypes.byref(bufs_c), _stream_ptr(device))
    N.check(st, "lvsa_build_mask")
    return BlockMask(
        total_frames=T, num_patches=int(num_patches), window_size=int(window_size),
        n_first_frames=int(n_first_frames), key_frame_interval=key_frame_interval,
        keyframe_offset=int(keyframe_offset), expand_window=bool(expand_window), n_text=int(n_text),
        block_q=int(block_q), block_k=int(block_k), n_video=lay.n_video,
        n_q_video_tiles=lay.n_q_video_tiles, n_q_tiles=lay.n_q_tiles,
        n_k_video_tiles=lay.n_k_video_tiles, n_k_tiles=lay.n_k_tiles,
        frame_words=lay.frame_words, max_nnz=max(int(lay.max_nnz), reuse.max_nnz if same else 0),
        **t)


_DTYPES = {torch.bfloat16: N.LVSA_DTYPE_BF16, torch.float16: N.LVSA_DTYPE_F16}


def _tview(x: Optional[torch.Tensor]) -> N.LvsaTensor:
    if x is None:
        return N.LvsaTensor(None, 0, 0, 0)
    if x.dim() != 4 or x.stride(-1) != 1:
        raise ValueError("expected a [B, N, H, D] tensor with a contiguous last dim")
    return N.LvsaTensor(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2))


def _prep(x: Optional[torch.Tensor], dtype: torch.dtype) -> Optional[torch.Tensor]:
    if x is None:
        return None
    if x.dtype != dtype:
        x = x.to(dtype)
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def quantize_e4m3(x: torch.Tensor, head_max: Optional[torch.Tensor] = None):
    """[B, N, H, D] bf16/fp16 -> (contiguous E4M3 bytes [B, N, H, D] uint8,
    per-128-token-tile scales [B, H, ceil(N/128)] fp32).  ``head_max`` [B, H]
    fp32 receives the running max of the tile scales."""
    B, Nn, H, D = x.shape
    if x.dtype not in _DTYPES:
        x = x.to(torch.bfloat16)
    if x.stride(-1) != 1:
        x = x.contiguous()
    q8 = torch.empty(B, Nn, H, D, dtype=torch.uint8, device=x.device)
    sc = torch.empty(B, H, -(-Nn // 128), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        st = N.load().lvsa_quantize_e4m3(ctypes.byref(_tview(x)), _DTYPES[x.dtype], B, Nn, H, D,
                                         q8.data_ptr(), sc.data_ptr(),
                                         head_max.data_ptr() if head_max is not None else None,
                                         _stream_ptr(x.device))
    N.check(st, "lvsa_quantize_e4m3")
    return q8, sc


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: BlockMask,
                           text_q: Optional[torch.Tensor] = None,
                           text_k: Optional[torch.Tensor] = None,
                           text_v: Optional[torch.Tensor] = None,
                           scale: Optional[float] = None, return_lse: bool = False,
                           out: Optional[torch.Tensor] = None,
                           text_out: Optional[torch.Tensor] = None, fp8: bool = False,
                           q_tiles: Optional[Tuple[int, int]] = None, wait_timeout_us: int = 0,
                           inject_fault: int = 0):
    """LVSA attention of one layer on the GPU.

    q [B, Nv, H, D], k/v [B, Nv, Hkv, D] (video, frame-major tokens);
    text_k/text_v [B, Nt, Hkv, D] (attended by every query); text_q
    [B, Nt, H, D] (optional, dense rows).  bf16/fp16 compute; fp32 inputs
    are rounded to bf16 and the output is returned in the input dtype.
    Returns (out, text_out) or, with ``return_lse``, (out, text_out, lse,
    text_lse) where lse is natural-log [B, H, N] fp32.

    ``q_tiles=(t0, t1)`` computes only tile-CSR rows [t0, t1) (video rows
    first, then text rows); the other rows of ``out`` / ``text_out`` are
    left as they are, so pass them to keep their contents.

    ``wait_timeout_us`` bounds every wait inside the kernel (default 2 s);
    ``inject_fault=1`` is a test hook that makes one CTA's waits expire
    (its rows are not written; the device error word reports it).
    """
    if not q.is_cuda:
        raise RuntimeError("block_sparse_attention needs CUDA tensors (no CPU fallback)")
    in_dtype = q.dtype
    cdt = in_dtype if in_dtype in _DTYPES else torch.bfloat16
    B, Nv, H, D = q.shape
    Hkv = k.shape[2]
    Nt = 0 if text_k is None else int(text_k.shape[1])
    if (mask.block_q, mask.block_k) != (ATTN_BLOCK_Q, ATTN_BLOCK_K):
        raise ValueError(f"the attention kernel needs a {ATTN_BLOCK_Q}x{ATTN_BLOCK_K} tile CSR, "
                         f"got {mask.block_q}x{mask.block_k}")
    n_kv = int(k.shape[1])
    if n_kv != Nv and n_kv != getattr(mask, "n_kv_video", Nv):
        raise AssertionError(f"key length {n_kv} does not match the mask ({getattr(mask, 'n_kv_video', Nv)})")
    if Nv != mask.n_video or Nt != mask.n_text:
        raise AssertionError(f"sequence ({Nv} video, {Nt} text) does not match the mask "
                             f"({mask.n_video} video, {mask.n_text} text)")
    qc, kc, vc = _prep(q, cdt), _prep(k, cdt), _prep(v, cdt)
    tq = _prep(text_q, cdt) if Nt > 0 else None
    tk = _prep(text_k, cdt) if Nt > 0 else None
    tv = _prep(text_v, cdt) if Nt > 0 else None
    o = out if (out is not None and out.dtype == cdt) else torch.empty(B, Nv, H, D, dtype=cdt, device=q.device)
    to = None
    if tq is not None:
        to = text_out if (text_out is not None and text_out.dtype == cdt) else \
            torch.empty(B, Nt, H, D, dtype=cdt, device=q.device)
    lse = tlse = None
    if return_lse:
        lse = torch.empty(B, H, Nv, dtype=torch.float32, device=q.device)
        if tq is not None:
            tlse = torch.empty(B, H, Nt, dtype=torch.float32, device=q.device)
    sc_c = None
    if fp8:
        # E4M3 copies with per-tile scales; V's tile scales share one per-head reference.
        vref = torch.zeros(B, Hkv, dtype=torch.float32, device=q.device)
        qc, qs = quantize_e4m3(qc)
        kc, ks = quantize_e4m3(kc)
        vc, vs = quantize_e4m3(vc, vref)
        tqs = tks = tvs = None
        if tk is not None:
            tk, tks = quantize_e4m3(tk)
            tv, tvs = quantize_e4m3(tv, vref)
        if tq is not None:
            tq, tqs = quantize_e4m3(tq)
        keep = (qs, ks, vs, tqs, tks, tvs, vref)
        sc_c = N.LvsaFp8Scales(*[t.data_ptr() if t is not None else None for t in keep])
    args = N.LvsaAttnArgs(
        _tview(qc), _tview(kc), _tview(vc), _tview(o), _tview(tq), _tview(tk), _tview(tv), _tview(to),
        lse.data_ptr() if lse is not None else None, tlse.data_ptr() if tlse is not None else None,
        B, Nv, Nt, H, Hkv, D, _DTYPES[cdt], float(scale) if scale else 0.0,
        mask.total_frames, mask.num_patches, mask.frame_words, mask.block_q, mask.block_k,
        mask.n_q_video_tiles, mask.n_q_tiles, mask.n_k_video_tiles,
        mask.frame_bits.data_ptr(), mask.tile_indptr.data_ptr(), mask.tile_indices.data_ptr(),
        mask.tile_flags.data_ptr(), error_word(q.device).data_ptr(),
        getattr(mask, "token_offset", 0),
        int(q_tiles[0]) if q_tiles is not None else getattr(mask, "first_q_tile", 0),
        int(q_tiles[1]) if q_tiles is not None else 0, int(wait_timeout_us), int(inject_fault),
        n_kv if n_kv != Nv else 0)
    with torch.cuda.device(q.device), nvtx_range("lvsa_attn_fwd_fp8" if fp8 else "lvsa_attn_fwd"):
        if fp8:
            st = N.load().lvsa_attn_fwd_fp8(ctypes.byref(args), ctypes.byref(sc_c), _stream_ptr(q.device))
        else:
            st = N.load().lvsa_attn_fwd(ctypes.byref(args), _stream_ptr(q.device))
    N.check(st, "lvsa_attn_fwd_fp8" if fp8 else "lvsa_attn_fwd")
    if cdt != in_dtype:
        o = o.to(in_dtype)
        to = to.to(in_dtype) if to is not None else None
    if out is not None and o is not out:
        out.copy_(o)
        o = out
    if text_out is not None and to is not None and to is not text_out:
        text_out.copy_(to)
        to = text_out
    if return_lse:
        return o, to, lse, tlse
    return o, to


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


def copy_segments(segments: Sequence[Tuple[torch.Tensor, torch.Tensor]]) -> None:
    """dst.copy_(src) for every (src, dst) pair of [B, N, H, D] views, in one
    launch of the batched strided copy kernel (CUDA tensors; strides and
    pointers multiples of 16 bytes).  CPU tensors (the gloo test ranks) are
    copied by torch."""
    segs = [(s, d) for s, d in segments if s.numel()]
    if not segs:
        return
    if not segs[0][0].is_cuda:
        for s, d in segs:
            d.copy_(s)
        return
    dev = segs[0][0].device
    es = segs[0][0].element_size()
    D = segs[0][0].shape[-1]
    lib = N.load()
    for i in range(0, len(segs), N.LVSA_MAX_COPY_SEGMENTS):
        chunk = segs[i:i + N.LVSA_MAX_COPY_SEGMENTS]
        arr = (N.LvsaCopySegment * len(chunk))()
        for j, (s, d) in enumerate(chunk):
            if s.shape != d.shape or s.dim() != 4 or s.stride(-1) != 1 or d.stride(-1) != 1 \
                    or s.shape[-1] != D or s.dtype != d.dtype:
                raise ValueError("copy_segments: matching [B, N, H, D] views with a contiguous last dim")
            arr[j] = N.LvsaCopySegment(s.data_ptr(), d.data_ptr(),
                                       s.stride(0) * es, s.stride(1) * es, s.stride(2) * es,
                                       d.stride(0) * es, d.stride(1) * es, d.stride(2) * es,
                                       s.shape[0], s.shape[1], s.shape[2])
        with torch.cuda.device(dev):
            st = lib.lvsa_copy_segments(arr, len(chunk), D * es, _stream_ptr(dev))
        N.check(st, "lvsa_copy_segments")
