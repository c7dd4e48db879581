"""Block-sparse (BSR) attention with FlashInfer's plan / run interface, on
the sm_100a kernel: the drop-in for the ``fi_wrapper`` the reference's
FlashInfer path plans and runs (lvsa/lvsa_processor.py:768-913,
lvsa/sparse_attention.py:709-742, lvsa-vllm-omni/lvsa_vllm_omni/
flashinfer_runner.py:58-198).

The reference plans ``flashinfer.BlockSparseAttentionWrapper`` with the
frame-level CSR of LVSAMetadata (``fi_indptr`` / ``fi_indices``; R = C = P,
one block per latent frame) over a padded query of M = MB x P tokens and a
compact K/V of N = compact_n x P tokens, then runs it per batch element and
merges a dense text term through the returned base-2 log-sum-exp.

``LvsaBlockSparseWrapper.plan`` takes the same arguments and turns the
block CSR into the kernel's inputs on the host, once: a bitset of allowed
key blocks per query block (the kernel's in-tile mask) and the 128 x 128
tile CSR with a flag on every tile that is not fully allowed.  ``run``
launches the kernel with the query and key lengths given separately
(``n_kv_video``) and returns the output and, on request, the LSE in base 2
as FlashInfer does.  Blocks must be square (R == C), as in every LVSA plan.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch

from .block_sparse import ATTN_BLOCK_K, ATTN_BLOCK_Q, block_sparse_attention

LN2 = math.log(2.0)


@dataclass
class BsrMask:
    """The fields ``block_sparse_attention`` reads, for a BSR plan."""
    total_frames: int
    num_patches: int
    frame_words: int
    n_video: int
    n_kv_video: int
    n_q_video_tiles: int
    n_q_tiles: int
    n_k_video_tiles: int
    frame_bits: torch.Tensor
    tile_indptr: torch.Tensor
    tile_indices: torch.Tensor
    tile_flags: torch.Tensor
    n_text: int = 0
    token_offset: int = 0
    first_q_tile: int = 0
    block_q: int = ATTN_BLOCK_Q
    block_k: int = ATTN_BLOCK_K


def bsr_tile_csr(indptr: np.ndarray, indices: np.ndarray, M: int, N: int, R: int
                 ) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray, int]:
    """Host expansion of a square-block CSR (block size R) over M query and N
    key tokens into (frame_bits [T, words] uint32, tile indptr, tile indices,
    tile flags, T) with 128 x 128 tiles; flag 1 = the tile holds a key that
    some query row of the tile may not attend (or keys past N)."""
    indptr = np.asarray(indptr, dtype=np.int64)
    indices = np.asarray(indices, dtype=np.int64)
    MB, NB = -(-M // R), -(-N // R)
    if len(indptr) != MB + 1:
        raise ValueError(f"indptr has {len(indptr)} entries, expected M/R + 1 = {MB + 1}")
    if len(indices) and (indices.min() < 0 or indices.max() >= NB):
        raise ValueError("block column index out of range")
    T = max(MB, NB)
    allow = np.zeros((MB, NB), dtype=bool)
    for r in range(MB):
        allow[r, indices[indptr[r]:indptr[r + 1]]] = True
    words = -(-T // 32)
    bits = np.zeros((T, words), dtype=np.uint32)
    for r in range(MB):
        for c in np.nonzero(allow[r])[0]:
            bits[r, c >> 5] |= np.uint32(1) << np.uint32(c & 31)
    BQ, BK = ATTN_BLOCK_Q, ATTN_BLOCK_K
    nqv, nkv = -(-M // BQ), -(-N // BK)
    kt = np.arange(nkv)
    kf_lo = (kt * BK) // R
    kf_hi = (np.minimum((kt + 1) * BK, N) - 1) // R
    width = kf_hi - kf_lo + 1
    partial = (kt + 1) * BK > N
    ip, ix, fl = [0], [], []
    for t in range(nqv):
        qf_lo, qf_hi = (t * BQ) // R, (min((t + 1) * BQ, M) - 1) // R
        rows = allow[qf_lo:qf_hi + 1]
        any_c = np.concatenate([[0], np.cumsum(rows.any(axis=0))])
        all_c = np.concatenate([[0], np.cumsum(rows.all(axis=0))])
        active = any_c[kf_hi + 1] - any_c[kf_lo] > 0
        full = (all_c[kf_hi + 1] - all_c[kf_lo] == width) & ~partial
        sel = np.nonzero(active)[0]
        ix.extend(sel.tolist())
        fl.extend((~full[sel]).astype(np.uint8).tolist())
        ip.append(len(ix))
    return (bits, np.asarray(ip, np.int32), np.asarray(ix, np.int32), np.asarray(fl, np.uint8), T)


class LvsaBlockSparseWrapper:
    """``flashinfer.BlockSparseAttentionWrapper`` interface on the sm_100a
    kernel.  ``workspace`` is accepted for signature compatibility and not
    used (the kernel needs no workspace)."""

    def __init__(self, workspace: Optional[torch.Tensor] = None, backend: str = "auto") -> None:
        self._mask: Optional[BsrMask] = None
        self._heads = self._kv_heads = self._head_dim = None
        self._scale: Optional[float] = None

    def plan(self, indptr, indices, M: int, N: int, R: int, C: int, num_qo_heads: int, num_kv_heads: int,
             head_dim: int, mask=None, causal: bool = False, sm_scale: Optional[float] = None,
             q_data_type=None, kv_data_type=None, o_data_type=None, **_unused) -> None:
        if R != C:
            raise NotImplementedError(f"square blocks only (R = C), got R={R} C={C}")
        if mask is not None or causal:
            raise NotImplementedError("element masks and causal plans are not part of LVSA")
        dev = indptr.device if isinstance(indptr, torch.Tensor) and indptr.is_cuda else torch.device("cuda")
        to_np = lambda x: x.detach().cpu().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)
        bits, ip, ix, fl, T = bsr_tile_csr(to_np(indptr), to_np(indices), int(M), int(N), int(R))
        t = lambda a, dt: torch.from_numpy(a if len(a) else np.zeros(1, a.dtype)).to(dev)
        self._mask = BsrMask(T, int(R), bits.shape[1], int(M), int(N), -(-int(M) // ATTN_BLOCK_Q),
                             -(-int(M) // ATTN_BLOCK_Q), -(-int(N) // ATTN_BLOCK_K),
                             torch.from_numpy(bits.view(np.int32)).to(dev), t(ip, None), t(ix, None),
                             t(fl, None))
        self._heads, self._kv_heads, self._head_dim = num_qo_heads, num_kv_heads, head_dim
        self._scale = sm_scale

    def run(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, return_lse: bool = False, **_unused):
        """q [M, H, D], k / v [N, Hkv, D] (or with a leading batch dim) ->
        out like q, and with ``return_lse`` the base-2 LSE [M, H]."""
        if self._mask is None:
            raise RuntimeError("plan() must be called before run()")
        batched = q.dim() == 4
        qb, kb, vb = (x if batched else x.unsqueeze(0) for x in (q, k, v))
        o, _, lse, _ = block_sparse_attention(qb, kb, vb, self._mask, scale=self._scale, return_lse=True)
        if not batched:
            o = o[0]
        if not return_lse:
            return o
        lse2 = (lse / LN2).transpose(-1, -2)            # [B, M, H] base 2
        return o, (lse2 if batched else lse2[0]).contiguous()
