"""Opt-in run-time diagnostics (the reference's env-gated logs and this
package's own counters).

* ``LVSA_MEM_LOG=1``: at every denoising-step boundary print
  ``[LVSA-MEM] step=N cuda=D alloc=..GB reserved=..GB peak=..GB``
  (lvsa/device.py:77-101, printed as lvsa-vllm-omni/lvsa_vllm_omni/
  attention_impl.py:105-116 does).
* ``LVSA_STEP_TIME_LOG=1``: at every step boundary print the wall time of the
  step that just completed, ``[LVSA-TIME] step=N dt=..s`` (attention_impl.py:
  118-128).
* ``LVSA_NVTX=1``: NVTX ranges around the mask build and every attention
  launch (``lvsa_build_mask``, ``lvsa_attn_fwd``), for Nsight timelines.
* ``lvsa_stats(mask, heads, head_dim)``: active tiles, density and useful
  FLOPs of one launch over a mask (one synchronising read of its counters).
"""

from __future__ import annotations

import contextlib
import os
import time
from typing import Dict, Optional, Tuple

import torch


def memory_stats() -> Optional[Tuple[str, int, float, float, float]]:
    """(kind, device, allocated GB, reserved GB, peak allocated GB) of the
    current CUDA device, or None without CUDA (lvsa/device.py:77-101)."""
    if not torch.cuda.is_available():
        return None
    dev = torch.cuda.current_device()
    return ("cuda", dev, torch.cuda.memory_allocated(dev) / 1e9, torch.cuda.memory_reserved(dev) / 1e9,
            torch.cuda.max_memory_allocated(dev) / 1e9)


class StepLogger:
    """Prints the env-gated per-step logs when a step counter advances."""

    def __init__(self) -> None:
        self._last_time: Optional[float] = None

    def step_boundary(self, step: int) -> None:
        """``step`` is the step that begins now."""
        if os.environ.get("LVSA_MEM_LOG", "0") == "1":
            st = memory_stats()
            if st is not None:
                kind, dev, alloc, reserved, peak = st
                print(f"[LVSA-MEM] step={step} {kind}={dev} alloc={alloc:.2f}GB reserved={reserved:.2f}GB "
                      f"peak={peak:.2f}GB", flush=True)
        if os.environ.get("LVSA_STEP_TIME_LOG", "0") == "1":
            now = time.perf_counter()
            if self._last_time is not None:
                print(f"[LVSA-TIME] step={step - 1} dt={now - self._last_time:.3f}s", flush=True)
            self._last_time = now

    def reset(self) -> None:
        self._last_time = None


def nvtx_range(name: str):
    """An NVTX range when ``LVSA_NVTX=1`` (a no-op context otherwise)."""
    if os.environ.get("LVSA_NVTX", "0") == "1" and torch.cuda.is_available():
        return torch.cuda.nvtx.range(name)
    return contextlib.nullcontext()


def lvsa_stats(mask, heads: int, head_dim: int, batch: int = 1) -> Dict[str, float]:
    """Work of one attention launch over ``mask`` (a BlockMask): active
    128 x 128 tiles, their share of the dense tile grid, and useful FLOPs
    (4 x head_dim per attended query-key pair over the active tiles at their
    full area; the clipped count is ``sparse_attention.tile_flop_counts``)."""
    nnz = int(mask.counters[0].item())
    dense = mask.n_q_tiles * mask.n_k_tiles
    flops = 4.0 * head_dim * mask.block_q * mask.block_k * nnz * heads * batch
    return {"tiles": nnz, "dense_tiles": dense, "density": nnz / dense if dense else 0.0,
            "tile_flops": flops, "q_tiles": mask.n_q_tiles, "k_tiles": mask.n_k_tiles}
