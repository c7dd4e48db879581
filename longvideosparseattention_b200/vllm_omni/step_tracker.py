"""Denoising-step and frame-geometry state for the plugin (interface of
lvsa-vllm-omni/lvsa_vllm_omni/step_tracker.py:1-155).

``forward_cuda`` does not see the step index or the frame count, so they are
kept per thread: set explicitly (``set_step``, ``set_total_latent_frames``,
``set_num_patches``) by a serving script or a hook, or inferred by counting
self-attention calls (``BlockCountStepTracker``: one denoising step is one
call per transformer block)."""

import threading
from typing import Optional

from ..observability import StepLogger

_state = threading.local()
_logger = StepLogger()
_global_tracker: Optional["BlockCountStepTracker"] = None


def set_step(step_idx: int) -> None:
    _state.step = int(step_idx)


def get_step() -> int:
    return getattr(_state, "step", 0)


def set_total_latent_frames(n: int) -> None:
    _state.total_latent_frames = int(n)


def get_total_latent_frames() -> Optional[int]:
    return getattr(_state, "total_latent_frames", None)


def set_num_patches(p: int) -> None:
    _state.num_patches = int(p)


def get_num_patches() -> Optional[int]:
    return getattr(_state, "num_patches", None)


def reset() -> None:
    """Clear the per-thread state, the shared tracker and the attention
    implementation's call counter (so calibrations do not leak between
    generations)."""
    global _global_tracker
    for attr in ("step", "total_latent_frames", "num_patches"):
        if hasattr(_state, attr):
            delattr(_state, attr)
    _global_tracker = None
    try:
        from . import attention_impl
        attention_impl._reset_step_counter()
    except ImportError:
        pass


class BlockCountStepTracker:
    """Step index from the number of self-attention calls: after calibration
    (``set_n_blocks`` or ``mark_step_boundary`` at the end of the first step)
    the step advances every ``n_blocks`` calls."""

    def __init__(self) -> None:
        self._call_count = 0
        self._n_blocks: Optional[int] = None
        self._step = 0
        self._calibrated = False

    def set_n_blocks(self, n: int) -> None:
        self._n_blocks = int(n)
        self._calibrated = True

    def tick(self) -> int:
        """One self-attention call; returns the step it belongs to."""
        step = self._step
        self._call_count += 1
        if self._calibrated and self._n_blocks is not None and self._call_count >= self._n_blocks:
            self._call_count = 0
            self._step += 1
            _logger.step_boundary(self._step)   # LVSA_MEM_LOG / LVSA_STEP_TIME_LOG
        _state.step = step
        return step

    def mark_step_boundary(self) -> None:
        if not self._calibrated:
            self._n_blocks = self._call_count
            self._calibrated = True
            self._call_count = 0
            self._step = 1
            _logger.step_boundary(1)

    @property
    def current_step(self) -> int:
        return self._step

    @property
    def n_blocks(self) -> Optional[int]:
        return self._n_blocks

    def reset(self) -> None:
        self.__init__()


def get_global_tracker() -> BlockCountStepTracker:
    global _global_tracker
    if _global_tracker is None:
        _global_tracker = BlockCountStepTracker()
    return _global_tracker


def tick_self_attention() -> int:
    """Record one self-attention call on the shared tracker; returns the step."""
    return get_global_tracker().tick()
