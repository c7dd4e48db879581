"""Denoising-step counter shared by the attention instances (interface of
lvsa-vllm-omni/lvsa_vllm_omni/step_tracker.py): the pipeline (or a hook)
calls ``set_step``; attention instances read ``get_step`` to rotate keyframes."""

_STEP = 0


def set_step(step: int) -> None:
    global _STEP
    _STEP = int(step)


def get_step() -> int:
    return _STEP


def reset() -> None:
    set_step(0)
