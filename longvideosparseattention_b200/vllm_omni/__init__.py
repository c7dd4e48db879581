"""vLLM-Omni plugin surface (mirror of lvsa-vllm-omni/lvsa_vllm_omni/):
configuration, geometry detection, step tracking, the ``LVSA`` attention
backend and its ``LVSAAttentionImpl``.  vllm-omni itself is not required to
import these; registering them with vllm-omni is the caller's business."""

from .attention_impl import LVSAAttentionImpl  # noqa: F401
from .backend import LVSABackend  # noqa: F401
from .config import LVSAConfig, candidate_patches_per_frame  # noqa: F401
from .global_kv import build_global_kv  # noqa: F401
