"""The ``LVSA`` attention backend descriptor (interface of
lvsa-vllm-omni/lvsa_vllm_omni/backend.py:23-53)."""

from .attention_impl import LVSAAttentionImpl


class LVSABackend:
    accept_output_buffer: bool = False

    @staticmethod
    def get_name() -> str:
        return "LVSA"

    @staticmethod
    def get_impl_cls():
        return LVSAAttentionImpl

    @staticmethod
    def get_supported_head_sizes():
        return [64, 128]
