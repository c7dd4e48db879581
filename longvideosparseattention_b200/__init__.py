"""B200-native (sm_100a) LVSA block-sparse attention.

The hot path -- GPU mask builder and tcgen05/TMEM block-sparse attention --
lives in the in-tree ``liblvsa_b200.so`` (C ABI: ``include/lvsa_b200.h``);
the Python modules mirror the reference LVSA interface on top of it.
"""

__version__ = "0.1.0"

from .block_sparse import (BlockMask, block_sparse_attention, build_block_mask,  # noqa: F401
                           check_device_errors, mask_layout)
from .observability import lvsa_stats, memory_stats  # noqa: F401,E402
