"""ctypes binding of the C ABI in ``include/lvsa_b200.h``.

The structures below mirror the header field for field.  Loading fails loudly
(``RuntimeError``) when the in-tree ``liblvsa_b200.so`` is missing: there is no
CPU or library fallback for the attention path.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "liblvsa_b200.so")

LVSA_OK = 0
LVSA_ERR_INVALID_ARG = 1
LVSA_ERR_GEOMETRY = 2
LVSA_ERR_UNSUPPORTED = 3
LVSA_ERR_ALIGNMENT = 4
LVSA_ERR_CAPACITY = 5
LVSA_ERR_CUDA = 6
LVSA_ERR_DEVICE_TIMEOUT = 7
LVSA_DTYPE_BF16 = 0
LVSA_DTYPE_F16 = 1
LVSA_MAX_FRAMES = 2048

EXPORTED_SYMBOLS = ("lvsa_mask_layout", "lvsa_build_mask", "lvsa_attn_fwd", "lvsa_quantize_e4m3",
                    "lvsa_attn_fwd_fp8", "lvsa_attn_fwd_fp8_noalloc", "lvsa_qk_prologue", "lvsa_copy_segments", "lvsa_out_proj", "lvsa_status_str",
                    "lvsa_abi_version")
LVSA_DTYPE_E4M3 = 2
LVSA_DTYPE_F32 = 3
LVSA_NORM_NONE, LVSA_NORM_RMS_ROW, LVSA_NORM_RMS_HEAD, LVSA_NORM_LAYER_HEAD = 0, 1, 2, 3

_i32, _i64, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p


class LvsaPattern(ctypes.Structure):
    _fields_ = [("total_frames", _i32), ("num_patches", _i32), ("window_size", _i32),
                ("n_first_frames", _i32), ("key_frame_interval", _i32), ("keyframe_offset", _i32),
                ("expand_window", _i32), ("n_text", _i32), ("block_q", _i32), ("block_k", _i32),
                ("n_guards", _i32), ("guards", ctypes.POINTER(_i32)), ("device_step", _vp)]


class LvsaMaskLayout(ctypes.Structure):
    _fields_ = [("n_video", _i32), ("n_q_video_tiles", _i32), ("n_q_tiles", _i32),
                ("n_k_video_tiles", _i32), ("n_k_tiles", _i32), ("frame_words", _i32),
                ("max_nnz", _i64)]


class LvsaMaskBuffers(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("global_frame_mask", "window_bounds", "frame_bits",
                                   "attended_indices", "frame_indptr", "frame_indices",
                                   "tile_indptr", "tile_indices", "tile_flags", "counters")]


class LvsaTensor(ctypes.Structure):
    _fields_ = [("ptr", _vp), ("stride_b", _i64), ("stride_t", _i64), ("stride_h", _i64)]


class LvsaAttnArgs(ctypes.Structure):
    _fields_ = [("q", LvsaTensor), ("k", LvsaTensor), ("v", LvsaTensor), ("o", LvsaTensor),
                ("text_q", LvsaTensor), ("text_k", LvsaTensor), ("text_v", LvsaTensor),
                ("text_o", LvsaTensor), ("lse", _vp), ("text_lse", _vp),
                ("batch", _i32), ("n_video", _i32), ("n_text", _i32), ("heads", _i32),
                ("kv_heads", _i32), ("head_dim", _i32), ("dtype", _i32), ("scale", ctypes.c_float),
                ("total_frames", _i32), ("num_patches", _i32), ("frame_words", _i32),
                ("block_q", _i32), ("block_k", _i32), ("n_q_video_tiles", _i32),
                ("n_q_tiles", _i32), ("n_k_video_tiles", _i32),
                ("frame_bits", _vp), ("tile_indptr", _vp), ("tile_indices", _vp),
                ("tile_flags", _vp), ("error_word", _vp), ("token_offset", _i32), ("first_q_tile", _i32),
                ("end_q_tile", _i32), ("wait_timeout_us", _i32), ("inject_fault", _i32),
                ("n_kv_video", _i32)]


LVSA_MAX_COPY_SEGMENTS = 64


class LvsaCopySegment(ctypes.Structure):
    _fields_ = [("src", _vp), ("dst", _vp), ("src_sb", _i64), ("src_st", _i64), ("src_sh", _i64),
                ("dst_sb", _i64), ("dst_st", _i64), ("dst_sh", _i64), ("batch", _i32), ("rows", _i32),
                ("heads", _i32)]


class LvsaOutProjArgs(ctypes.Structure):
    _fields_ = [("a", _vp), ("weight", _vp), ("bias", _vp), ("out", _vp), ("lda", _i64), ("ldw", _i64),
                ("ldo", _i64), ("m", _i32), ("n", _i32), ("k", _i32), ("dtype", _i32), ("error_word", _vp)]


class LvsaQkPrologue(ctypes.Structure):
    _fields_ = [("x", LvsaTensor), ("dtype", _i32), ("batch", _i32), ("seq", _i32), ("heads", _i32),
                ("head_dim", _i32), ("norm", _i32), ("weight_dtype", _i32), ("weight", _vp), ("bias", _vp),
                ("eps", ctypes.c_float), ("cos", _vp), ("sin", _vp), ("rope_stride_b", _i64),
                ("rope_offset", _i32)]


class LvsaFp8Scales(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("q", "k", "v", "text_q", "text_k", "text_v", "v_ref")]


_lib = None
_lock = threading.Lock()


class LvsaError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_str(status)} (status {status})")


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the native library; raise if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"LVSA native library not found at {path}; build it with "
                "`python -m longvideosparseattention_b200.build` (nvcc, sm_100a). "
                "There is no CPU fallback.")
        lib = ctypes.CDLL(path)
        lib.lvsa_mask_layout.argtypes = [ctypes.POINTER(LvsaPattern), ctypes.POINTER(LvsaMaskLayout)]
        lib.lvsa_mask_layout.restype = ctypes.c_int
        lib.lvsa_build_mask.argtypes = [ctypes.POINTER(LvsaPattern), ctypes.POINTER(LvsaMaskBuffers), _vp]
        lib.lvsa_build_mask.restype = ctypes.c_int
        lib.lvsa_attn_fwd.argtypes = [ctypes.POINTER(LvsaAttnArgs), _vp]
        lib.lvsa_attn_fwd.restype = ctypes.c_int
        lib.lvsa_quantize_e4m3.argtypes = [ctypes.POINTER(LvsaTensor), _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                                           _vp, _vp]
        lib.lvsa_quantize_e4m3.restype = ctypes.c_int
        lib.lvsa_attn_fwd_fp8.argtypes = [ctypes.POINTER(LvsaAttnArgs), ctypes.POINTER(LvsaFp8Scales), _vp]
        lib.lvsa_attn_fwd_fp8.restype = ctypes.c_int
        lib.lvsa_attn_fwd_fp8_noalloc.argtypes = [ctypes.POINTER(LvsaAttnArgs), _vp]
        lib.lvsa_attn_fwd_fp8_noalloc.restype = ctypes.c_int
        lib.lvsa_qk_prologue.argtypes = [ctypes.POINTER(LvsaQkPrologue), _vp]
        lib.lvsa_qk_prologue.restype = ctypes.c_int
        lib.lvsa_out_proj.argtypes = [ctypes.POINTER(LvsaOutProjArgs), _vp]
        lib.lvsa_out_proj.restype = ctypes.c_int
        lib.lvsa_copy_segments.argtypes = [ctypes.POINTER(LvsaCopySegment), _i32, _i32, _vp]
        lib.lvsa_copy_segments.restype = ctypes.c_int
        lib.lvsa_status_str.argtypes = [ctypes.c_int]
        lib.lvsa_status_str.restype = ctypes.c_char_p
        lib.lvsa_abi_version.argtypes = []
        lib.lvsa_abi_version.restype = ctypes.c_int
        _lib = lib
        return lib


def status_str(status: int) -> str:
    try:
        return load().lvsa_status_str(int(status)).decode()
    except RuntimeError:
        return f"status {status}"


def check(status: int, where: str) -> None:
    if status != LVSA_OK:
        if status in (LVSA_ERR_GEOMETRY,):
            raise LvsaGeometryError(status, where)
        raise LvsaError(status, where)


class LvsaGeometryError(LvsaError, AssertionError):
    """Geometry errors are AssertionErrors, as in the reference's builder
    (lvsa/sparse_attention.py:360-362)."""
