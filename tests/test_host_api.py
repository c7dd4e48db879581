"""Host side of the drop-in (no GPU): the mirrored LVSAMetadata and pattern
helpers against the reference goldens, the C ABI library's exports, and the
reference's error conventions."""

import ctypes
import json
import os
import re
import subprocess

import numpy as np
import pytest
import torch

import longvideosparseattention_b200.sparse_attention as SA
from oracle import lvsa_oracle as O
from tests.conftest import GOLDEN, ROOT

PATS = np.load(os.path.join(GOLDEN, "patterns.npz"))
with open(os.path.join(GOLDEN, "patterns.json")) as fh:
    META = json.load(fh)


@pytest.mark.parametrize("name", sorted(META))
def test_metadata_build_matches_reference(name):
    c = META[name]
    m = SA.LVSAMetadata.build(c["T"], c["P"], c["W"], c["n_first"], c["kfi"], c["rank"], c["world"],
                              expand_window=c["expand"], keyframe_offset=c["offset"],
                              boundary_guards=c["guards"] or None)
    assert m.global_indices == PATS[f"{name}.global_indices"].tolist()
    assert m.global_frame_mask.dtype == torch.int8 and m.window_bounds.dtype == torch.int32
    np.testing.assert_array_equal(m.global_frame_mask.numpy(), PATS[f"{name}.global_frame_mask"])
    np.testing.assert_array_equal(m.window_bounds.numpy(), PATS[f"{name}.window_bounds"])
    np.testing.assert_array_equal(m.attended_indices.numpy(), PATS[f"{name}.attended_indices"])
    np.testing.assert_array_equal(m.fi_indptr.numpy(), PATS[f"{name}.fi_indptr"])
    np.testing.assert_array_equal(m.fi_indices.numpy(), PATS[f"{name}.fi_indices"])
    np.testing.assert_array_equal(np.asarray(m.local_frames), PATS[f"{name}.local_frames"])
    wc = [(f, s, e) for f, parts in sorted(m.window_ctx.items()) for s, e in parts]
    np.testing.assert_array_equal(np.asarray(wc, dtype=np.int64).reshape(-1, 3), PATS[f"{name}.window_ctx"])
    assert (m.fi_MB, m.fi_compact_n, m.attended_C, m.local_seq) == (
        c["fi_MB"], c["fi_compact_n"], c["attended_C"], c["local_seq"])


def test_metadata_copy_indices_match_reference_semantics():
    # global_src/dst and local_src/dst as the reference's token loops (:419-439)
    m = SA.LVSAMetadata.build(20, 10, 2, 1, 5, 1, 2, keyframe_offset=1)
    P, gts = 10, m.global_token_start
    gs = [gi * P + t for gi, _ in enumerate(m.global_indices) for t in range(P)]
    gd = [gf * P + t for gf in m.global_indices for t in range(P)]
    assert m.global_src_idx.tolist() == gs and m.global_dst_idx.tolist() == gd
    ls, ld = [], []
    for f in range(gts // P, (gts + m.local_seq - 1) // P + 1):
        if f in m.global_set:
            continue
        s, e = max(f * P, gts), min((f + 1) * P, gts + m.local_seq)
        ls += [s - gts + t for t in range(e - s)]
        ld += [s + t for t in range(e - s)]
    assert m.local_src_idx.tolist() == ls and m.local_dst_idx.tolist() == ld


def test_helpers_match_oracle_exhaustively():
    for T in range(1, 30):
        for W in range(0, 4):
            for kfi in (None, 1, 2, 5):
                for off in range(0, 6):
                    g = SA.compute_global_indices(T, 1, kfi, off)
                    assert g == O.compute_global_indices(T, 1, kfi, off)
                    gs = set(g)
                    for f in range(T):
                        for ex in (True, False):
                            assert SA.get_window_bounds(f, W, T, ex, gs, len(g)) == \
                                O.get_window_bounds(f, W, T, ex, gs, len(g))
        for W in range(0, 4):
            assert SA.compute_auto_kfi(T * 3, W, 1, 21) == O.compute_auto_kfi(T * 3, W, 1, 21)
            assert SA.compute_auto_kfi(T * 3, W, 2, 33, 0.7) == O.compute_auto_kfi(T * 3, W, 2, 33, 0.7)


def test_divisibility_assertion_like_reference():
    with pytest.raises(AssertionError, match="divisible"):
        SA.LVSAMetadata.build(21, 7, 1, 1, 4, 0, 2)


def test_flashinfer_backend_assertion_like_reference():
    m = SA.LVSAMetadata.build(4, 8, 1, 1, 2, 0, 1)
    x = torch.zeros(1, 32, 1, 64)
    with pytest.raises(AssertionError, match="FlashInfer backend requires"):
        SA.sparse_windowed_attention(x, x, x, x, x, m, backend="flashinfer")


def test_cpu_tensors_fail_loudly():
    m = SA.LVSAMetadata.build(4, 8, 1, 1, 2, 0, 1)
    x = torch.zeros(1, 32, 1, 64)
    with pytest.raises(RuntimeError):
        SA.lvsa_sdpa(x, x, x, x[:, :16], x[:, :16], m)


def test_tile_flop_counts_match_oracle_and_baseline():
    for (T, P, W, kfi, off, nt, H, D, BQ, want_tiles) in [
            (9, 1560, 1, 4, 3, 0, 12, 128, 128, 964.5), (81, 1560, 2, 4, 0, 0, 12, 128, 128, 33103),
            (49, 1590, 2, 4, 0, 256, 16, 128, 128, 19483)]:
        m = SA.LVSAMetadata.build(T, P, W, 1, kfi, 0, 1, keyframe_offset=off)
        tiles, exact = SA.tile_flop_counts(m, nt, H, D, BQ, 128)
        fp = O.frame_pattern(T, P, W, 1, kfi, off)
        assert (tiles, exact) == O.flop_counts(fp["attended"], T, P, T * P, nt, H, D, BQ, 128)
        assert round(tiles / 1e9, 1 if want_tiles < 1000 else 0) == want_tiles


# ---------------------------------------------------------------- C ABI
def _header_functions():
    with open(os.path.join(ROOT, "include", "lvsa_b200.h")) as fh:
        src = fh.read()
    return set(re.findall(r"^\s*(?:int|const char\*)\s+(lvsa_\w+)\s*\(", src, re.M))


def test_library_exports_every_header_symbol():
    from longvideosparseattention_b200 import _native
    lib = _native.load()
    declared = _header_functions()
    assert declared == set(_native.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name
    nm = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True)
    exported = set(re.findall(r" T (lvsa_\w+)", nm.stdout))
    assert declared <= exported
    assert lib.lvsa_abi_version() == 102
    assert lib.lvsa_status_str(0) == b"ok"


def test_struct_layouts_match_header():
    """ctypes mirrors vs the C structs, measured by compiling a probe with gcc."""
    from longvideosparseattention_b200 import _native as N
    probe = r'''
#include <stdio.h>
#include <stddef.h>
#include "lvsa_b200.h"
int main(void){
 printf("%zu %zu %zu %zu %zu\n", sizeof(LvsaPattern), sizeof(LvsaMaskLayout), sizeof(LvsaMaskBuffers),
        sizeof(LvsaTensor), sizeof(LvsaAttnArgs));
 printf("%zu %zu %zu %zu %zu %zu\n", offsetof(LvsaAttnArgs, scale), offsetof(LvsaAttnArgs, frame_bits),
        offsetof(LvsaAttnArgs, error_word), offsetof(LvsaAttnArgs, end_q_tile), sizeof(LvsaCopySegment),
        offsetof(LvsaAttnArgs, inject_fault));
 return 0;}
'''
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "p.c")
        with open(c, "w") as fh:
            fh.write(probe)
        exe = os.path.join(d, "p")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    got = [int(x) for x in out]
    want = [ctypes.sizeof(N.LvsaPattern), ctypes.sizeof(N.LvsaMaskLayout),
            ctypes.sizeof(N.LvsaMaskBuffers), ctypes.sizeof(N.LvsaTensor), ctypes.sizeof(N.LvsaAttnArgs),
            N.LvsaAttnArgs.scale.offset, N.LvsaAttnArgs.frame_bits.offset, N.LvsaAttnArgs.error_word.offset,
            N.LvsaAttnArgs.end_q_tile.offset, ctypes.sizeof(N.LvsaCopySegment),
            N.LvsaAttnArgs.inject_fault.offset]
    assert got == want


def test_mask_layout_host_call_and_errors():
    from longvideosparseattention_b200 import mask_layout
    from longvideosparseattention_b200 import _native as N
    _, lay, _ = mask_layout(81, 1560, 2, 1, 4, 0, True, 0, 128, 128)
    assert (lay.n_video, lay.n_q_video_tiles, lay.n_k_video_tiles, lay.frame_words) == (126360, 988, 988, 3)
    fp = O.frame_pattern(81, 1560, 2, 1, 4, 0)
    _, idx, _, _, _ = O.tile_csr(fp["attended"], 81, 1560, 126360)
    assert lay.max_nnz >= len(idx)
    with pytest.raises(AssertionError):
        mask_layout(0, 1560, 2, 1, 4)
    with pytest.raises(N.LvsaError):
        mask_layout(9, 16, 1, 1, 4, block_q=100)
    with pytest.raises(AssertionError):
        mask_layout(N.LVSA_MAX_FRAMES + 1, 4, 1, 1, 4)


def test_noalloc_entry_rejects_oversize_before_any_cuda_call():
    """The fixed-scratch FP8 entry checks its arguments, geometry and limit before touching CUDA, so
    this runs without a GPU; the pointers are never dereferenced."""
    import ctypes
    from longvideosparseattention_b200 import _native as N
    lib = N.load()
    fake = N.LvsaTensor(16, 0, 0, 0)
    a = N.LvsaAttnArgs()
    a.q = a.k = a.v = a.o = fake
    a.batch, a.n_video, a.n_text, a.heads, a.kv_heads, a.head_dim, a.dtype = 1, 126360, 0, 12, 12, 128, 0
    a.total_frames, a.num_patches, a.frame_words, a.block_q, a.block_k = 81, 1560, 3, 128, 128
    a.n_q_video_tiles = a.n_q_tiles = a.n_k_video_tiles = 988
    a.frame_bits = a.tile_indptr = a.tile_indices = a.tile_flags = 16
    # E4M3 q, k and v alone: 3 x 126360 x 12 x 128 bytes = 582 MB > 96 MiB
    assert lib.lvsa_attn_fwd_fp8_noalloc(ctypes.byref(a), None) == N.LVSA_ERR_CAPACITY
    a.head_dim = 64
    assert lib.lvsa_attn_fwd_fp8_noalloc(ctypes.byref(a), None) == N.LVSA_ERR_UNSUPPORTED
    assert lib.lvsa_attn_fwd_fp8_noalloc(None, None) == N.LVSA_ERR_INVALID_ARG
    a.head_dim = 128
    a.n_q_video_tiles = 987           # geometry checked before capacity and before any launch
    assert lib.lvsa_attn_fwd_fp8_noalloc(ctypes.byref(a), None) == N.LVSA_ERR_GEOMETRY
