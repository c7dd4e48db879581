"""lvsa_attn_fwd_fp8_noalloc: the FP8 attention entry point that allocates no
device memory.  It is for callers that cannot call cudaMalloc: serving
runtimes whose device memory is one fixed pool owned by their own allocator,
and hosts that bind the library from a language runtime with no CUDA
allocator.  The test calls it through the C ABI.

It runs the same quantiser and attention kernels as the allocating FP8 entry
(lvsa_attn_fwd_fp8, reached through block_sparse_attention(fp8=True)), only
with its scratch in the library's static array, so its outputs must equal
that entry's to the bit (torch.equal).  One case is also checked against the
fp32 oracle at the FP8 bound of tests/test_gpu_fp8.py.  Each case makes two
calls in a row with different inputs (V scaled up, then down), so anything
the first call leaves in the shared array, in particular the per-head V
reference, would show in the second.  Cases cover batch 2, grouped K/V heads,
text rows, and the sequence-shard arguments (token_offset, first_q_tile).
Calls over the array's capacity and calls with bad geometry must return
their status and launch nothing.

This file is collected last, so that a run stopping at the first failure
has run every other test before it; it also passes when run alone."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import lvsa_oracle as O
from tests.gpu_util import seeded, to_np

pytestmark = pytest.mark.gpu

FP8_MAX_ABS = 6e-2
FP8_MEAN_ABS = 6e-3
SCRATCH_BYTES = 96 * 2 ** 20   # LVSA_NOALLOC_SCRATCH_BYTES in include/lvsa_b200.h


def _args(q, k, v, mask, tq, tk, tv, o, to, lse, tlse):
    from longvideosparseattention_b200 import _native as N
    from longvideosparseattention_b200.block_sparse import _tview, error_word
    B, Nv, H, D = q.shape
    Hkv, Nt = k.shape[2], 0 if tk is None else tk.shape[1]
    return N.LvsaAttnArgs(
        _tview(q), _tview(k), _tview(v), _tview(o), _tview(tq), _tview(tk), _tview(tv), _tview(to),
        lse.data_ptr(), tlse.data_ptr() if tlse is not None else None,
        B, Nv, Nt, H, Hkv, D, 0, 0.0,
        mask.total_frames, mask.num_patches, mask.frame_words, mask.block_q, mask.block_k,
        mask.n_q_video_tiles, mask.n_q_tiles, mask.n_k_video_tiles,
        mask.frame_bits.data_ptr(), mask.tile_indptr.data_ptr(), mask.tile_indices.data_ptr(),
        mask.tile_flags.data_ptr(), error_word(q.device).data_ptr(),
        getattr(mask, "token_offset", 0), getattr(mask, "first_q_tile", 0))


def _raw_call(args, device):
    from longvideosparseattention_b200 import _native as N
    from longvideosparseattention_b200.block_sparse import _stream_ptr
    return N.load().lvsa_attn_fwd_fp8_noalloc(ctypes.byref(args), _stream_ptr(device))


def _noalloc_call(q, k, v, mask, tq, tk, tv, out=None):
    """Fill LvsaAttnArgs as lvsa_attn_fwd takes them and call the entry."""
    from longvideosparseattention_b200 import _native as N
    B, Nv, H, D = q.shape
    Nt = 0 if tk is None else tk.shape[1]
    o = out if out is not None else torch.empty_like(q)
    to = torch.empty(B, Nt, H, D, dtype=q.dtype, device=q.device) if tq is not None else None
    lse = torch.empty(B, H, Nv, dtype=torch.float32, device=q.device)
    tlse = torch.empty(B, H, Nt, dtype=torch.float32, device=q.device) if tq is not None else None
    N.check(_raw_call(_args(q, k, v, mask, tq, tk, tv, o, to, lse, tlse), q.device),
            "lvsa_attn_fwd_fp8_noalloc")
    return o, to, lse, tlse


def _inputs(B, N_, H, Hkv, nt, seed, v_scale, with_tq=True):
    sc = 128 ** -0.5
    q = seeded((B, N_, H, 128), seed, scale=sc)
    k = seeded((B, N_, Hkv, 128), seed + 1, scale=sc)
    v = seeded((B, N_, Hkv, 128), seed + 2, scale=v_scale)
    tq = tk = tv = None
    if nt:
        tq = seeded((B, nt, H, 128), seed + 3, scale=sc) if with_tq else None
        tk = seeded((B, nt, Hkv, 128), seed + 4, scale=sc)
        tv = seeded((B, nt, Hkv, 128), seed + 5, scale=v_scale)
    return q, k, v, tq, tk, tv


def _assert_equal(got, want, call, names=("out", "text_out", "lse", "text_lse")):
    for name, g, w in zip(names, got, want):
        if w is None:
            assert g is None, name
            continue
        if not torch.equal(g, w):
            d = (g.float() - w.float()).abs().max().item()
            raise AssertionError(f"call {call} {name}: differs from lvsa_attn_fwd_fp8 (max-abs {d:.3e})")


@pytest.mark.parametrize("case", [
    dict(B=1, T=9, P=150, H=2, Hkv=2, nt=0),
    dict(B=1, T=13, P=256, H=3, Hkv=3, nt=77),
    dict(B=1, T=6, P=130, H=4, Hkv=2, nt=130),   # grouped K/V heads
    dict(B=2, T=7, P=200, H=3, Hkv=3, nt=60),    # batch offsets of the scratch layout
])
def test_noalloc_equals_allocating_fp8_entry_two_calls(case):
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask, check_device_errors
    B, T, P, H, Hkv, nt = case["B"], case["T"], case["P"], case["H"], case["Hkv"], case["nt"]
    mask = build_block_mask(T, P, 1, 1, 4, 1, True, nt, device="cuda")
    for call, (seed, v_scale) in enumerate(((11, 4.0), (23, 0.25))):
        q, k, v, tq, tk, tv = _inputs(B, T * P, H, Hkv, nt, seed, v_scale)
        want = block_sparse_attention(q, k, v, mask, tq, tk, tv, return_lse=True, fp8=True)
        got = _noalloc_call(q, k, v, mask, tq, tk, tv)
        torch.cuda.synchronize()
        check_device_errors(torch.device("cuda"))
        _assert_equal(got, want, call)


def test_noalloc_vs_oracle():
    from longvideosparseattention_b200 import build_block_mask, check_device_errors
    T, P, H, W, kfi, off, nt = 9, 150, 2, 1, 4, 3, 60
    mask = build_block_mask(T, P, W, 1, kfi, off, True, nt, device="cuda")
    q, k, v, tq, tk, tv = _inputs(1, T * P, H, H, nt, 5, 1.0)
    out, tout, _, _ = _noalloc_call(q, k, v, mask, tq, tk, tv)
    torch.cuda.synchronize()
    check_device_errors(torch.device("cuda"))
    fp = O.frame_pattern(T, P, W, 1, kfi, off)
    want, twant = O.attention(to_np(q), to_np(k), to_np(v), fp, to_np(tq), to_np(tk), to_np(tv))
    for got, ref, what in ((to_np(out), want, "video"), (to_np(tout), twant, "text")):
        d = np.abs(got - ref)
        assert d.max() <= FP8_MAX_ABS and d.mean() <= FP8_MEAN_ABS, (what, d.max(), d.mean())


def test_noalloc_sequence_shard_two_calls():
    """Rank 1 of 2 under the reference's context parallelism: the video-row
    launch (token_offset > 0, dense [globals; text] segment) and the text-row
    launch (first_q_tile > 0)."""
    from longvideosparseattention_b200 import block_sparse_attention, check_device_errors
    from longvideosparseattention_b200.cp_mode import build_shard_pattern
    T, P, H, W, nt, world, rank = 8, 200, 2, 1, 70, 2, 1
    dev = torch.device("cuda")
    pat = build_shard_pattern(T, P, W, 1, 4, 2, rank, world, nt, device=dev)
    S_r = T * P // world
    G = len(pat.global_indices) * P
    assert pat.video.token_offset > 0 and pat.text.first_q_tile > 0
    for call, (seed, v_scale) in enumerate(((31, 4.0), (43, 0.25))):
        q, k, v, tq, tk, tv = _inputs(1, S_r, H, H, nt, seed, v_scale)
        kd = torch.cat([seeded((1, G, H, 128), seed + 6, scale=128 ** -0.5), tk], 1)
        vd = torch.cat([seeded((1, G, H, 128), seed + 7, scale=v_scale), tv], 1)
        want = block_sparse_attention(q, k, v, pat.video, None, kd, vd, return_lse=True, fp8=True)
        got = _noalloc_call(q, k, v, pat.video, None, kd, vd)
        # Text rows only: the video rows of `out` are not written.
        filler = torch.full_like(q, 7.0)
        want_t = block_sparse_attention(q, k, v, pat.text, tq, tk, tv, return_lse=True, fp8=True,
                                        out=filler.clone())
        got_t = _noalloc_call(q, k, v, pat.text, tq, tk, tv, out=filler.clone())
        torch.cuda.synchronize()
        check_device_errors(dev)
        _assert_equal(got[:1] + got[2:3], want[:1] + want[2:3], call, ("out", "lse"))
        _assert_equal(got_t[1:2] + got_t[3:], want_t[1:2] + want_t[3:], call, ("text_out", "text_lse"))
        assert torch.equal(got_t[0], filler)


def test_noalloc_rejects_before_launching():
    """Over capacity (E4M3 copies alone above the array's size) and bad
    geometry: the status comes back and the output is left untouched."""
    from longvideosparseattention_b200 import _native as N, build_block_mask
    dev = torch.device("cuda")
    T, P, H = 64, 1024, 5          # 3 x 64 Ki tokens x 5 heads x 128 B > 96 MiB
    mask = build_block_mask(T, P, 1, 1, 4, 0, True, 0, device=dev)
    assert 3 * T * P * H * 128 > SCRATCH_BYTES
    q, k, v, _, _, _ = _inputs(1, T * P, H, H, 0, 3, 1.0)
    o = torch.full_like(q, 3.0)
    lse = torch.full((1, H, T * P), 5.0, device=dev)
    st = _raw_call(_args(q, k, v, mask, None, None, None, o, None, lse, None), dev)
    assert st == N.LVSA_ERR_CAPACITY, N.load().lvsa_status_str(st)

    small = build_block_mask(9, 150, 1, 1, 4, 0, True, 0, device=dev)
    q, k, v, _, _, _ = _inputs(1, 9 * 150, 2, 2, 0, 4, 1.0)
    o2 = torch.full_like(q, 3.0)
    lse2 = torch.full((1, 2, 9 * 150), 5.0, device=dev)
    bad = _args(q, k, v, small, None, None, None, o2, None, lse2, None)
    bad.n_q_video_tiles += 1
    st = _raw_call(bad, dev)
    assert st == N.LVSA_ERR_GEOMETRY, N.load().lvsa_status_str(st)
    bad = _args(q, k, v, small, None, None, None, o2, None, lse2, None)
    bad.kv_heads = 3               # heads % kv_heads != 0
    assert _raw_call(bad, dev) == N.LVSA_ERR_INVALID_ARG
    torch.cuda.synchronize()
    assert (o == 3.0).all() and (lse == 5.0).all()
    assert (o2 == 3.0).all() and (lse2 == 5.0).all()
