"""lvsa_attn_fwd_fp8_noalloc, the FP8 attention entry for callers that cannot
allocate device memory (fixed-pool serving runtimes, allocator-less host
bindings), called through the C ABI and checked against the allocating FP8
entry (lvsa_attn_fwd_fp8 via block_sparse_attention(fp8=True)).

Both run the same quantiser and attention kernels, so the outputs should
agree to the bit; the test asserts the FP8 tolerance of the other FP8 tests
(max-abs 6e-2, mean-abs 6e-3) and reports any difference.  Two calls in a
row with different inputs (V scaled up, then down) check that nothing left
in the shared scratch array, in particular the per-head V reference, leaks
into the next call.  This file is collected last so that a run stopping at
the first failure has run every other test first; it also passes alone."""

import ctypes

import pytest
import torch

from tests.gpu_util import seeded

pytestmark = pytest.mark.gpu

MAX_ABS = 6e-2
MEAN_ABS = 6e-3


def _noalloc_call(q, k, v, mask, tq, tk, tv):
    """Fill LvsaAttnArgs as lvsa_attn_fwd takes them and call the entry."""
    from longvideosparseattention_b200 import _native as N
    from longvideosparseattention_b200.block_sparse import _stream_ptr, _tview, error_word
    B, Nv, H, D = q.shape
    Hkv, Nt = k.shape[2], 0 if tk is None else tk.shape[1]
    o = torch.empty_like(q)
    to = torch.empty_like(tq) if tq is not None else None
    lse = torch.empty(B, H, Nv, dtype=torch.float32, device=q.device)
    tlse = torch.empty(B, H, Nt, dtype=torch.float32, device=q.device) if tq is not None else None
    args = N.LvsaAttnArgs(
        _tview(q), _tview(k), _tview(v), _tview(o), _tview(tq), _tview(tk), _tview(tv), _tview(to),
        lse.data_ptr(), tlse.data_ptr() if tlse is not None else None,
        B, Nv, Nt, H, Hkv, D, 0, 0.0,
        mask.total_frames, mask.num_patches, mask.frame_words, mask.block_q, mask.block_k,
        mask.n_q_video_tiles, mask.n_q_tiles, mask.n_k_video_tiles,
        mask.frame_bits.data_ptr(), mask.tile_indptr.data_ptr(), mask.tile_indices.data_ptr(),
        mask.tile_flags.data_ptr(), error_word(q.device).data_ptr())
    st = N.load().lvsa_attn_fwd_fp8_noalloc(ctypes.byref(args), _stream_ptr(q.device))
    N.check(st, "lvsa_attn_fwd_fp8_noalloc")
    return o, to, lse, tlse


@pytest.mark.parametrize("case", [
    dict(T=9, P=150, H=2, Hkv=2, nt=0),
    dict(T=13, P=256, H=3, Hkv=3, nt=77),
    dict(T=6, P=130, H=4, Hkv=2, nt=130),   # grouped K/V heads
])
def test_noalloc_matches_allocating_fp8_entry_two_calls(case):
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask, check_device_errors
    T, P, H, Hkv, nt = case["T"], case["P"], case["H"], case["Hkv"], case["nt"]
    N_ = T * P
    sc = 128 ** -0.5
    mask = build_block_mask(T, P, 1, 1, 4, 1, True, nt, device="cuda")
    for call, (seed, v_scale) in enumerate(((11, 4.0), (23, 0.25))):
        q = seeded((1, N_, H, 128), seed, scale=sc)
        k = seeded((1, N_, Hkv, 128), seed + 1, scale=sc)
        v = seeded((1, N_, Hkv, 128), seed + 2, scale=v_scale)
        tq = tk = tv = None
        if nt:
            tq = seeded((1, nt, H, 128), seed + 3, scale=sc)
            tk = seeded((1, nt, Hkv, 128), seed + 4, scale=sc)
            tv = seeded((1, nt, Hkv, 128), seed + 5, scale=v_scale)
        want = block_sparse_attention(q, k, v, mask, tq, tk, tv, return_lse=True, fp8=True)
        got = _noalloc_call(q, k, v, mask, tq, tk, tv)
        torch.cuda.synchronize()
        check_device_errors(torch.device("cuda"))
        for name, g, w in zip(("out", "text_out", "lse", "text_lse"), got, want):
            if w is None:
                assert g is None, name
                continue
            d = (g.float() - w.float()).abs()
            # outputs are relative to V's magnitude; the LSE is not
            s = v_scale if name in ("out", "text_out") else 1.0
            assert d.max().item() <= MAX_ABS * s, f"call {call} {name}: max {d.max().item()}"
            assert d.mean().item() <= MEAN_ABS * s, f"call {call} {name}: mean {d.mean().item()}"
