"""FP8-E4M3 mode (per-tile Q/K/V scales, E4M3 P): its own, looser bound vs
the fp32 reference.  Bound: max-abs <= 6e-2, mean-abs <= 6e-3 on outputs of
unit-scale data (E4M3 keeps 3 mantissa bits: 2^-4 relative per element)."""

import numpy as np
import pytest
import torch

from oracle import lvsa_oracle as O
from tests.gpu_util import seeded, to_np

pytestmark = pytest.mark.gpu

FP8_MAX_ABS = 6e-2
FP8_MEAN_ABS = 6e-3


def test_quantize_e4m3_roundtrip():
    from longvideosparseattention_b200.block_sparse import quantize_e4m3
    x = seeded((2, 300, 3, 128), 1)
    vref = torch.zeros(2, 3, device="cuda")
    q8, sc = quantize_e4m3(x, vref)
    deq = q8.view(torch.float8_e4m3fn).float() * sc.repeat_interleave(128, dim=2)[:, :, :300].transpose(1, 2)[..., None]
    rel = ((deq - x.float()).abs() / x.float().abs().clamp_min(1e-3)).median().item()
    assert rel < 0.04
    amax = x.float().abs().view(2, 300, 3, 128).permute(0, 2, 1, 3)
    assert torch.allclose(vref, sc.max(dim=2).values)
    assert (q8.view(torch.float8_e4m3fn).float().abs().max() <= 448).item()


def _run(T, P, H, D, W, kfi, off, nt, seed, frames=None, heads=None, scale_v=1.0):
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask, check_device_errors
    N = T * P
    sc = 1.0 / np.sqrt(D)
    q, k = seeded((1, N, H, D), seed, scale=sc), seeded((1, N, H, D), seed + 1, scale=sc)
    v = seeded((1, N, H, D), seed + 2, scale=scale_v)
    tq = tk = tv = None
    if nt:
        tq, tk = seeded((1, nt, H, D), seed + 3, scale=sc), seeded((1, nt, H, D), seed + 4, scale=sc)
        tv = seeded((1, nt, H, D), seed + 5, scale=scale_v)
    m = build_block_mask(T, P, W, 1, kfi, off, True, nt, device="cuda")
    out, tout = block_sparse_attention(q, k, v, m, tq, tk, tv, fp8=True)
    torch.cuda.synchronize()
    check_device_errors(torch.device("cuda"))
    fp = O.frame_pattern(T, P, W, 1, kfi, off)
    want, twant = O.attention(to_np(q), to_np(k), to_np(v), fp, None if tq is None else to_np(tq),
                              None if tk is None else to_np(tk), None if tv is None else to_np(tv),
                              frames=frames, heads=heads)
    res = []
    for got, ref in ((to_np(out), want), (None if tout is None else to_np(tout), twant)):
        if got is None:
            continue
        sel = ~np.isnan(ref)
        d = np.abs(got[sel] - ref[sel])
        res.append((d.max(), d.mean()))
    return res


@pytest.mark.parametrize("case", [
    dict(T=9, P=150, H=2, W=1, kfi=4, off=3, nt=0),
    dict(T=7, P=200, H=3, W=2, kfi=3, off=1, nt=60),
])
def test_fp8_small_vs_oracle(case):
    for mx, mean in _run(case["T"], case["P"], case["H"], 128, case["W"], case["kfi"], case["off"], case["nt"], 11):
        print(f"fp8 small: max-abs {mx:.3e} mean-abs {mean:.3e}")
        assert mx <= FP8_MAX_ABS and mean <= FP8_MEAN_ABS


def test_fp8_cfg3_sampled():
    # BASELINE cfg3 geometry (121 frames x 1560), offset 3; sampled frames / heads.
    res = _run(121, 1560, 12, 128, 2, 4, 3, 0, 21, frames=[2, 60, 119], heads=[0, 11])
    for mx, mean in res:
        print(f"fp8 cfg3: max-abs {mx:.3e} mean-abs {mean:.3e}")
        assert mx <= FP8_MAX_ABS and mean <= FP8_MEAN_ABS
