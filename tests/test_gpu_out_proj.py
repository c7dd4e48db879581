"""The output projection on the hand-written tcgen05 GEMM (lvsa_out_proj)
against an fp32 torch reference of the same Linear, on the adapters' shapes
(Wan2.1-1.3B 12 x 128 -> 1536, HunyuanVideo 16 x 128 -> 2048, CogVideoX
48 x 64 -> 3072), ragged row counts, bias on and off, bf16 and fp16, and a
strided view of o; then attention + projection against the kernel output
projected by torch.  Tolerance: max-abs 2e-2 and mean-abs 2e-3 on outputs of
unit scale (the bf16 attention tolerance)."""

import pytest
import torch
import torch.nn.functional as F

from tests.gpu_util import assert_close, seeded, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,H,D,Nout,bias,dtype", [
    (1000, 12, 128, 1536, True, torch.bfloat16),
    (4097, 16, 128, 2048, False, torch.bfloat16),
    (777, 48, 64, 3072, True, torch.float16),
    (128, 2, 64, 96, True, torch.bfloat16),       # one tile, n not a multiple of 256
])
def test_out_proj_vs_torch_linear(M, H, D, Nout, bias, dtype):
    from longvideosparseattention_b200 import check_device_errors
    from longvideosparseattention_b200.out_proj import out_projection
    K = H * D
    o = seeded((1, M, H, D), 1, dtype)
    w = seeded((Nout, K), 2, dtype, scale=K ** -0.5)
    b = seeded((Nout,), 3, dtype) if bias else None
    y = out_projection(o, w, b)
    torch.cuda.synchronize()
    check_device_errors(o.device)
    want = F.linear(o.float().reshape(1, M, K), w.float(), None if b is None else b.float())
    assert y.shape == (1, M, Nout) and y.dtype == dtype
    assert_close(to_np(y), to_np(want), what="out_proj")


def test_out_proj_strided_rows():
    from longvideosparseattention_b200.out_proj import out_projection
    M, K, Nout = 300, 256, 512
    base = seeded((M, K + 64), 5)
    a = base[:, :K]                                   # row stride K + 64
    w = seeded((Nout, K), 6, scale=K ** -0.5)
    y = out_projection(a, w)
    torch.cuda.synchronize()
    assert_close(to_np(y), to_np(F.linear(a.float(), w.float())), what="strided")


def test_attention_then_projection():
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask
    from longvideosparseattention_b200.out_proj import attention_out_projection
    T, P, H, D, nt, dim = 9, 160, 4, 128, 40, 512
    m = build_block_mask(T, P, 1, 1, 3, 1, True, nt, device="cuda")
    q, k, v = (seeded((1, T * P, H, D), s, scale=D ** -0.5) for s in (1, 2, 3))
    tq, tk, tv = (seeded((1, nt, H, D), s, scale=D ** -0.5) for s in (4, 5, 6))
    w, tw = seeded((dim, H * D), 7, scale=(H * D) ** -0.5), seeded((dim, H * D), 8, scale=(H * D) ** -0.5)
    b = seeded((dim,), 9)
    y, ty = attention_out_projection(q, k, v, m, w, b, tq, tk, tv, tw, None)
    o, to = block_sparse_attention(q, k, v, m, tq, tk, tv)
    torch.cuda.synchronize()
    assert_close(to_np(y), to_np(F.linear(o.float().flatten(2), w.float(), b.float())), what="video")
    assert_close(to_np(ty), to_np(F.linear(to.float().flatten(2), tw.float())), what="text")


def test_out_proj_full_size_cfg2_vs_cublas():
    """cfg2 shape: 126 360 tokens x 1536 -> 1536, against torch's bf16 Linear."""
    from longvideosparseattention_b200.out_proj import out_projection
    o = seeded((1, 126360, 12, 128), 11)
    w = seeded((1536, 1536), 12, scale=1536 ** -0.5)
    b = seeded((1536,), 13)
    y = out_projection(o, w, b)
    ref = F.linear(o.flatten(2), w, b)
    torch.cuda.synchronize()
    d = (y.float() - ref.float()).abs()
    assert d.max().item() <= 3e-2 and d.mean().item() <= 2e-3, (d.max().item(), d.mean().item())
