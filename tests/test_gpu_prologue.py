"""QK prologue kernel (norm + rotary embedding in one pass) vs the fp32
oracle restatement.  Bound: |got - ref| <= 1e-2 * |ref| + 1e-2 (bf16/fp16
output, one rounding), checked elementwise."""

import math

import pytest
import torch

from oracle import lvsa_oracle as O

pytestmark = pytest.mark.gpu


def _tables(S, D, seed, batch=None):
    g = torch.Generator().manual_seed(seed)
    shape = (S, D // 2) if batch is None else (batch, S, D // 2)
    ang = torch.rand(*shape, generator=g) * 2 * math.pi
    return torch.cos(ang).cuda(), torch.sin(ang).cuda()


def _check(got, ref):
    d = (got.float().cpu() - ref).abs()
    bound = 1e-2 * ref.abs() + 1e-2
    assert bool((d <= bound).all()), f"max excess {(d - bound).max().item()}"


@pytest.mark.parametrize("case", [
    dict(B=1, S=300, H=12, D=128, norm="rms_row", wdt=torch.bfloat16, rope=True),      # Wan 1.3B
    dict(B=1, S=257, H=16, D=128, norm="rms_head", wdt=torch.bfloat16, rope=True),     # HunyuanVideo
    dict(B=2, S=133, H=48, D=64, norm="layer_head", wdt=torch.float32, rope=True),     # CogVideoX-5B
    dict(B=1, S=96, H=40, D=128, norm="rms_row", wdt=torch.float32, rope=True),        # Wan 14B (5120 / row)
    dict(B=1, S=77, H=12, D=128, norm=None, wdt=None, rope=True),                      # rotation only
    dict(B=1, S=64, H=16, D=128, norm="rms_head", wdt=torch.bfloat16, rope=False),     # text tokens
    dict(B=1, S=50, H=48, D=64, norm="layer_head", wdt=torch.bfloat16, rope=False, dtype=torch.float16),
])
def test_prologue_matches_oracle(case):
    from longvideosparseattention_b200.prologue import qk_norm_rope
    B, S, H, D = case["B"], case["S"], case["H"], case["D"]
    dtype = case.get("dtype", torch.bfloat16)
    g = torch.Generator().manual_seed(S * 7 + H)
    x = (torch.randn(B, S, H, D, generator=g) * 2.0).to(dtype).cuda()
    w = b = None
    if case["norm"] == "rms_row":
        w = (1 + 0.3 * torch.randn(H * D, generator=g)).to(case["wdt"]).cuda()
    elif case["norm"] is not None:
        w = (1 + 0.3 * torch.randn(D, generator=g)).to(case["wdt"]).cuda()
        if case["norm"] == "layer_head":
            b = (0.2 * torch.randn(D, generator=g)).to(case["wdt"]).cuda()
    cs = sn = None
    if case["rope"]:
        cs, sn = _tables(S, D, S, batch=B if B > 1 else None)
    ref = O.norm_rope(x.cpu(), case["norm"], None if w is None else w.cpu(), None if b is None else b.cpu(),
                      eps=1e-6, cos=None if cs is None else cs.cpu(), sin=None if sn is None else sn.cpu())
    got = qk_norm_rope(x, case["norm"], w, b, eps=1e-6, cos=cs, sin=sn)
    torch.cuda.synchronize()
    assert got.data_ptr() == x.data_ptr()
    _check(got, ref)


def test_prologue_strided_view_and_offset():
    """q of a packed [B, S, 3, H, D] projection, sequence shard at offset 40."""
    from longvideosparseattention_b200.prologue import qk_norm_rope
    B, S, H, D = 1, 90, 12, 128
    g = torch.Generator().manual_seed(11)
    qkv = torch.randn(B, S, 3, H, D, generator=g).bfloat16().cuda()
    before = qkv.clone()
    cs, sn = _tables(200, D, 5)
    w = (1 + 0.3 * torch.randn(H * D, generator=g)).bfloat16().cuda()
    q = qkv[:, :, 0]
    ref = O.norm_rope(q.cpu(), "rms_row", w.cpu(), eps=1e-6, cos=cs.cpu(), sin=sn.cpu(), rope_offset=40)
    qk_norm_rope(q, "rms_row", w, eps=1e-6, cos=cs, sin=sn, rope_offset=40)
    torch.cuda.synchronize()
    _check(qkv[:, :, 0], ref)
    assert torch.equal(qkv[:, :, 1:], before[:, :, 1:])  # k and v untouched


def test_rotation_preserves_pair_norms_at_full_size():
    """Size-independent property at cfg2 size (126 360 x 12 x 128): the rotation
    keeps every (x0, x1) pair's length."""
    from longvideosparseattention_b200.prologue import qk_norm_rope
    S, H, D = 81 * 1560, 12, 128
    x = torch.randn(1, S, H, D, device="cuda", dtype=torch.bfloat16)
    cs, sn = _tables(S, D, 9)
    pre = x.float().unflatten(-1, (-1, 2)).pow(2).sum(-1)
    qk_norm_rope(x, None, cos=cs, sin=sn)
    post = x.float().unflatten(-1, (-1, 2)).pow(2).sum(-1)
    assert ((post - pre).abs() <= 1e-2 * pre + 1e-3).all()
