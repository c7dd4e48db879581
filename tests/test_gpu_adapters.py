"""Adapters on CUDA: the fused prologue path (norm + rotation in one kernel
pass per tensor) against the unfused module calls on the same bf16 inputs.
Bound: |fused - unfused| <= 2e-2 |unfused| + 2e-2 (the unfused path rounds
to bf16 after the norm and again after the rotation, the fused one once)."""

import pytest
import torch

from tests.adapter_mocks import MockAttn, rope_pair

pytestmark = pytest.mark.gpu


def _close(a, b):
    d = (a.float() - b.float()).abs()
    assert bool((d <= 2e-2 * b.float().abs() + 2e-2).all()), f"max diff {d.max().item()}"


@pytest.mark.parametrize("name,norm,dual", [("hunyuan_video", "rms", True), ("cogvideox", "ln", False)])
@pytest.mark.parametrize("world,rank", [(1, 0), (3, 2)])
def test_dual_stream_fused_matches_unfused(name, norm, dual, world, rank):
    from longvideosparseattention_b200.adapters import get_adapter
    ad = get_adapter(name)
    attn = MockAttn(512, 4, norm, dual, seed=3).cuda().bfloat16()
    S_loc = 40
    hs = torch.randn(1, S_loc, 512, device="cuda").bfloat16()
    cos, sin = rope_pair(S_loc * world, 128, seed=2)
    rot = (cos.cuda(), sin.cuda())
    with torch.no_grad():
        q, k, v = ad.project_qkv(attn, hs, None, rot, S_loc, rank, world)
        q0, k0, v0 = ad.extract_qkv(attn, hs, None)
        q0, k0 = ad.apply_rotary(q0, k0, rot, S_loc, rank, world)
    _close(q, q0)
    _close(k, k0)
    assert torch.equal(v, v0)


def test_wan_fused_matches_unfused():
    from longvideosparseattention_b200.adapters import get_adapter

    class WanAttn(torch.nn.Module):
        def __init__(self, dim, heads):
            super().__init__()
            self.heads = heads
            self.to_q, self.to_k, self.to_v = (torch.nn.Linear(dim, dim) for _ in range(3))
            self.norm_q, self.norm_k = torch.nn.RMSNorm(dim, eps=1e-6), torch.nn.RMSNorm(dim, eps=1e-6)
            with torch.no_grad():
                self.norm_q.weight.uniform_(0.5, 1.5)
                self.norm_k.weight.uniform_(0.5, 1.5)
            self.to_out = torch.nn.ModuleList([torch.nn.Linear(dim, dim), torch.nn.Dropout(0.0)])

    ad = get_adapter("wan")
    attn = WanAttn(1536, 12).cuda().bfloat16()
    hs = torch.randn(1, 300, 1536, device="cuda").bfloat16()
    cos, sin = rope_pair(300, 128, seed=8)
    rot = (cos.cuda(), sin.cuda())
    with torch.no_grad():
        q, k, v = ad.project_qkv(attn, hs, None, rot, 300, 0, 1)
        q0, k0, v0 = ad.extract_qkv(attn, hs, None)
        q0, k0 = ad.apply_rotary(q0, k0, rot, 300, 0, 1)
    _close(q, q0)
    _close(k, k0)


def test_processor_layer_hunyuan_video_fused_vs_unfused():
    """A full HunyuanVideo-style layer through DistributedLVSAProcessor:
    (video, text) outputs with the fused prologue equal those with the module
    calls, within the bound above."""
    from longvideosparseattention_b200.adapters.base import ModelAdapter
    from longvideosparseattention_b200.adapters.hunyuan_video import HunyuanVideoAdapter
    from longvideosparseattention_b200.lvsa_processor import DistributedLVSAProcessor

    class Unfused(HunyuanVideoAdapter):
        def project_qkv(self, *args):
            return ModelAdapter.project_qkv(self, *args)

    T, P, dim, St = 9, 160, 512, 40
    attn = MockAttn(dim, 4, "rms", True, seed=4).cuda().bfloat16()
    hs = torch.randn(1, T * P, dim, device="cuda").bfloat16()
    ehs = torch.randn(1, St, dim, device="cuda").bfloat16()
    cos, sin = rope_pair(T * P, 128, seed=6)
    outs = []
    for ad in (HunyuanVideoAdapter(), Unfused()):
        proc = DistributedLVSAProcessor(T, P, 1, 1, 4, 0, 1, adapter=ad)
        with torch.no_grad():
            outs.append(proc(attn, hs, ehs, image_rotary_emb=(cos.cuda(), sin.cuda())))
    (v1, t1), (v2, t2) = outs
    assert v1.shape == (1, T * P, dim) and t1.shape == (1, St, dim)
    _close(v1, v2)
    _close(t1, t2)
