"""The vLLM-Omni block-level hooks run end to end on the GPU against
stand-in vllm-omni model classes (only the fields the hooks read): the
patched forward's output equals the model's own projections followed by the
oracle's LVSA attention (fp32) and the output projection, within a relative
Frobenius error of 1e-2; non-grid shapes go to the original forward."""

import sys
import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import lvsa_oracle as O

pytestmark = pytest.mark.gpu

T, P, W, NF, KFI = 9, 160, 1, 1, 3


def _rotate(x, cos, sin):
    from longvideosparseattention_b200.adapters.wan import apply_rotary_interleaved
    return apply_rotary_interleaved(x, cos, sin)


class _QKV(torch.nn.Module):
    def __init__(self, dim, nh, nkv, hd):
        super().__init__()
        self.lin = torch.nn.Linear(dim, (nh + 2 * nkv) * hd)
        self.num_heads, self.num_kv_heads = nh, nkv

    def forward(self, x):
        return self.lin(x), None


@pytest.fixture
def fake_vllm(monkeypatch):
    for k, v in dict(LVSA_WINDOW_SIZE="4", LVSA_N_FIRST_FRAMES="4", LVSA_KEY_FRAME_INTERVAL="12",
                     LVSA_AUTO_KEYFRAMES="0", LVSA_CFG_PASSES="1").items():
        monkeypatch.setenv(k, v)
    from longvideosparseattention_b200.vllm_omni.attention_impl import LVSAAttentionImpl
    monkeypatch.setattr(LVSAAttentionImpl, "_hook_active", False)

    def mod(name):
        m = types.ModuleType(name)
        monkeypatch.setitem(sys.modules, name, m)
        return m
    for n in ("vllm_omni", "vllm_omni.diffusion", "vllm_omni.diffusion.models", "vllm_omni.diffusion.layers",
              "vllm_omni.diffusion.models.wan2_2", "vllm_omni.diffusion.models.hunyuan_video",
              "vllm_omni.diffusion.models.cosmos3"):
        mod(n)
    wan = mod("vllm_omni.diffusion.models.wan2_2.wan2_2_transformer")
    rope = mod("vllm_omni.diffusion.layers.rope")
    hv = mod("vllm_omni.diffusion.models.hunyuan_video.hunyuan_video_15_transformer")
    cos3 = mod("vllm_omni.diffusion.models.cosmos3.transformer_cosmos3")

    class RotaryEmbeddingWan:
        def __init__(self, is_neox_style, half_head_dim):
            assert not is_neox_style

        def __call__(self, x, cos, sin):
            return _rotate(x, cos, sin)

    class WanSelfAttention(torch.nn.Module):
        def __init__(self, dim, heads):
            super().__init__()
            self.num_heads = self.num_kv_heads = heads
            self.head_dim = dim // heads
            self.to_qkv = _QKV(dim, heads, heads, dim // heads)
            self.norm_q, self.norm_k = torch.nn.RMSNorm(dim, eps=1e-6), torch.nn.RMSNorm(dim, eps=1e-6)
            self.to_out = torch.nn.Linear(dim, dim)
            self.dropout = torch.nn.Identity()

        def forward(self, hidden_states, rotary_emb=None, attn_metadata=None):
            return "original"

    class HunyuanVideo15Attention(torch.nn.Module):
        def __init__(self, dim, heads):
            super().__init__()
            hd = dim // heads
            self.head_dim = hd
            self.to_qkv, self.add_kv_proj = _QKV(dim, heads, heads, hd), _QKV(dim, heads, heads, hd)
            self.norm_q, self.norm_k = torch.nn.RMSNorm(hd, eps=1e-6), torch.nn.RMSNorm(hd, eps=1e-6)
            self.norm_added_q, self.norm_added_k = torch.nn.RMSNorm(hd, eps=1e-6), torch.nn.RMSNorm(hd, eps=1e-6)
            self.to_out = torch.nn.ModuleList([torch.nn.Linear(dim, dim)])
            self.to_add_out = torch.nn.Linear(dim, dim)

        def rope(self, x, cos, sin):
            return _rotate(x, cos[None, :, None, :], sin[None, :, None, :])

        def forward(self, hidden_states, encoder_hidden_states=None, attention_mask=None,
                    image_rotary_emb=None, hidden_states_mask=None):
            return "original"

    class _Norm(torch.nn.Module):
        def __init__(self, d):
            super().__init__()
            self.weight = torch.nn.Parameter(1 + 0.1 * torch.randn(d))
            self.variance_epsilon = 1e-6

    class Cosmos3CrossAttention(torch.nn.Module):
        def __init__(self, dim, heads, kv_heads):
            super().__init__()
            hd = dim // heads
            self.num_heads_local, self.num_kv_heads_local, self.head_dim = heads, kv_heads, hd
            self.to_q = torch.nn.Linear(dim, heads * hd)
            self.to_k, self.to_v = torch.nn.Linear(dim, kv_heads * hd), torch.nn.Linear(dim, kv_heads * hd)
            self.norm_q, self.norm_k = _Norm(hd), _Norm(hd)
            self.to_out = torch.nn.Linear(dim, dim)

        def forward(self, hidden_states, k_und, v_und, freqs_cos, freqs_sin):
            return "original"

    wan.WanSelfAttention, rope.RotaryEmbeddingWan = WanSelfAttention, RotaryEmbeddingWan
    hv.HunyuanVideo15Attention = HunyuanVideo15Attention
    cos3.Cosmos3CrossAttention = Cosmos3CrossAttention
    cos3._apply_rotary_pos_emb = lambda q, k, c, s: (_rotate(q, c, s), _rotate(k, c, s))
    cos3._is_sp_active = lambda: False
    yield types.SimpleNamespace(wan=WanSelfAttention, hv=HunyuanVideo15Attention, cos3=Cosmos3CrossAttention)


def _tables(S, D, seed):
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand(S, D // 2, generator=g) * 6
    return torch.cos(ang).repeat_interleave(2, -1), torch.sin(ang).repeat_interleave(2, -1)


def _oracle(q, k, v, tq=None, tk=None, tv=None):
    fp = O.frame_pattern(T, P, W, NF, KFI, 0)
    f = lambda x: None if x is None else x.float().cpu().numpy()
    out, tout = O.attention(f(q), f(k), f(v), fp, f(tq), f(tk), f(tv))
    conv = lambda a: None if a is None else torch.from_numpy(a).cuda().bfloat16()
    return conv(out), conv(tout)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_wan_hook(fake_vllm):
    from longvideosparseattention_b200.vllm_omni.wan_hook import install_wan_lvsa_hook
    install_wan_lvsa_hook(total_latent_frames=T)
    m = fake_vllm.wan(256, 2).cuda().bfloat16()
    x = torch.randn(1, T * P, 256, device="cuda").bfloat16()
    c, s = _tables(T * P, 128, 1)
    rot = (c[None, :, None, :].cuda(), s[None, :, None, :].cuda())
    with torch.no_grad():
        got = m(x, rot)
        qkv, _ = m.to_qkv(x)
        q, k, v = qkv.split([256, 256, 256], -1)
        q, k = m.norm_q(q).unflatten(2, (2, 128)), m.norm_k(k).unflatten(2, (2, 128))
        q, k = _rotate(q, *rot), _rotate(k, *rot)
        o, _ = _oracle(q, k, v.unflatten(2, (2, 128)))
        want = m.to_out(o.flatten(2, 3))
        assert m(x[:, :100], rot) == "original"   # not a T x P grid
    assert _rel(got, want) < 1e-2


def test_hunyuan_hook(fake_vllm):
    from longvideosparseattention_b200.vllm_omni.hunyuan_hook import install_hunyuan_lvsa_hook
    install_hunyuan_lvsa_hook(total_latent_frames=T)
    m = fake_vllm.hv(256, 2).cuda().bfloat16()
    x = torch.randn(1, T * P, 256, device="cuda").bfloat16()
    e = torch.randn(1, 77, 256, device="cuda").bfloat16()
    c, s = _tables(T * P, 128, 2)
    rot = (c.cuda(), s.cuda())
    with torch.no_grad():
        vid, txt = m(x, e, None, rot)
        qkv, _ = m.to_qkv(x)
        q, k, v = (t.unflatten(-1, (2, -1)) for t in qkv.split([256, 256, 256], -1))
        q, k = m.rope(m.norm_q(q), *rot), m.rope(m.norm_k(k), *rot)
        eqkv, _ = m.add_kv_proj(e)
        eq, ek, ev = (t.unflatten(-1, (2, -1)) for t in eqkv.split([256, 256, 256], -1))
        eq, ek = m.norm_added_q(eq), m.norm_added_k(ek)
        o, to = _oracle(q, k, v, eq, ek, ev)
        wv, wt = m.to_out[0](o.flatten(2, 3)), m.to_add_out(to.flatten(2, 3))
        assert m(x, None, None, rot) == "original"  # no encoder stream
    assert _rel(vid, wv) < 1e-2 and _rel(txt, wt) < 1e-2


def test_cosmos3_hook_gqa(fake_vllm):
    from longvideosparseattention_b200.vllm_omni.cosmos3_hook import install_cosmos3_lvsa_hook
    install_cosmos3_lvsa_hook(total_latent_frames=T)
    m = fake_vllm.cos3(512, 4, 2).cuda().bfloat16()
    x = torch.randn(1, T * P, 512, device="cuda").bfloat16()
    ku = (torch.randn(1, 50, 2, 128, device="cuda") / 3).bfloat16()
    vu = torch.randn(1, 50, 2, 128, device="cuda").bfloat16()
    c, s = _tables(T * P, 128, 3)
    rc, rs = c[None, :, None, :].cuda(), s[None, :, None, :].cuda()
    with torch.no_grad():
        got = m(x, ku, vu, rc, rs)
        q = m.to_q(x).view(1, T * P, 4, 128)
        k, v = m.to_k(x).view(1, T * P, 2, 128), m.to_v(x).view(1, T * P, 2, 128)
        q = F.rms_norm(q, (128,), m.norm_q.weight, 1e-6)
        k = F.rms_norm(k, (128,), m.norm_k.weight, 1e-6)
        q, k = _rotate(q, rc, rs), _rotate(k, rc, rs)
        o, _ = _oracle(q, k, v, None, ku, vu)
        want = m.to_out(o.reshape(1, T * P, -1))
        assert m(x[:, :77], ku, vu, rc[:, :77], rs[:, :77]) == "original"
    assert _rel(got, want) < 1e-2
