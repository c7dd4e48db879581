"""DistributedLVSAProcessor / adapters: the reference's processor contract
(state, rotation, geometry guard, adapter registry) on CPU, and an end-to-end
attention layer on the GPU against the oracle."""

import json
import os
import types

import numpy as np
import pytest
import torch
import torch.nn as nn

from longvideosparseattention_b200.adapters import ModelAdapter, get_adapter, register_adapter
from longvideosparseattention_b200.lvsa_processor import DistributedLVSAProcessor, WanDistributedLVSAProcessor
from oracle import lvsa_oracle as O
from tests.conftest import GOLDEN

PATS = np.load(os.path.join(GOLDEN, "patterns.npz"))


def test_alias_and_registry():
    assert WanDistributedLVSAProcessor is DistributedLVSAProcessor
    a = get_adapter("wan")
    assert isinstance(a, ModelAdapter)
    with pytest.raises(KeyError, match="Available adapters"):
        get_adapter("nope")
    register_adapter("wan2", "longvideosparseattention_b200.adapters.wan", "WanAdapter")
    assert type(get_adapter("wan2")).__name__ == "WanAdapter"


@pytest.mark.parametrize("step", range(8))
def test_rotation_matches_reference_patterns(step):
    p = DistributedLVSAProcessor(121, 1560, 2, 1, 4, 0, 1)
    p.set_step(step)
    name = f"cfg3_s{step % 4}"
    assert p._global_indices == PATS[f"{name}.global_indices"].tolist()
    np.testing.assert_array_equal(p._window_bounds.numpy(), PATS[f"{name}.window_bounds"])
    assert p._current_offset == step % 4


def test_set_window_and_sparsity_rederive_kfi():
    p = DistributedLVSAProcessor(81, 16, 3, 1, 6, 0, 1)
    p.set_window_size(0)
    assert p.window_size == 0 and p.key_frame_interval == O.compute_auto_kfi(81, 0, 1, 21)
    assert all(lo > hi for lo, hi in p._window_bounds.tolist())  # globals only
    p.set_sparsity_scale(0.5)
    assert p.key_frame_interval == O.compute_auto_kfi(81, 0, 1, 21, 0.5)


def test_geometry_guard_and_cp_divisibility():
    p = DistributedLVSAProcessor(20, 10, 2, 1, 5, 0, 2)
    assert p.local_seq == 100 and p._geometry_matches(100) and not p._geometry_matches(101)
    assert p._boundary_guards == [8, 9, 10, 11, 12]
    with pytest.raises(AssertionError, match="divisible"):
        DistributedLVSAProcessor(21, 7, 1, 1, 4, 0, 2)


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight).to(x.dtype)


def _wan_attn(C, H, device, dtype):
    torch.manual_seed(0)
    a = types.SimpleNamespace()
    a.heads = H
    a.to_q, a.to_k, a.to_v = (nn.Linear(C, C).to(device, dtype) for _ in range(3))
    a.norm_q, a.norm_k = RMSNorm(C).to(device), RMSNorm(C).to(device)
    a.to_out = [nn.Linear(C, C).to(device, dtype), nn.Dropout(0.0)]
    a.add_k_proj = None
    return a


@pytest.mark.gpu
def test_processor_layer_matches_oracle():
    T, P, H, D, W, kfi = 7, 96, 2, 64, 1, 3
    C = H * D
    dev, dt = torch.device("cuda"), torch.bfloat16
    attn = _wan_attn(C, H, dev, dt)
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(1, T * P, C, generator=g) * 0.5).to(dev, dt)
    ang = torch.randn(1, T * P, 1, D, generator=g).to(dev)
    rot = (ang.cos(), ang.sin())
    proc = DistributedLVSAProcessor(T, P, W, 1, kfi, 0, 1)
    for step in (0, 1, 2):
        proc.set_step(step)
        with torch.no_grad():
            got = proc(attn, x, None, rotary_emb=rot)
            ad = get_adapter("wan")
            q, k, v = ad.extract_qkv(attn, x, None)
            q, k = ad.apply_rotary(q, k, rot, T * P, 0, 1)
            fp = O.frame_pattern(T, P, W, 1, kfi, step % kfi)
            f = lambda t: t.float().cpu().numpy()
            att, _ = O.attention(f(q), f(k), f(v), fp)
            want = ad.output_projection(attn, torch.from_numpy(att).to(dev, dt), dt)
        d = (got.float() - want.float()).abs()
        assert d.max().item() < 3e-2 and d.mean().item() < 3e-3, (step, d.max().item())


@pytest.mark.gpu
def test_processor_dense_fallback_on_geometry_mismatch(capsys):
    T, P, H, D = 4, 64, 2, 64
    C = H * D
    attn = _wan_attn(C, H, torch.device("cuda"), torch.bfloat16)
    proc = DistributedLVSAProcessor(T, P, 1, 1, 2, 0, 1)
    x = torch.randn(1, T * P + 5, C, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        out = proc(attn, x)
    assert out.shape == x.shape and torch.isfinite(out.float()).all()
    assert "geometry mismatch" in capsys.readouterr().out


def test_cp_mode_option_and_shard_invalidation():
    from longvideosparseattention_b200.lvsa_processor import DistributedLVSAProcessor
    with pytest.raises(ValueError):
        DistributedLVSAProcessor(9, 40, 1, 1, 4, 0, 2, cp_mode="ring")
    p = DistributedLVSAProcessor(9, 40, 1, 1, 4, 0, 2, cp_mode="reference")
    assert p.cp_mode == "reference" and p._shard is None
    p._shard = object()
    p.set_step(1)  # rotation: the shard pattern is rebuilt lazily
    assert p._shard is None
