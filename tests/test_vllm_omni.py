"""vLLM-Omni plugin mirror: config, geometry, global-KV known answers (CPU)
and LVSAAttentionImpl.forward_cuda on the GPU against the oracle."""

import numpy as np
import pytest
import torch

from longvideosparseattention_b200.vllm_omni import (LVSAAttentionImpl, LVSABackend, LVSAConfig,
                                                      build_global_kv, candidate_patches_per_frame)
from longvideosparseattention_b200.vllm_omni import step_tracker
from oracle import lvsa_oracle as O


def test_config_defaults_env_json(monkeypatch):
    c = LVSAConfig()
    assert (c.window_size, c.n_first_frames, c.key_frame_interval, c.backend) == (12, 4, 16, "sdpa")
    assert (c.latent_window_size, c.latent_n_first_frames, c.latent_key_frame_interval) == (3, 1, 4)
    monkeypatch.setenv("LVSA_WINDOW_SIZE", "8")
    monkeypatch.setenv("LVSA_ROTATE_KEYFRAMES", "yes")
    c = LVSAConfig.from_env()
    assert c.window_size == 8 and c.rotate_keyframes
    monkeypatch.setenv("LVSA_CONFIG", '{"n_first_frames": 8, "bogus": 1}')
    assert LVSAConfig.from_env().n_first_frames == 8


def test_candidate_patches(monkeypatch):
    monkeypatch.delenv("LVSA_PATCHES_PER_FRAME", raising=False)
    monkeypatch.delenv("LVSA_VIDEO_HEIGHT", raising=False)
    assert candidate_patches_per_frame() == [1560]
    monkeypatch.setenv("LVSA_VIDEO_HEIGHT", "480")
    monkeypatch.setenv("LVSA_VIDEO_WIDTH", "832")
    assert candidate_patches_per_frame() == [1560]
    monkeypatch.setenv("LVSA_PATCHES_PER_FRAME", "8, 16")
    assert candidate_patches_per_frame() == [8, 16]


def test_build_global_kv_known_answer():
    # reference test: frames [1, 3], P = 2 -> tokens [2, 3, 6, 7]
    k = torch.arange(8).view(1, 8, 1, 1).float()
    kg, vg = build_global_kv(k, k, [1, 3], 2)
    assert kg.flatten().tolist() == [2, 3, 6, 7]
    e, _ = build_global_kv(k, k, [], 2)
    assert e.shape == (1, 0, 1, 1)


def test_backend_and_geometry(monkeypatch):
    assert LVSABackend.get_name() == "LVSA" and LVSABackend.get_impl_cls() is LVSAAttentionImpl
    monkeypatch.setenv("LVSA_PATCHES_PER_FRAME", "16")
    assert LVSAAttentionImpl.detect_geometry(10 * 16 + 7, 10) == (16, 7)
    assert LVSAAttentionImpl.detect_geometry(10 * 16 - 1, 10) == (None, None)


@pytest.mark.gpu
def test_forward_cuda_matches_oracle(monkeypatch):
    T, P, H, D, nt = 9, 96, 2, 128, 24
    monkeypatch.setenv("LVSA_TOTAL_LATENT_FRAMES", str(T))
    monkeypatch.setenv("LVSA_PATCHES_PER_FRAME", str(P))
    monkeypatch.setenv("LVSA_CONFIG", '{"window_size": 4, "n_first_frames": 4, "key_frame_interval": 12,'
                       ' "auto_keyframes": false, "rotate_keyframes": true, "total_latent_frames": %d}' % T)
    impl = LVSAAttentionImpl(H, D, D ** -0.5)
    g = torch.Generator().manual_seed(3)
    mk = lambda: (torch.randn(1, T * P + nt, H, D, generator=g) / D ** 0.25).to(torch.bfloat16).cuda()
    q, k, v = mk(), mk(), mk()
    f = lambda x: x.float().cpu().numpy()
    for step in (0, 1, 2):
        step_tracker.set_step(step)
        out = impl.forward_cuda(q, k, v)
        torch.cuda.synchronize()
        fp = O.frame_pattern(T, P, 1, 1, 3, step % 3)
        nv = T * P
        want, twant = O.attention(f(q[:, :nv]), f(k[:, :nv]), f(v[:, :nv]), fp, f(q[:, nv:]), f(k[:, nv:]),
                                  f(v[:, nv:]))
        got = f(out)
        for a, b, what in ((got[:, :nv], want, "video"), (got[:, nv:], twant, "text")):
            d = np.abs(a - b)
            assert d.max() < 2e-2 and d.mean() < 2e-3, (step, what, d.max())
    step_tracker.reset()
