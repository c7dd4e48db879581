"""One GPU mask per pattern for every attention layer (the plugin's
LVSAAttentionImpl instances and hooks share ``step_mask.SHARED``): 30
instances x 3 denoising steps run exactly one builder pass per step, the
mask buffers never move and no memory is reserved after the first step;
outputs equal the kernel on a freshly built mask of each step bitwise.  The
builder reading the step index on the GPU (``device_step``) gives the same
tile CSR as the host keyframe offset, also under CUDA-graph replay."""

import pytest
import torch

from tests.gpu_util import seeded

pytestmark = pytest.mark.gpu

T, P, H, D, NT = 13, 200, 2, 128, 40


@pytest.fixture
def plugin_env(monkeypatch):
    for k, v in dict(LVSA_WINDOW_SIZE="4", LVSA_N_FIRST_FRAMES="4", LVSA_KEY_FRAME_INTERVAL="16",  # video frames (/4)
                     LVSA_AUTO_KEYFRAMES="0", LVSA_ROTATE_KEYFRAMES="1", LVSA_TOTAL_LATENT_FRAMES=str(T),
                     LVSA_PATCHES_PER_FRAME=str(P)).items():
        monkeypatch.setenv(k, v)
    from longvideosparseattention_b200.step_mask import SHARED
    from longvideosparseattention_b200.vllm_omni.attention_impl import LVSAAttentionImpl
    monkeypatch.setattr(LVSAAttentionImpl, "_hook_active", False)
    SHARED.clear()
    yield
    from longvideosparseattention_b200.vllm_omni import step_tracker
    step_tracker.reset()


def test_thirty_instances_three_steps_one_build_per_step(plugin_env):
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask, check_device_errors
    from longvideosparseattention_b200.step_mask import SHARED
    from longvideosparseattention_b200.vllm_omni import step_tracker
    from longvideosparseattention_b200.vllm_omni.attention_impl import LVSAAttentionImpl
    impls = [LVSAAttentionImpl(H, D, D ** -0.5) for _ in range(30)]
    assert impls[0].config.rotate_keyframes and impls[0].config.latent_key_frame_interval == 4
    n = T * P + NT
    xs = [(seeded((1, n, H, D), 3 * i, scale=D ** -0.5), seeded((1, n, H, D), 3 * i + 1, scale=D ** -0.5),
           seeded((1, n, H, D), 3 * i + 2)) for i in range(3)]
    ptrs, reserved = None, None
    for step in range(3):
        step_tracker.set_step(step)
        builds = SHARED.builds
        outs = [impl.forward_cuda(*xs[i % 3]) for i, impl in enumerate(impls)]
        torch.cuda.synchronize()
        check_device_errors(torch.device("cuda"))
        assert SHARED.builds == builds + 1, "one mask build per step, shared by all 30 instances"
        m = impls[0]._mask(T, P, NT, torch.device("cuda"))
        p = (m.tile_indptr.data_ptr(), m.tile_indices.data_ptr(), m.frame_bits.data_ptr())
        if ptrs is None:
            ptrs, reserved = p, torch.cuda.memory_reserved()
        else:
            assert p == ptrs, "rotation rebuilds into the same buffers"
            assert torch.cuda.memory_reserved() == reserved
        ref = build_block_mask(T, P, 1, 1, 4, step % 4, True, NT, device="cuda")
        for i in range(3):
            q, k, v = xs[i]
            o, to = block_sparse_attention(q[:, :T * P], k[:, :T * P], v[:, :T * P], ref,
                                           q[:, T * P:], k[:, T * P:], v[:, T * P:], scale=D ** -0.5)
            assert torch.equal(outs[i][:, :T * P], o) and torch.equal(outs[i][:, T * P:], to), (step, i)


@pytest.mark.parametrize("graph", [False, True])
def test_device_step_equals_host_offset(graph):
    from longvideosparseattention_b200 import build_block_mask
    kfi = 4
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    m = build_block_mask(21, 150, 2, 1, kfi, 0, True, 30, device="cuda", device_step=ctr)
    if graph:
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            build_block_mask(21, 150, 2, 1, kfi, 0, True, 30, device="cuda", device_step=ctr, reuse=m)
    for step in (0, 1, 2, 3, 4, 7, 10, 49):
        ctr.fill_(step)
        if graph:
            g.replay()
        else:
            build_block_mask(21, 150, 2, 1, kfi, 0, True, 30, device="cuda", device_step=ctr, reuse=m)
        want = build_block_mask(21, 150, 2, 1, kfi, step % kfi, True, 30, device="cuda")
        torch.cuda.synchronize()
        for a, b in zip(m.host_csr(), want.host_csr()):
            assert torch.equal(a, b), step
        assert torch.equal(m.window_bounds, want.window_bounds)


def test_lvsa_stats_counts_the_launch():
    from longvideosparseattention_b200 import build_block_mask, lvsa_stats
    m = build_block_mask(21, 150, 2, 1, 4, 1, True, 30, device="cuda")
    st = lvsa_stats(m, heads=3, head_dim=128)
    ip, idx, _ = m.host_csr()
    assert st["tiles"] == len(idx) == int(ip[-1])
    assert st["dense_tiles"] == m.n_q_tiles * m.n_k_tiles and 0 < st["density"] <= 1
    assert st["tile_flops"] == 4 * 128 * 128 * 128 * len(idx) * 3
