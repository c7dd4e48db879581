"""QK prologue, host side: the oracle's norm + rotation pinned to the
reference's rotary golden vectors and to torch's norm implementations, the
table conversion, and the C ABI's argument checks (no GPU needed)."""

import ctypes
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import lvsa_oracle as O
from tests.conftest import GOLDEN

ROPE = np.load(os.path.join(GOLDEN, "rope.npz"))


@pytest.mark.parametrize("name", ["d128", "d64"])
def test_oracle_rotation_matches_reference_apply_rotary_emb(name):
    from longvideosparseattention_b200.prologue import rope_tables
    x = torch.from_numpy(ROPE[f"{name}.x"])
    cs, sn = rope_tables(torch.from_numpy(ROPE[f"{name}.cos"]), torch.from_numpy(ROPE[f"{name}.sin"]))
    assert cs.shape == (x.shape[1], x.shape[3] // 2)
    got = O.norm_rope(x, None, cos=cs, sin=sn)
    np.testing.assert_allclose(got.numpy(), ROPE[f"{name}.out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", ["d128", "d64"])
def test_rope_offset_equals_reference_slice(name):
    """Table row rope_offset + s (sequence shards) is the reference's
    slice_rotary_emb for that rank (lvsa/rope.py:31-57)."""
    from longvideosparseattention_b200.prologue import rope_tables
    S = ROPE[f"{name}.x"].shape[1]
    local = S // 3
    cs, sn = rope_tables(torch.from_numpy(ROPE[f"{name}.cos"]), torch.from_numpy(ROPE[f"{name}.sin"]))
    c1, s1 = rope_tables(torch.from_numpy(ROPE[f"{name}.slice_cos"]), torch.from_numpy(ROPE[f"{name}.slice_sin"]))
    if S % 3:
        # No table dimension equals local * world: the reference returns it unsliced.
        np.testing.assert_array_equal(cs.numpy(), c1.numpy())
        return
    np.testing.assert_array_equal(cs[local:2 * local].numpy(), c1.numpy())
    np.testing.assert_array_equal(sn[local:2 * local].numpy(), s1.numpy())
    x = torch.from_numpy(ROPE[f"{name}.x"])[:, local:2 * local]
    np.testing.assert_allclose(O.norm_rope(x, None, cos=cs, sin=sn, rope_offset=local).numpy(),
                               O.norm_rope(x, None, cos=c1, sin=s1).numpy(), rtol=0, atol=0)


def test_oracle_norms_match_torch():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 5, 4, 64, generator=g)
    w = torch.randn(4 * 64, generator=g)
    wh, bh = torch.randn(64, generator=g), torch.randn(64, generator=g)
    want = F.rms_norm(x.reshape(2, 5, 256), (256,), w, eps=1e-6).reshape(2, 5, 4, 64)
    torch.testing.assert_close(O.norm_rope(x, "rms_row", w, eps=1e-6), want, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(O.norm_rope(x, "rms_head", wh, eps=1e-5), F.rms_norm(x, (64,), wh, eps=1e-5),
                               rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(O.norm_rope(x, "layer_head", wh, bh, eps=1e-5),
                               F.layer_norm(x, (64,), wh, bh, eps=1e-5), rtol=1e-5, atol=1e-5)


def test_prologue_abi_rejects_bad_arguments_without_launching():
    from longvideosparseattention_b200 import _native as N
    lib = N.load()
    a = N.LvsaQkPrologue()
    assert lib.lvsa_qk_prologue(None, None) == N.LVSA_ERR_INVALID_ARG
    a.x = N.LvsaTensor(4096, 12 * 128 * 100, 12 * 128, 128)
    a.dtype, a.batch, a.seq, a.heads, a.head_dim = 0, 1, 100, 12, 128
    a.norm, a.weight_dtype = N.LVSA_NORM_RMS_ROW, N.LVSA_DTYPE_BF16
    a.head_dim = 100
    assert lib.lvsa_qk_prologue(ctypes.byref(a), None) == N.LVSA_ERR_UNSUPPORTED
    a.head_dim = 128
    a.dtype = N.LVSA_DTYPE_F32
    assert lib.lvsa_qk_prologue(ctypes.byref(a), None) == N.LVSA_ERR_UNSUPPORTED
    a.dtype = 0
    a.x = N.LvsaTensor(4098, 12 * 128 * 100, 12 * 128, 128)      # not 16-byte aligned
    assert lib.lvsa_qk_prologue(ctypes.byref(a), None) == N.LVSA_ERR_ALIGNMENT
    a.x = N.LvsaTensor(4096, 12 * 128 * 100, 12 * 128 + 4, 128)  # row stride not 16-byte multiple
    assert lib.lvsa_qk_prologue(ctypes.byref(a), None) == N.LVSA_ERR_ALIGNMENT
    a.x = N.LvsaTensor(4096, 12 * 128 * 100, 12 * 128, 128)
    a.cos = 4096                                                   # cos without sin
    assert lib.lvsa_qk_prologue(ctypes.byref(a), None) == N.LVSA_ERR_INVALID_ARG
    a.cos = None
    a.norm = 7
    assert lib.lvsa_qk_prologue(ctypes.byref(a), None) == N.LVSA_ERR_INVALID_ARG
    a.norm = 0
    a.seq = 0                                                      # empty: nothing to do
    assert lib.lvsa_qk_prologue(ctypes.byref(a), None) == N.LVSA_OK
