"""GPU mask builder vs the oracle: bit-exact frame structures and tile CSR."""

import json
import os
import random

import numpy as np
import pytest
import torch

from oracle import lvsa_oracle as O
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

with open(os.path.join(GOLDEN, "patterns.json")) as fh:
    META = json.load(fh)
PATS = np.load(os.path.join(GOLDEN, "patterns.npz"))


def _check(T, P, W, nf, kfi, off, expand, n_text=0, BQ=128, BK=128, guards=None, golden=None):
    from longvideosparseattention_b200 import build_block_mask
    m = build_block_mask(T, P, W, nf, kfi, off, expand, n_text, BQ, BK, guards, device="cuda")
    torch.cuda.synchronize()
    fp = O.frame_pattern(T, P, W, nf, kfi, off, expand, boundary_guards=guards)
    c = m.counts()
    np.testing.assert_array_equal(m.global_frame_mask.cpu().numpy(), fp["global_frame_mask"])
    np.testing.assert_array_equal(m.window_bounds.cpu().numpy(), fp["window_bounds"])
    C = c["attended_C"]
    assert C == fp["attended_C"]
    np.testing.assert_array_equal(m.attended_indices.cpu().numpy()[:, :C], fp["attended_indices"])
    np.testing.assert_array_equal(m.frame_indptr.cpu().numpy(), fp["fi_indptr"])
    np.testing.assert_array_equal(m.frame_indices.cpu().numpy()[:c["frame_nnz"]], fp["fi_indices"])
    assert c["compact_n"] == fp["fi_compact_n"]
    if golden is not None:  # straight against the reference's own tensors
        np.testing.assert_array_equal(m.window_bounds.cpu().numpy(), PATS[f"{golden}.window_bounds"])
        np.testing.assert_array_equal(m.attended_indices.cpu().numpy()[:, :C],
                                      PATS[f"{golden}.attended_indices"])
        np.testing.assert_array_equal(m.frame_indices.cpu().numpy()[:c["frame_nnz"]],
                                      PATS[f"{golden}.fi_indices"])
    # attended bitsets
    bits = m.frame_bits.cpu().numpy().view(np.uint32)
    for f in range(T):
        got = [w * 32 + b for w in range(bits.shape[1]) for b in range(32) if (bits[f, w] >> b) & 1]
        assert got == fp["attended"][f]
    indptr, idx, fl = m.host_csr()
    wi, wx, wf, nqv, nkv = O.tile_csr(fp["attended"], T, P, T * P, n_text, BQ, BK)
    assert (m.n_q_video_tiles, m.n_k_video_tiles) == (nqv, nkv)
    np.testing.assert_array_equal(indptr.numpy(), wi)
    np.testing.assert_array_equal(idx.numpy(), wx)
    np.testing.assert_array_equal(fl.numpy(), wf)
    assert c["nnz"] == len(wx) <= m.max_nnz


@pytest.mark.parametrize("name", [n for n in sorted(META) if META[n]["world"] == 1])
def test_mask_matches_reference_patterns(name):
    c = META[name]
    _check(c["T"], c["P"], c["W"], c["n_first"], c["kfi"], c["offset"], c["expand"], golden=name)


@pytest.mark.parametrize("step", range(0, 50, 7))
def test_mask_cfg3_rotation_steps(step):
    _check(121, 1560, 2, 1, 4, step % 4, True)


@pytest.mark.parametrize("cfg", [
    dict(T=49, P=1590, W=2, nf=1, kfi=4, off=0, n_text=256),            # cfg4 HV
    dict(T=49, P=1350, W=1, nf=1, kfi=3, off=0, n_text=226, BQ=64),     # cfg5 Cog, 64-row Q
    dict(T=49, P=1350, W=1, nf=1, kfi=3, off=2, n_text=226),
])
def test_mask_text_configs(cfg):
    _check(cfg["T"], cfg["P"], cfg["W"], cfg["nf"], cfg["kfi"], cfg["off"], True,
           cfg["n_text"], cfg.get("BQ", 128), 128)


def test_mask_random_small():
    rng = random.Random(1234)
    for _ in range(60):
        T = rng.randint(1, 70)
        P = rng.choice([1, 3, 4, 8, 16, 100, 128, 130, 257])
        W = rng.randint(0, 5)
        kfi = rng.choice([None, 1, 2, 3, 5, 9])
        nf = rng.randint(1 if kfi is None else 0, 3)
        off = rng.randint(0, 12)
        BQ = rng.choice([16, 64, 128])
        BK = rng.choice([16, 64, 128, 256])
        nt = rng.choice([0, 0, 5, 128, 200])
        guards = sorted(rng.sample(range(T), min(T, rng.randint(0, 3))))
        _check(T, P, W, nf, kfi, off, rng.random() < 0.8, nt, BQ, BK, guards or None)


def test_mask_large_T():
    _check(2048, 16, 3, 1, 37, 5, True, n_text=64)


def test_mask_buffer_reuse_across_steps():
    from longvideosparseattention_b200 import build_block_mask
    m = build_block_mask(81, 1560, 2, 1, 4, 0, device="cuda")
    for step in range(1, 6):
        m2 = build_block_mask(81, 1560, 2, 1, 4, step % 4, reuse=m, device="cuda")
        assert m2.tile_indices.data_ptr() == m.tile_indices.data_ptr()
        fp = O.frame_pattern(81, 1560, 2, 1, 4, step % 4)
        wi, wx, wf, _, _ = O.tile_csr(fp["attended"], 81, 1560, 81 * 1560, 0, m.block_q, m.block_k)
        indptr, idx, fl = m2.host_csr()
        np.testing.assert_array_equal(idx.numpy(), wx)
        np.testing.assert_array_equal(fl.numpy(), wf)
