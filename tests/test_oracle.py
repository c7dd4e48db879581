"""The oracle pinned against the reference: golden vectors produced by the
unmodified reference (tests/golden/make_golden.py) and the reference test
suite's known answers (tests/test_swa_processor.py, tests/test_sparse_attention.py,
lvsa-vllm-omni/tests/test_global_kv.py of the reference)."""

import json
import os

import numpy as np
import pytest

from oracle import lvsa_oracle as O
from tests.conftest import GOLDEN

PATS = np.load(os.path.join(GOLDEN, "patterns.npz"))
with open(os.path.join(GOLDEN, "patterns.json")) as fh:
    META = json.load(fh)


@pytest.mark.parametrize("name", sorted(META))
def test_frame_pattern_matches_reference(name):
    c = META[name]
    fp = O.frame_pattern(c["T"], c["P"], c["W"], c["n_first"], c["kfi"], c["offset"],
                         c["expand"], c["rank"], c["world"], c["guards"] or None)
    assert fp["global_indices"] == PATS[f"{name}.global_indices"].tolist()
    np.testing.assert_array_equal(fp["global_frame_mask"], PATS[f"{name}.global_frame_mask"])
    np.testing.assert_array_equal(fp["window_bounds"], PATS[f"{name}.window_bounds"])
    np.testing.assert_array_equal(fp["attended_indices"], PATS[f"{name}.attended_indices"])
    np.testing.assert_array_equal(fp["fi_indptr"], PATS[f"{name}.fi_indptr"])
    np.testing.assert_array_equal(fp["fi_indices"], PATS[f"{name}.fi_indices"])
    np.testing.assert_array_equal(np.asarray(fp["local_frames"]), PATS[f"{name}.local_frames"])
    wc = [(f, s, e) for f, parts in sorted(fp["window_ctx"].items()) for s, e in parts]
    np.testing.assert_array_equal(np.asarray(wc, dtype=np.int64).reshape(-1, 3),
                                  PATS[f"{name}.window_ctx"])
    assert fp["fi_MB"] == c["fi_MB"] and fp["fi_compact_n"] == c["fi_compact_n"]
    assert fp["attended_C"] == c["attended_C"] and fp["local_seq"] == c["local_seq"]


# Known answers from the reference test suite.
def test_known_adaptive_bounds():
    assert O.adaptive_window_bounds(10, 3, 21) == (7, 13)          # test_swa_processor.py:18-22
    for f in range(21):
        lo, hi = O.adaptive_window_bounds(f, 3, 21)
        assert hi - lo + 1 == 7                                     # :37-42


def test_known_boundary_guards():
    assert O.compute_boundary_guard_frames(20, 100, 10, 2, 2) == [8, 9, 10, 11, 12]  # :73-84


def test_known_globals_and_rotation():
    assert O.compute_global_indices(21, 1, 5) == [0, 5, 10, 15, 20]           # :119-125
    assert O.compute_global_indices(21, 1, 5, 2) == [0, 1, 2, 7, 12, 17]      # :127-137
    assert O.compute_global_indices(9, 1, 4, 3) == [0, 2, 3, 7]               # cfg1 pattern
    covered = set()
    for off in range(5):
        covered |= set(O.compute_global_indices(21, 1, 5, off))
    assert covered == set(range(21))                                          # :175-184


@pytest.mark.parametrize("T,ref", [(21, 21), (20, 21), (17, 33), (33, 33), (1, 21)])
def test_known_kfi_one_at_or_below_reference(T, ref):
    assert O.compute_auto_kfi(T, 3, 1, ref) == 1                              # test_sparse_attention.py:416-429


def test_known_auto_kfi_values():
    assert O.compute_auto_kfi(81, 3, 1, 21) == 6
    assert O.compute_auto_kfi(121, 3, 1, 21) == 9
    assert O.compute_auto_kfi(49, 3, 1, 33) == 2


def test_attended_count_constant_for_baseline_configs():
    for (T, P, W, kfi, off, want) in [(9, 1560, 1, 4, 3, 7), (81, 1560, 2, 4, 0, 26),
                                      (49, 1590, 2, 4, 0, 18), (49, 1350, 1, 3, 0, 20)]:
        fp = O.frame_pattern(T, P, W, 1, kfi, off)
        assert {len(a) for a in fp["attended"]} == {want}


ATTN = sorted(f[5:-4] for f in os.listdir(GOLDEN) if f.startswith("attn_"))


@pytest.mark.parametrize("name", ATTN)
def test_oracle_attention_matches_reference(name):
    z = np.load(os.path.join(GOLDEN, f"attn_{name}.npz"))
    T, P, H, Hkv, D, W, nf, kfi, off, nt, B, seed = z["params"].tolist()
    fp = O.frame_pattern(T, P, W, nf, kfi, off)
    out, tout = O.attention(z["q"], z["k"], z["v"], fp, z["text_q"], z["text_k"], z["text_v"])
    np.testing.assert_allclose(out, z["out"], atol=2e-5, rtol=1e-4)
    if nt > 0:
        np.testing.assert_allclose(tout, z["text_out"], atol=2e-5, rtol=1e-4)


def _brute_tiles(att, T, P, Nv, BQ, BK):
    allowed = np.zeros((Nv, Nv), dtype=bool)
    fr = np.arange(Nv) // P
    A = np.zeros((T, T), dtype=bool)
    for f in range(T):
        A[f, att[f]] = True
    allowed = A[fr[:, None], fr[None, :]]
    nq, nk = -(-Nv // BQ), -(-Nv // BK)
    res = {}
    for qb in range(nq):
        for kb in range(nk):
            blk = allowed[qb * BQ:(qb + 1) * BQ, kb * BK:(kb + 1) * BK]
            if blk.any():
                res[(qb, kb)] = int(not (blk.all() and (kb + 1) * BK <= Nv))
    return res


@pytest.mark.parametrize("T,P,W,kfi,off,BQ,BK", [
    (9, 8, 1, 4, 3, 16, 16), (7, 130, 1, 3, 1, 128, 128), (12, 50, 2, 4, 2, 64, 128),
    (5, 3, 1, 2, 0, 8, 4), (11, 128, 1, 3, 0, 128, 128), (6, 200, 0, 2, 1, 128, 64)])
def test_tile_csr_definition_brute_force(T, P, W, kfi, off, BQ, BK):
    fp = O.frame_pattern(T, P, W, 1, kfi, off)
    Nv = T * P
    indptr, idx, fl, nq, nk = O.tile_csr(fp["attended"], T, P, Nv, 0, BQ, BK)
    brute = _brute_tiles(fp["attended"], T, P, Nv, BQ, BK)
    got = {}
    for qb in range(nq):
        row = idx[indptr[qb]:indptr[qb + 1]]
        assert np.all(np.diff(row) > 0)
        for kb, f in zip(row, fl[indptr[qb]:indptr[qb + 1]]):
            got[(qb, int(kb))] = int(f)
    assert got == brute


def test_tile_csr_text_segment():
    fp = O.frame_pattern(5, 40, 1, 1, 2, 0)
    indptr, idx, fl, nq, nk = O.tile_csr(fp["attended"], 5, 40, 200, 130, 64, 128)
    assert nq == 4 and nk == 2
    assert len(indptr) == nq + 3 + 1
    for r in range(nq):  # video rows end with the two text tiles, second one ragged
        assert idx[indptr[r + 1] - 2:indptr[r + 1]].tolist() == [2, 3]
        assert fl[indptr[r + 1] - 2:indptr[r + 1]].tolist() == [0, 1]
    for r in range(nq, nq + 3):  # text rows dense
        assert idx[indptr[r]:indptr[r + 1]].tolist() == [0, 1, 2, 3]
        assert fl[indptr[r]:indptr[r + 1]].tolist() == [0, 1, 0, 1]


def test_flop_counts_baseline_cfg1():
    fp = O.frame_pattern(9, 1560, 1, 1, 4, 3)
    tiles, exact = O.flop_counts(fp["attended"], 9, 1560, 9 * 1560, 0, 12, 128)
    assert round(exact / 1e9, 1) == 942.0
    assert round(tiles / 1e9, 1) == 964.5


def test_oracle_attention_cfg1_full_size_matches_reference():
    """BASELINE configs[0] at full size (fp32): the oracle on one query frame
    against the reference's lvsa_sdpa rows kept in tests/golden/cfg1.npz."""
    from tests.golden.make_golden import CFG1, cfg1_inputs
    z = np.load(os.path.join(GOLDEN, "cfg1.npz"))
    q, k, v = (x.numpy() for x in cfg1_inputs())
    c = CFG1
    fp = O.frame_pattern(c["T"], c["P"], c["W"], c["n_first"], c["kfi"], c["step"] % c["kfi"])
    frame = 3
    want, _ = O.attention(q, k, v, fp, frames=[frame])
    sel = (z["rows"] // c["P"]) == frame
    assert sel.sum() == c["rows_per_frame"]
    np.testing.assert_allclose(want[0, z["rows"][sel]], z["out"][sel], atol=2e-6, rtol=0)
