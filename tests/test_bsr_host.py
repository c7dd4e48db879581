"""Host expansion of a square-block CSR (the reference's FlashInfer plan:
LVSAMetadata's fi_indptr / fi_indices, R = C = P) into the kernel's frame
bitsets and 128 x 128 tile CSR, against a token-level brute force."""

import numpy as np
import pytest

from longvideosparseattention_b200.bsr import bsr_tile_csr
from longvideosparseattention_b200.sparse_attention import LVSAMetadata


def _brute(indptr, indices, M, N, R):
    MB, NB = -(-M // R), -(-N // R)
    allow = np.zeros((MB, NB), bool)
    for r in range(MB):
        allow[r, indices[indptr[r]:indptr[r + 1]]] = True
    tok = allow[np.arange(M)[:, None] // R, np.arange(N)[None, :] // R]
    ip, ix, fl = [0], [], []
    for t in range(-(-M // 128)):
        rows = tok[t * 128:min(M, t * 128 + 128)]
        for kt in range(-(-N // 128)):
            blk = rows[:, kt * 128:kt * 128 + 128]
            if blk.any():
                ix.append(kt)
                fl.append(0 if (blk.all() and kt * 128 + 128 <= N) else 1)
        ip.append(len(ix))
    return np.array(ip), np.array(ix), np.array(fl)


@pytest.mark.parametrize("T,P,W,kfi,off", [(9, 150, 1, 4, 3), (21, 64, 2, 5, 1), (13, 200, 1, 3, 0), (7, 96, 3, 2, 1)])
def test_bsr_tile_csr_matches_token_brute_force(T, P, W, kfi, off):
    m = LVSAMetadata.build(T, P, W, 1, kfi, 0, 1, keyframe_offset=off)
    ip, ix = m.fi_indptr.numpy(), m.fi_indices.numpy()
    bits, tip, tix, tfl, TT = bsr_tile_csr(ip, ix, m.fi_M, m.fi_N, P)
    wip, wix, wfl = _brute(ip, ix, m.fi_M, m.fi_N, P)
    np.testing.assert_array_equal(tip, wip)
    np.testing.assert_array_equal(tix, wix)
    np.testing.assert_array_equal(tfl, wfl)
    assert TT == max(m.fi_MB, m.fi_compact_n)
    for r in range(m.fi_MB):
        got = {c for c in range(TT) if (bits[r, c >> 5] >> (c & 31)) & 1}
        assert got == set(ix[ip[r]:ip[r + 1]].tolist())


def test_bsr_rejects_bad_csr():
    with pytest.raises(ValueError):
        bsr_tile_csr(np.array([0, 1]), np.array([5]), 128, 256, 128)
