"""The reference's FlashInfer path on the kernel: the frame CSR of
LVSAMetadata (fi_indptr / fi_indices, pinned to the reference by the golden
patterns) planned on ``LvsaBlockSparseWrapper`` exactly as
lvsa/lvsa_processor.py:768-829 plans flashinfer's wrapper, the compact K/V
filled from fi_global_copies / fi_local_copies and the query padded to fi_M
(:853-879), ``lvsa_flashinfer`` (lvsa/sparse_attention.py:709-742) run, and
the dense text term merged through the base-2 LSE as :881-913 does.  Result
vs the oracle at the bf16 tolerance; the LSE vs a float64 computation."""

import math

import numpy as np
import pytest
import torch

from oracle import lvsa_oracle as O
from tests.gpu_util import assert_close, seeded, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,P,H,D,W,kfi,off,nt,B", [(9, 150, 2, 128, 1, 4, 3, 37, 1), (13, 200, 3, 128, 1, 3, 1, 0, 2),
                                                    (11, 96, 2, 64, 2, 4, 2, 20, 1)])
def test_lvsa_flashinfer_dropin_with_lse_merge(T, P, H, D, W, kfi, off, nt, B):
    from longvideosparseattention_b200 import check_device_errors
    from longvideosparseattention_b200.bsr import LvsaBlockSparseWrapper
    from longvideosparseattention_b200.sparse_attention import LVSAMetadata, lvsa_flashinfer
    dev = torch.device("cuda")
    m = LVSAMetadata.build(T, P, W, 1, kfi, 0, 1, keyframe_offset=off)
    N = T * P
    q, k = seeded((B, N, H, D), 1, scale=D ** -0.5), seeded((B, N, H, D), 2, scale=D ** -0.5)
    v = seeded((B, N, H, D), 3)
    tk, tv = seeded((B, nt, H, D), 4, scale=D ** -0.5), seeded((B, nt, H, D), 5)
    gi = torch.tensor(m.global_indices)
    idx = (gi[:, None] * P + torch.arange(P)[None, :]).flatten().to(dev)
    kg, vg = k[:, idx], v[:, idx]
    # compact K/V and padded Q as the processor fills them
    ck = q.new_zeros(B, m.fi_compact_n * P, H, D)
    cv = q.new_zeros(B, m.fi_compact_n * P, H, D)
    for s, d in m.fi_global_copies:
        ck[:, d:d + P], cv[:, d:d + P] = kg[:, s:s + P], vg[:, s:s + P]
    for s, d in m.fi_local_copies:
        ck[:, d:d + P], cv[:, d:d + P] = k[:, s:s + P], v[:, s:s + P]
    qp = q.new_zeros(B, m.fi_M, H, D)
    qp[:, :N] = q
    w = LvsaBlockSparseWrapper(torch.empty(16, dtype=torch.uint8, device=dev))
    w.plan(indptr=m.fi_indptr.to(dev), indices=m.fi_indices.to(dev), M=m.fi_M, N=m.fi_N, R=P, C=P,
           num_qo_heads=H, num_kv_heads=H, head_dim=D, q_data_type="bfloat16")
    out = lvsa_flashinfer(qp, ck, cv, w, N, m.fi_M)
    fp = O.frame_pattern(T, P, W, 1, kfi, off)
    want, _ = O.attention(to_np(q), to_np(k), to_np(v), fp)
    torch.cuda.synchronize()
    check_device_errors(dev)
    assert out.shape == q.shape
    assert_close(to_np(out), want, what="lvsa_flashinfer")
    if not nt:
        return
    # The reference's merge with a dense text term, through the base-2 LSE.
    merged = torch.empty_like(q)
    for b in range(B):
        o_gen, lse_gen = w.run(qp[b], ck[b], cv[b], return_lse=True)
        o_gen, lse_gen = o_gen[:N].float(), lse_gen[:N]
        s = torch.einsum("nhd,thd->hnt", q[b].float(), tk[b].float()) / math.sqrt(D)
        lse_txt = (torch.logsumexp(s, -1) / math.log(2)).T              # [N, H], base 2
        o_txt = torch.einsum("hnt,thd->nhd", torch.softmax(s, -1), tv[b].float())
        mm = torch.maximum(lse_gen, lse_txt)
        wg, wt = torch.exp2(lse_gen - mm)[..., None], torch.exp2(lse_txt - mm)[..., None]
        merged[b] = ((o_gen * wg + o_txt * wt) / (wg + wt)).to(q.dtype)
    want_t, _ = O.attention(to_np(q), to_np(k), to_np(v), fp, None, to_np(tk), to_np(tv))
    assert_close(to_np(merged), want_t, what="LSE merge with text")
    # LSE against float64 on a few rows
    _, lse_gen = w.run(qp[0], ck[0], cv[0], return_lse=True)
    qn, kn = to_np(q)[0].astype(np.float64), to_np(k)[0].astype(np.float64)
    for t in (0, N // 2, N - 1):
        keys = np.concatenate([np.arange(f * P, (f + 1) * P) for f in fp["attended"][t // P]])
        for h in range(H):
            sc = kn[keys, h] @ qn[t, h] / math.sqrt(D)
            ref = (np.log(np.exp(sc - sc.max()).sum()) + sc.max()) / math.log(2)
            assert abs(lse_gen[t, h].item() - ref) < 3e-3
