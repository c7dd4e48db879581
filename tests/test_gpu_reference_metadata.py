"""The reference's LVSAMetadata at the boundary, on the GPU: lvsa_sdpa and
sparse_windowed_attention given a reference-shaped metadata object (the
fields the reference's dataclass carries, lvsa/sparse_attention.py:286-353;
no keyframe interval, no offset, no block_mask method) equal the same calls
with this package's metadata bitwise at world = 1, and reproduce the
reference's per-rank outputs at world > 1 (tests/golden/cp.npz)."""

import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN
from tests.gpu_util import MAX_ABS_TOL, MEAN_ABS_TOL, seeded
from tests.test_reference_metadata import META, standin

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["cfg1", "cfg5", "w0", "noexpand", "kfi_none", "nfirst3", "wide_w", "big_off"])
def test_lvsa_sdpa_with_reference_metadata_world1(name):
    from longvideosparseattention_b200 import check_device_errors
    from longvideosparseattention_b200.sparse_attention import LVSAMetadata, lvsa_sdpa, \
        sparse_windowed_attention
    c = META[name]
    T, P = c["T"], c["P"]
    H, D, nt = 2, 128, 37
    ref_like = standin(name)
    ours = LVSAMetadata.build(T, P, c["W"], c["n_first"], c["kfi"], 0, 1, expand_window=c["expand"],
                              keyframe_offset=c["offset"])
    q, k, v = (seeded((1, T * P, H, D), s, scale=D ** -0.5) for s in (1, 2, 3))
    tk, tv = seeded((1, nt, H, D), 4, scale=D ** -0.5), seeded((1, nt, H, D), 5)
    gi = torch.tensor(ref_like.global_indices, dtype=torch.long)
    idx = (gi[:, None] * P + torch.arange(P)[None, :]).flatten().cuda()
    kg, vg = torch.cat([k[:, idx], tk], 1), torch.cat([v[:, idx], tv], 1)
    want = lvsa_sdpa(q, k, v, kg, vg, ours)
    got = lvsa_sdpa(q, k, v, kg, vg, ref_like)
    got2 = sparse_windowed_attention(q, k, v, kg, vg, ref_like, "sdpa")
    torch.cuda.synchronize()
    check_device_errors(q.device)
    assert torch.equal(got, want) and torch.equal(got2, want)


CP = np.load(os.path.join(GOLDEN, "cp.npz"))


@pytest.mark.parametrize("name", sorted({k.split(".")[0] for k in CP.files}))
def test_lvsa_sdpa_with_reference_metadata_per_rank(name):
    """world > 1: the rank's shard + the gathered [globals; text] K/V, as the
    reference's processor hands them to lvsa_sdpa, against its outputs."""
    from longvideosparseattention_b200 import check_device_errors
    from longvideosparseattention_b200.sparse_attention import lvsa_sdpa
    dev = torch.device("cuda")
    T, P, H, Hkv, D, W, nf, kfi, off, nt, world, _ = [int(x) for x in CP[f"{name}.params"]]
    t = lambda key: torch.from_numpy(CP[f"{name}.{key}"]).to(torch.bfloat16).to(dev)
    q, k, v = t("q"), t("k"), t("v")
    S_r = T * P // world
    for r in range(world):
        gidx = CP[f"{name}.globals{r}"].tolist()
        meta = SimpleNamespace(total_latent_frames=T, num_patches=P, window_size=W, expand_window=True,
                               global_indices=gidx, rank=r, world=world)
        idx = torch.tensor([g * P + i for g in gidx for i in range(P)], device=dev)
        kg, vg = k[:, idx], v[:, idx]
        if nt:
            kg, vg = torch.cat([kg, t("text_k")], 1), torch.cat([vg, t("text_v")], 1)
        sl = slice(r * S_r, (r + 1) * S_r)
        out = lvsa_sdpa(q[:, sl], k[:, sl], v[:, sl], kg, vg, meta)
        torch.cuda.synchronize()
        check_device_errors(dev)
        d = np.abs(out.float().cpu().numpy() - CP[f"{name}.out{r}"])
        assert d.max() <= MAX_ABS_TOL and d.mean() <= MEAN_ABS_TOL, (r, d.max(), d.mean())
