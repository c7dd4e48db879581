"""Reference-compatible context parallelism on the GPU: each rank's output
(video rows and text rows) against the reference's own per-rank output
(tests/golden/cp.npz), within the attention tolerance of tests/gpu_util.py.
Ranks are emulated one after another on one GPU (global K/V assembled by
slicing, which the gloo test shows equals the all-reduce); a 2-GPU NCCL run
checks the collective path."""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import GOLDEN
from tests.gpu_util import MAX_ABS_TOL as MAX_ABS, MEAN_ABS_TOL as MEAN_ABS

pytestmark = pytest.mark.gpu

CP = np.load(os.path.join(GOLDEN, "cp.npz"))
NAMES = sorted({k.split(".")[0] for k in CP.files})


def _t(name, key, dev):
    return torch.from_numpy(CP[f"{name}.{key}"]).to(torch.bfloat16).to(dev)


def _cmp(got, want):
    d = np.abs(got.float().cpu().numpy() - want)
    assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (d.max(), d.mean())


@pytest.mark.parametrize("name", NAMES)
def test_cp_ranks_match_reference(name):
    from longvideosparseattention_b200.cp_mode import build_shard_pattern, cp_attend
    from longvideosparseattention_b200 import check_device_errors
    dev = torch.device("cuda")
    T, P, H, Hkv, D, W, nf, kfi, off, nt, world, _ = [int(x) for x in CP[f"{name}.params"]]
    q, k, v = _t(name, "q", dev), _t(name, "k", dev), _t(name, "v", dev)
    tq, tk, tv = (_t(name, x, dev) if nt else None for x in ("text_q", "text_k", "text_v"))
    S_r = T * P // world
    for r in range(world):
        pat = build_shard_pattern(T, P, W, nf, kfi, off, r, world, nt, device=dev)
        idx = torch.cat([torch.arange(g * P, (g + 1) * P) for g in pat.global_indices]).to(dev)
        kg, vg = k[:, idx], v[:, idx]
        if nt:
            kg, vg = torch.cat([kg, tk], 1), torch.cat([vg, tv], 1)
        sl = slice(r * S_r, (r + 1) * S_r)
        qr = q[:, sl].clone()
        out, tout = cp_attend(qr, k[:, sl], v[:, sl], pat, kg, vg, tq, tk, tv)
        torch.cuda.synchronize()
        check_device_errors(dev)
        _cmp(out, CP[f"{name}.out{r}"])
        assert torch.equal(qr, q[:, sl])  # the text-row launch leaves the video rows alone
        if nt:
            _cmp(tout, CP[f"{name}.text_out{r}"])


def _worker(rank, world, port, out_dir):
    os.environ.update(NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # File rendezvous: no TCP port to race for between back-to-back tests.
    dist.init_process_group("nccl", init_method="file://" + port, rank=rank, world_size=world, device_id=dev)
    try:
        from longvideosparseattention_b200.cp_mode import GlobalKV, build_shard_pattern, cp_attention
        name = "cp_w2"
        T, P, H, Hkv, D, W, nf, kfi, off, nt, _, _ = [int(x) for x in CP[f"{name}.params"]]
        S_r = T * P // world
        sl = slice(rank * S_r, (rank + 1) * S_r)
        q, k, v = (_t(name, x, dev)[:, sl].contiguous() for x in ("q", "k", "v"))
        tq, tk, tv = (_t(name, x, dev) for x in ("text_q", "text_k", "text_v"))
        pat = build_shard_pattern(T, P, W, nf, kfi, off, rank, world, nt, device=dev)
        out, tout = cp_attention(q, k, v, pat, GlobalKV(), tq, tk, tv)
        torch.cuda.synchronize()
        torch.save({"out": out.cpu(), "tout": tout.cpu()}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_cp_two_gpus_nccl(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_worker, args=(2, os.path.join(str(tmp_path), "rdzv"), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(os.path.join(tmp_path, f"r{r}.pt"))
        _cmp(res["out"], CP[f"cp_w2.out{r}"])
        _cmp(res["tout"], CP[f"cp_w2.text_out{r}"])
