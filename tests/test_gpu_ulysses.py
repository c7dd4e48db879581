"""Ulysses head parallelism on 2 GPUs (NCCL): every rank's output shard equals
the single-GPU kernel output.  Skipped with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


CASE = dict(T=9, P=230, H=4, D=128, W=1, kfi=4, off=1, nt=40)


def _inputs(device):
    c = CASE
    g = torch.Generator().manual_seed(5)
    mk = lambda n: (torch.randn(1, n, c["H"], c["D"], generator=g) / c["D"] ** 0.25).to(torch.bfloat16).to(device)
    N = c["T"] * c["P"]
    return mk(N), mk(N), mk(N), mk(c["nt"]), mk(c["nt"]), mk(c["nt"])


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from longvideosparseattention_b200.sparse_attention import LVSAMetadata
        from longvideosparseattention_b200.ulysses import kernel_local_attention, shard_sizes, ulysses_attention
        c = CASE
        q, k, v, tq, tk, tv = _inputs(dev)
        sizes = shard_sizes(c["T"] * c["P"], world)
        a = sum(sizes[:rank])
        sl = slice(a, a + sizes[rank])
        meta = LVSAMetadata.build(c["T"], c["P"], c["W"], 1, c["kfi"], 0, 1, keyframe_offset=c["off"])
        out, tout = ulysses_attention(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(),
                                      sizes, kernel_local_attention(meta), tq, tk, tv)
        torch.cuda.synchronize()
        torch.save({"out": out.cpu(), "tout": tout.cpu()}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_ulysses_two_gpus_match_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    mp.spawn(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    from longvideosparseattention_b200.sparse_attention import LVSAMetadata, lvsa_attention
    c = CASE
    q, k, v, tq, tk, tv = _inputs(torch.device("cuda", 0))
    meta = LVSAMetadata.build(c["T"], c["P"], c["W"], 1, c["kfi"], 0, 1, keyframe_offset=c["off"])
    ref, tref = lvsa_attention(q, k, v, meta, tq, tk, tv)
    got = torch.cat([torch.load(tmp_path / f"r{r}.pt")["out"] for r in range(world)], dim=1)
    assert torch.equal(got, ref.cpu())  # same kernel on the same per-head data: bitwise
    for r in range(world):
        assert torch.equal(torch.load(tmp_path / f"r{r}.pt")["tout"], tref.cpu())
