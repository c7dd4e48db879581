"""Ulysses head parallelism on 2-4 GPUs (NCCL): every rank's output shard
equals the single-GPU kernel output, bitwise, for whole-head schedules and
for head-and-tile schedules (head count not divisible by the GPU count, GQA).
The piece-by-piece launches themselves are checked on one GPU as well (the
ranks' schedules emulated one after another).  The multi-GPU cases skip with
fewer than 2 GPUs."""

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


CASES = [dict(T=9, P=230, H=4, Hkv=4, D=128, W=1, kfi=4, off=1, nt=40),
         dict(T=9, P=230, H=3, Hkv=3, D=128, W=1, kfi=4, off=1, nt=40),    # 3 heads on 2 / 4 GPUs
         dict(T=8, P=300, H=6, Hkv=2, D=128, W=2, kfi=3, off=2, nt=0),     # GQA, 6 heads on 4 GPUs
         dict(T=10, P=250, H=5, Hkv=5, D=64, W=1, kfi=4, off=0, nt=130)]   # D = 64


def _inputs(device, c):
    g = torch.Generator().manual_seed(5)
    mk = lambda n, h: (torch.randn(1, n, h, c["D"], generator=g) / c["D"] ** 0.25).to(torch.bfloat16).to(device)
    N = c["T"] * c["P"]
    return (mk(N, c["H"]), mk(N, c["Hkv"]), mk(N, c["Hkv"]),
            mk(c["nt"], c["H"]), mk(c["nt"], c["Hkv"]), mk(c["nt"], c["Hkv"]))


def _worker(rank, world, port, out_dir, c):
    os.environ.update(NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # File rendezvous: no TCP port to race for between back-to-back tests.
    dist.init_process_group("nccl", init_method="file://" + port, rank=rank, world_size=world, device_id=dev)
    try:
        from longvideosparseattention_b200 import build_block_mask
        from longvideosparseattention_b200.ulysses import mask_local_attention, shard_sizes, tile_costs, \
            ulysses_attention
        q, k, v, tq, tk, tv = _inputs(dev, c)
        nt = c["nt"]
        sizes = shard_sizes(c["T"] * c["P"], world)
        a = sum(sizes[:rank])
        sl = slice(a, a + sizes[rank])
        mask = build_block_mask(c["T"], c["P"], c["W"], 1, c["kfi"], c["off"], True, nt, device=dev)
        out, tout = ulysses_attention(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(),
                                      sizes, mask_local_attention(mask), tq if nt else None,
                                      tk if nt else None, tv if nt else None,
                                      n_q_tiles=mask.n_q_tiles, costs=tile_costs(mask))
        torch.cuda.synchronize()
        torch.save({"out": out.cpu(), "tout": None if tout is None else tout.cpu()},
                   os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _single_gpu(c, dev):
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask
    q, k, v, tq, tk, tv = _inputs(dev, c)
    nt = c["nt"]
    mask = build_block_mask(c["T"], c["P"], c["W"], 1, c["kfi"], c["off"], True, nt, device=dev)
    return block_sparse_attention(q, k, v, mask, *((tq, tk, tv) if nt else (None, None, None)))


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_schedule_pieces_emulated_on_one_gpu(ci, world):
    """Every rank's pieces launched with q_tiles ranges on one GPU cover the
    output exactly once and equal the single launch bitwise."""
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask, check_device_errors
    from longvideosparseattention_b200.ulysses import make_schedule, tile_costs
    c = CASES[ci]
    dev = torch.device("cuda", 0)
    q, k, v, tq, tk, tv = _inputs(dev, c)
    nt = c["nt"]
    mask = build_block_mask(c["T"], c["P"], c["W"], 1, c["kfi"], c["off"], True, nt, device=dev)
    sch = make_schedule(c["H"], c["Hkv"], world, mask.n_q_tiles, tile_costs(mask))
    g = c["H"] // c["Hkv"]
    out = torch.full_like(q, float("nan"))
    tout = torch.full_like(tq, float("nan")) if nt else None
    for r in range(world):
        for p in sch.pieces[r]:
            hk = slice(p.h0 // g, (p.h1 - 1) // g + 1)
            block_sparse_attention(q[:, :, p.h0:p.h1], k[:, :, hk], v[:, :, hk], mask,
                                   tq[:, :, p.h0:p.h1] if nt else None, tk[:, :, hk] if nt else None,
                                   tv[:, :, hk] if nt else None, out=out[:, :, p.h0:p.h1],
                                   text_out=tout[:, :, p.h0:p.h1] if nt else None, q_tiles=(p.t0, p.t1))
    torch.cuda.synchronize()
    check_device_errors(dev)
    ref, tref = _single_gpu(c, dev)
    assert torch.equal(out, ref)
    if nt:
        assert torch.equal(tout, tref)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_ulysses_multi_gpu_match_single_gpu(tmp_path, ci, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    c = CASES[ci]
    mp.spawn(_worker, args=(world, os.path.join(str(tmp_path), "rdzv"), str(tmp_path), c), nprocs=world, join=True)
    ref, tref = _single_gpu(c, torch.device("cuda", 0))
    got = torch.cat([torch.load(tmp_path / f"r{r}.pt")["out"] for r in range(world)], dim=1)
    assert torch.equal(got, ref.cpu())  # same kernel on the same per-head rows: bitwise
    if c["nt"]:
        for r in range(world):
            assert torch.equal(torch.load(tmp_path / f"r{r}.pt")["tout"], tref.cpu())
