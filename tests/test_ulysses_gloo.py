"""Ulysses head-parallel plumbing on CPU ranks (gloo, world 2-4): every
rank's output shard equals the world = 1 oracle rows.  The local attention
step is the oracle here, restricted to the piece's tile rows (the CUDA
kernel's own parity is covered by the GPU tests); this pins the schedule
(whole heads, and heads split into tile-row ranges when the world does not
divide the head count), GQA head ranges, the all-to-all packing, uneven
shards and the text-row sum."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import lvsa_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


BQ = 128


def _case(B, T, P, H, Hkv, D, nt, seed=0):
    g = torch.Generator().manual_seed(seed)
    mk = lambda n, h: torch.randn(B, n, h, D, generator=g)
    return (mk(T * P, H), mk(T * P, Hkv), mk(T * P, Hkv), mk(nt, H), mk(nt, Hkv), mk(nt, Hkv))


def _worker(rank, world, port, B, T, P, H, Hkv, D, nt, W, kfi, off, q_ret, uniform):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from longvideosparseattention_b200.ulysses import shard_sizes, ulysses_attention
        q, k, v, tq, tk, tv = _case(B, T, P, H, Hkv, D, nt)
        sizes = shard_sizes(T * P, world)
        a = sum(sizes[:rank])
        sl = slice(a, a + sizes[rank])
        fp = O.frame_pattern(T, P, W, 1, kfi, off)
        N = T * P
        nqv = -(-N // BQ)
        nq = nqv + -(-nt // BQ)
        costs = [1 + ((7 * i) % 5) for i in range(nq)] if not uniform else None

        def local(qf, kf, vf, tq_, tk_, tv_, q_tiles, out, text_out):
            o, to = O.attention(qf.numpy(), kf.numpy(), vf.numpy(), fp,
                                None if tq_ is None else tq_.numpy(),
                                None if tk_ is None else tk_.numpy(),
                                None if tv_ is None else tv_.numpy())
            t0, t1 = q_tiles
            s, e = min(t0, nqv) * BQ, min(min(t1, nqv) * BQ, N)
            if e > s:
                out[:, s:e] = torch.from_numpy(o[:, s:e])
            if text_out is not None:
                s, e = max(t0 - nqv, 0) * BQ, min(max(t1 - nqv, 0) * BQ, nt)
                if e > s:
                    text_out[:, s:e] = torch.from_numpy(to[:, s:e])

        out, tout = ulysses_attention(q[:, sl], k[:, sl], v[:, sl], sizes, local,
                                      tq if nt else None, tk if nt else None, tv if nt else None,
                                      n_q_tiles=nq, costs=costs)
        q_ret.put((rank, out.numpy(), None if tout is None else tout.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B,T,P,H,Hkv,nt,uniform", [
    (2, 1, 7, 10, 4, 4, 6, True),        # whole heads
    (3, 1, 5, 11, 6, 6, 0, True),
    (2, 2, 6, 9, 2, 2, 5, True),         # batch 2
    (2, 1, 6, 100, 3, 3, 150, False),    # 3 heads on 2 ranks: one head split by tile rows
    (4, 1, 7, 90, 6, 3, 200, False),     # GQA, 6 heads on 4 ranks
    (3, 2, 5, 80, 4, 2, 70, True),       # GQA, batch 2, 4 heads on 3 ranks
    (4, 1, 5, 120, 2, 1, 0, False),      # fewer heads than ranks
])
def test_ulysses_matches_world1(world, B, T, P, H, Hkv, nt, uniform):
    D, W, kfi, off = 16, 1, 3, 1
    ctx = mp.get_context("spawn")
    qret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, T, P, H, Hkv, D, nt, W, kfi, off, qret,
                                               uniform))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, o, to = qret.get(timeout=180)
        res[r] = (o, to)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, tq, tk, tv = _case(B, T, P, H, Hkv, D, nt)
    fp = O.frame_pattern(T, P, W, 1, kfi, off)
    want, twant = O.attention(q.numpy(), k.numpy(), v.numpy(), fp,
                              tq.numpy() if nt else None, tk.numpy() if nt else None,
                              tv.numpy() if nt else None)
    got = np.concatenate([res[r][0] for r in range(world)], axis=1)
    np.testing.assert_allclose(got, want, atol=1e-5, rtol=1e-5)
    for r in range(world):
        if nt:
            np.testing.assert_allclose(res[r][1], twant, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("H,Hkv,world,nq", [(12, 12, 8, 988), (16, 16, 3, 611), (48, 48, 5, 520),
                                            (6, 2, 4, 37), (8, 2, 3, 20), (3, 3, 8, 5), (12, 4, 8, 99)])
def test_schedule_covers_every_unit_once_and_balances(H, Hkv, world, nq):
    from longvideosparseattention_b200.ulysses import make_schedule
    costs = [1 + (i * 37) % 11 for i in range(nq)]
    sch = make_schedule(H, Hkv, world, nq, costs)
    seen = np.zeros((H, nq), dtype=np.int32)
    g = H // Hkv
    for r in range(world):
        qa, qb = sch.q_heads[r]
        ka, kb = sch.kv_range[r]
        for p in sch.pieces[r]:
            seen[p.h0:p.h1, p.t0:p.t1] += 1
            assert qa <= p.h0 < p.h1 <= qb
            assert ka <= p.h0 // g and (p.h1 - 1) // g < kb
            # one launch maps its query heads onto its K/V heads as enable_gqa
            assert (p.h1 - p.h0) == 1 or (p.h0 % g == 0 and p.h1 % g == 0) or p.h0 // g == (p.h1 - 1) // g
    assert (seen == 1).all()
    total = H * sum(costs)
    loads = [sch.cost(r, costs) for r in range(world)]
    if H % world:
        # equal shares up to one tile row
        assert max(loads) - total / world <= max(costs) + 1e-6
    else:
        assert len(set(loads)) == 1


def test_shard_sizes_uneven():
    from longvideosparseattention_b200.ulysses import shard_sizes
    assert shard_sizes(77910, 4) == [19478, 19478, 19477, 19477]
    assert sum(shard_sizes(77910, 8)) == 77910
