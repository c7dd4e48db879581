"""Ulysses head-parallel plumbing on CPU ranks (gloo, world 2 and 3): every
rank's output shard equals the world = 1 oracle rows.  The local attention
step is the oracle here (the CUDA kernel's own parity is covered by the GPU
tests); this pins the all-to-all packing, uneven shards and the text gather."""

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


def _case(B, T, P, H, D, nt, seed=0):
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g)
    return (mk(B, T * P, H, D), mk(B, T * P, H, D), mk(B, T * P, H, D),
            mk(B, nt, H, D), mk(B, nt, H, D), mk(B, nt, H, D))


def _worker(rank, world, port, B, T, P, H, D, nt, W, kfi, off, q_ret, chunks=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from longvideosparseattention_b200.ulysses import shard_sizes, ulysses_attention
        q, k, v, tq, tk, tv = _case(B, T, P, H, D, nt)
        sizes = shard_sizes(T * P, world)
        a = sum(sizes[:rank])
        sl = slice(a, a + sizes[rank])
        fp = O.frame_pattern(T, P, W, 1, kfi, off)

        def local(qf, kf, vf, tq_, tk_, tv_):
            o, to = O.attention(qf.numpy(), kf.numpy(), vf.numpy(), fp,
                                None if tq_ is None else tq_.numpy(),
                                None if tk_ is None else tk_.numpy(),
                                None if tv_ is None else tv_.numpy())
            return torch.from_numpy(o), (None if to is None else torch.from_numpy(to))

        out, tout = ulysses_attention(q[:, sl], k[:, sl], v[:, sl], sizes, local,
                                      tq if nt else None, tk if nt else None, tv if nt else None,
                                      chunks=chunks)
        q_ret.put((rank, out.numpy(), None if tout is None else tout.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B,T,P,H,nt,chunks", [(2, 1, 7, 10, 4, 6, None), (3, 1, 5, 11, 6, 0, None),
                                                     (2, 2, 6, 9, 2, 5, None), (2, 1, 5, 12, 12, 7, 3),
                                                     (3, 2, 4, 9, 6, 4, 1)])
def test_ulysses_matches_world1(world, B, T, P, H, nt, chunks):
    """Head groups exchanged and computed one after another (chunks) give the
    same rows as one exchange."""
    D, W, kfi, off = 16, 1, 3, 1
    ctx = mp.get_context("spawn")
    qret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, T, P, H, D, nt, W, kfi, off, qret, chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, o, to = qret.get(timeout=120)
        res[r] = (o, to)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, tq, tk, tv = _case(B, T, P, H, D, nt)
    fp = O.frame_pattern(T, P, W, 1, kfi, off)
    want, twant = O.attention(q.numpy(), k.numpy(), v.numpy(), fp,
                              tq.numpy() if nt else None, tk.numpy() if nt else None,
                              tv.numpy() if nt else None)
    from longvideosparseattention_b200.ulysses import shard_sizes
    sizes = shard_sizes(T * P, world)
    got = np.concatenate([res[r][0] for r in range(world)], axis=1)
    np.testing.assert_allclose(got, want, atol=1e-5, rtol=1e-5)
    for r in range(world):
        if nt:
            np.testing.assert_allclose(res[r][1], twant, atol=1e-5, rtol=1e-5)


def test_shard_sizes_uneven():
    from longvideosparseattention_b200.ulysses import shard_sizes
    assert shard_sizes(77910, 4) == [19478, 19478, 19477, 19477]
    assert sum(shard_sizes(77910, 8)) == 77910


def test_heads_must_divide():
    from longvideosparseattention_b200.ulysses import pack_qkv
    x = torch.zeros(1, 4, 12, 8)
    with pytest.raises(ValueError):
        pack_qkv(x, x, x, 8)
