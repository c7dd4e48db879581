"""Reference-compatible context parallelism, host side: the per-rank tile
CSRs against a token-level brute force over the oracle's frame structures,
the global frames against the reference (tests/golden/cp.npz), and the
global K/V assembly with a real all_reduce over gloo (world 2 and 3)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import lvsa_oracle as O
from tests.conftest import GOLDEN

CP = np.load(os.path.join(GOLDEN, "cp.npz"))
NAMES = sorted({k.split(".")[0] for k in CP.files})


def _brute(T, P, W, nf, kfi, off, r, world, n_dense, BQ=128, BK=128):
    """Token-level expectation: tile (qt, kt) active iff some query token's
    frame allows some key token's frame (window minus globals, on this rank);
    flagged unless every pair is allowed and the tile is whole."""
    S_r = T * P // world
    gts = r * S_r
    guards = O.compute_boundary_guard_frames(T, S_r, P, world, W)
    fp = O.frame_pattern(T, P, W, nf, kfi, off, True, r, world, boundary_guards=guards)
    gset = set(np.nonzero(fp["global_frame_mask"])[0].tolist())
    allowed = {}
    for f in range(T):
        lo, hi = fp["window_bounds"][f]
        allowed[f] = {g for g in range(int(lo), int(hi) + 1) if g not in gset}
    fr = (gts + np.arange(S_r)) // P
    nq, nk = -(-S_r // BQ), -(-S_r // BK)
    ndt = -(-n_dense // BK)
    rows = []
    for qt in range(nq):
        qs = set(fr[qt * BQ:(qt + 1) * BQ].tolist())
        row = []
        for kt in range(nk):
            ks = set(fr[kt * BK:(kt + 1) * BK].tolist())
            pairs = [g in allowed[f] for f in qs for g in ks]
            if any(pairs):
                row.append((kt, 0 if all(pairs) and (kt + 1) * BK <= S_r else 1))
        row += [(nk + j, 1 if (j + 1) * BK > n_dense else 0) for j in range(ndt)]
        rows.append(row)
    return rows, sorted(gset)


@pytest.mark.parametrize("name", NAMES)
def test_shard_csr_matches_token_level_definition(name):
    from longvideosparseattention_b200.cp_mode import build_shard_pattern
    T, P, H, Hkv, D, W, nf, kfi, off, nt, world, _ = [int(x) for x in CP[f"{name}.params"]]
    for r in range(world):
        pat = build_shard_pattern(T, P, W, nf, kfi, off, r, world, nt, device=torch.device("cpu"))
        assert pat.global_indices == CP[f"{name}.globals{r}"].tolist()
        n_dense = len(pat.global_indices) * P + nt
        want, gl = _brute(T, P, W, nf, kfi, off, r, world, n_dense)
        assert gl == pat.global_indices
        m = pat.video
        ip, ix, fl = m.tile_indptr.numpy(), m.tile_indices.numpy(), m.tile_flags.numpy()
        for qt, row in enumerate(want):
            got = list(zip(ix[ip[qt]:ip[qt + 1]].tolist(), fl[ip[qt]:ip[qt + 1]].tolist()))
            assert got == row, (name, r, qt)
        assert m.token_offset == r * (T * P // world) and m.first_q_tile == 0
        if nt:
            assert pat.text.first_q_tile == m.n_q_video_tiles


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, name, q_ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from longvideosparseattention_b200.cp_mode import GlobalKV, build_shard_pattern
        T, P, H, Hkv, D, W, nf, kfi, off, nt, _, _ = [int(x) for x in CP[f"{name}.params"]]
        k, v = torch.from_numpy(CP[f"{name}.k"]), torch.from_numpy(CP[f"{name}.v"])
        tk, tv = torch.from_numpy(CP[f"{name}.text_k"]), torch.from_numpy(CP[f"{name}.text_v"])
        S_r = T * P // world
        pat = build_shard_pattern(T, P, W, nf, kfi, off, rank, world, nt, device=torch.device("cpu"))
        kv = GlobalKV()
        buf = kv.fill(k[:, rank * S_r:(rank + 1) * S_r], v[:, rank * S_r:(rank + 1) * S_r], pat)
        dist.all_reduce(buf, op=dist.ReduceOp.SUM)
        kg, vg = kv.finish(pat, tk if nt else None, tv if nt else None)
        idx = torch.cat([torch.arange(g * P, (g + 1) * P) for g in pat.global_indices])
        want_k, want_v = k[:, idx], v[:, idx]
        if nt:
            want_k, want_v = torch.cat([want_k, tk], 1), torch.cat([want_v, tv], 1)
        q_ret.put((rank, bool(torch.equal(kg, want_k) and torch.equal(vg, want_v))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["cp_w2", "cp_w3_mid"])
def test_global_kv_allreduce_gloo(name):
    world = int(CP[f"{name}.params"][10])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(res.values()), res
