"""LVSA block-sparse attention benchmark (B200, sm_100a).

Default workload ("cfg2"): Wan2.1-1.3B self-attention at
4x horizon -- 81 latent frames x 1560 tokens = 126 360 tokens, 12 heads,
head_dim 128, bf16, anchors = first frame, keyframe stride 4 rotating per
step, window +-2, 128x128 tiles.  One step = one denoising step of the
30-layer model: the GPU mask build for the step plus 30 attention layers,
each on its own seeded q/k/v (N(0,1)/sqrt(128), seeded 3-D RoPE applied).

Metric: useful TFLOP/s (active 128x128 tiles, clipped; BASELINE's FLOP_tiles)
and ms/layer.  Timing: CUDA events on the launching stream, warm-up steps
first, barrier + synchronize around the timed region, max over ranks.  The
30 layers' inputs (35 GB) exceed L2 and are cycled, so no L2 flush is needed.

--impl reference: the reference algorithm's CPU implementation (the oracle
port of lvsa_sdpa) on the host cores, bounded sample per step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "cfg2": dict(T=81, P=1560, H=12, D=128, W=2, n_first=1, kfi=4, step=0, n_text=0, layers=30,
                 desc="Wan2.1-1.3B 4x horizon (81 latent frames x 1560), 12x128, bf16, window +-2, kfi 4"),
    "cfg3": dict(T=121, P=1560, H=12, D=128, W=2, n_first=1, kfi=4, step=0, n_text=0, layers=30,
                 desc="Wan2.1-1.3B 6x horizon (121 x 1560), 12x128, bf16"),
    "cfg4": dict(T=49, P=1590, H=16, D=128, W=2, n_first=1, kfi=4, step=0, n_text=256, layers=30,
                 desc="HunyuanVideo-1.5 49 x 1590 + 256 text, 16x128, bf16"),
    "cfg5": dict(T=49, P=1350, H=48, D=64, W=1, n_first=1, kfi=3, step=0, n_text=226, layers=30,
                 desc="CogVideoX-5B 49 x 1350 + 226 text, 48x64, bf16"),
}
METRIC = "sparse-attn ms/layer & useful TFLOPS (% of B200 peak) at 1/2/4/8 GPUs"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per attention launch, from one ncu capture of a
# full-size layer (dram__bytes_read.sum + dram__bytes_write.sum); null where not captured.
NCU_TRAFFIC_BYTES = {"cfg2": 1.602e9}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def flops_for(cfg):
    """(FLOP_tiles, FLOP_exact) of one layer, from the pattern (host arithmetic)."""
    from longvideosparseattention_b200.sparse_attention import LVSAMetadata, tile_flop_counts
    m = LVSAMetadata.build(cfg["T"], cfg["P"], cfg["W"], cfg["n_first"], cfg["kfi"], 0, 1,
                           keyframe_offset=cfg["step"] % cfg["kfi"])
    return tile_flop_counts(m, cfg["n_text"], cfg["H"], cfg["D"], 128, 128)


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def seeded_layer(cfg, layer, device, gen_device=True):
    """Seeded q/k/v (+ text) of one layer: N(0,1)/sqrt(D) with a seeded 3-D RoPE on q, k."""
    import torch
    T, P, H, D, nt = cfg["T"], cfg["P"], cfg["H"], cfg["D"], cfg["n_text"]
    N = T * P
    g = torch.Generator(device=device).manual_seed(1000 + layer)
    sc = 1.0 / math.sqrt(D)
    q = torch.randn(1, N, H, D, generator=g, device=device) * sc
    k = torch.randn(1, N, H, D, generator=g, device=device) * sc
    v = torch.randn(1, N, H, D, generator=g, device=device) * sc
    q, k = apply_rope3d(q, k, cfg)
    out = [q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)]
    if nt:
        out += [(torch.randn(1, nt, H, D, generator=g, device=device) * sc).to(torch.bfloat16)
                for _ in range(3)]
    return out


def apply_rope3d(q, k, cfg):
    """3-D (t, h, w) rotary embedding on interleaved pairs, split of head_dim as
    in Wan (t: D/2 - 2*(D/6 rounded), h and w: the rest); seeded frequency base."""
    import torch
    T, P, D = cfg["T"], cfg["P"], cfg["D"]
    grid_w = {1560: 52, 1590: 53, 1350: 30}.get(P, P)
    grid_h = P // grid_w
    half = D // 2
    dh = dw = 2 * (half // 6)
    dt = half - dh - dw
    dev = q.device
    t_idx = torch.arange(T, device=dev).repeat_interleave(P)
    hw = torch.arange(P, device=dev).repeat(T)
    h_idx, w_idx = hw // grid_w, hw % grid_w

    def freqs(pos, n):
        inv = 1.0 / (10000 ** (torch.arange(n, device=dev, dtype=torch.float32) / n))
        return pos[:, None].float() * inv[None, :]
    ang = torch.cat([freqs(t_idx, dt), freqs(h_idx, dh), freqs(w_idx, dw)], dim=1)  # [N, D/2]
    cos, sin = ang.cos()[None, :, None, :], ang.sin()[None, :, None, :]

    def rot(x):
        x2 = x.view(*x.shape[:-1], half, 2)
        a, b = x2[..., 0], x2[..., 1]
        return torch.stack([a * cos - b * sin, a * sin + b * cos], dim=-1).flatten(-2)
    return rot(q), rot(k)


def run_b200(args, cfg):
    import torch
    import torch.distributed as dist
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask, check_device_errors

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    L = cfg["layers"]
    T, P, H, D, nt = cfg["T"], cfg["P"], cfg["H"], cfg["D"], cfg["n_text"]
    flop_tiles, flop_exact = flops_for(cfg)
    ulysses = args.parallel == "ulysses" and world > 1
    refcp = args.parallel == "cp" and world > 1
    if refcp:
        # Strong scaling with the reference's own world > 1 pattern: each rank
        # holds its token shard; global frames (keyframes + boundary guards)
        # are gathered by one NCCL all-reduce per layer, windows stay local.
        from longvideosparseattention_b200.cp_mode import GlobalKV, build_shard_pattern, cp_attention
        if (T * P) % world:
            raise SystemExit(f"reference CP needs T*P ({T * P}) divisible by the GPU count ({world})")
        S_r = T * P // world
        shard = build_shard_pattern(T, P, cfg["W"], cfg["n_first"], cfg["kfi"], cfg["step"] % cfg["kfi"],
                                    rank, world, nt, device=dev)
        gkv = GlobalKV()
        layers = []
        for i in range(L):
            lay = seeded_layer(cfg, i, dev)
            lay[:3] = [x[:, rank * S_r:(rank + 1) * S_r].contiguous() for x in lay[:3]]
            layers.append(lay)
            del lay
        torch.cuda.empty_cache()
        # Useful FLOPs of this rank's pattern (clipped tile areas, dense terms exact), summed over ranks.
        ip, ix = shard.video.tile_indptr.cpu().numpy(), shard.video.tile_indices.cpu().numpy()
        area = 0
        for qt in range(shard.video.n_q_video_tiles):
            rows_q = min(S_r, (qt + 1) * 128) - qt * 128
            for kt in ix[ip[qt]:ip[qt + 1]]:
                if kt < shard.video.n_k_video_tiles:
                    area += rows_q * (min(S_r, (int(kt) + 1) * 128) - int(kt) * 128)
        n_dense = len(shard.global_indices) * P + nt
        cp_flop = 4 * D * H * (area + S_r * n_dense + nt * (S_r + nt))
        tt = torch.tensor([cp_flop], dtype=torch.float64, device=dev)
        dist.all_reduce(tt)
        flop_tiles = float(tt.item())
    elif ulysses:
        # Strong scaling: the same 30 layers on every N; each rank holds its
        # contiguous token shard of q/k/v (heads are scattered by all-to-all).
        from longvideosparseattention_b200.ulysses import mask_local_attention, shard_sizes, ulysses_attention
        sizes = shard_sizes(T * P, world)
        a0 = sum(sizes[:rank])
        layers = []
        for i in range(L):
            lay = seeded_layer(cfg, i, dev)
            lay[:3] = [x[:, a0:a0 + sizes[rank]].contiguous() for x in lay[:3]]
            layers.append(lay)
            del lay
        torch.cuda.empty_cache()
    else:
        layers = [seeded_layer(cfg, rank * L + i, dev) for i in range(L)]
    outs = [torch.empty_like(layers[0][0]) for _ in range(2)]
    touts = [torch.empty_like(layers[0][3]) for _ in range(2)] if nt else [None, None]
    stream = torch.cuda.current_stream(dev)
    mask = build_block_mask(T, P, cfg["W"], cfg["n_first"], cfg["kfi"], cfg["step"] % cfg["kfi"],
                            True, nt, device=dev)
    phases = []
    if ulysses:
        # Work units (head, tile row) weighted by the row's key-tile count; the
        # pattern is fixed for the step, so the schedule is made once.
        from longvideosparseattention_b200.ulysses import make_schedule, tile_costs
        sched = make_schedule(H, H, world, mask.n_q_tiles, tile_costs(mask))
        local_attn = mask_local_attention(mask)
        if rank == 0:
            log(f"ulysses x{world}: pieces of rank 0 {sched.pieces[0]}")

    def step(s, ev=None):
        nonlocal mask
        mask = build_block_mask(T, P, cfg["W"], cfg["n_first"], cfg["kfi"],
                                cfg["step"] % cfg["kfi"], True, nt, device=dev, reuse=mask)
        for i, lay in enumerate(layers):
            if ev is not None:
                ev[i][0].record(stream)
            tx = (lay[3], lay[4], lay[5]) if nt else (None, None, None)
            if refcp:
                cp_attention(lay[0], lay[1], lay[2], shard, gkv, *tx)
            elif ulysses:
                tm = {} if ev is not None else None
                ulysses_attention(lay[0], lay[1], lay[2], sizes, local_attn, *tx, schedule=sched, timing=tm)
                if tm is not None:
                    phases.append(tm)
            else:
                block_sparse_attention(lay[0], lay[1], lay[2], mask, *tx, out=outs[i & 1], text_out=touts[i & 1],
                                       fp8=args.fp8)
            if ev is not None:
                ev[i][1].record(stream)

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    check_device_errors(dev)

    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
           for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for s in range(args.steps):
            step(s, evs[s])
        stop.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    check_device_errors(dev)
    ms = start.elapsed_time(stop)
    kern_ms = [a.elapsed_time(b) for e in evs for (a, b) in e]
    phase_ms = None
    if phases:
        names = ["start", "packed", "exchanged", "attended", "returned", "done"]
        acc = {n: [] for n in ("pack", "all_to_all_qkv", "attention", "return", "finish")}
        for tm in phases:
            for key, (a_, b_) in zip(acc, zip(names[:-1], names[1:])):
                acc[key].append(tm[a_].elapsed_time(tm[b_]))
        pm = torch.tensor([statistics.mean(v) for v in acc.values()], device=dev)
        if world > 1:
            dist.all_reduce(pm, op=dist.ReduceOp.MAX)
        phase_ms = {k: round(float(x), 4) for k, x in zip(acc, pm.tolist())}
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_step = ms_max / args.steps
    total_flop = flop_tiles * L * args.steps * (1 if (ulysses or refcp) else world)
    value = total_flop / (ms_max * 1e-3) / 1e12

    fp8_peak = measure_fp8_peak(dev) if (args.fp8 and rank == 0 and not args.no_peak) else None

    # ---- e2e through the public API with pinned host buffers (copies inside the timed region)
    e2e = None
    if not args.no_e2e and not (ulysses or refcp):
        e2e = run_e2e(args, cfg, dev, world, flop_tiles)
    elif not args.no_e2e and ulysses:
        e2e = run_e2e_ulysses(args, cfg, dev, world, rank, flop_tiles, sizes, sched, local_attn)

    if rank == 0:
        pk, pk_kind = peaks()
        mean_launch = statistics.mean(kern_ms)
        # per timed layer call: H/world heads under Ulysses (all-to-all included)
        kernel_ms = phase_ms["attention"] if phase_ms else mean_launch
        achieved = flop_tiles / (world if (ulysses or refcp) else 1) / (kernel_ms * 1e-3) / 1e12
        peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
        peak_source = f"{pk_kind} bf16_tflops_sustained (kernel runs back-to-back in a long step)"
        if args.fp8 and fp8_peak:
            peak = fp8_peak
            peak_source = ("measured in this run: cuBLASLt E4M3 GEMM (torch._scaled_mm, 8192^3, "
                           "back to back for 4 s, sustained under the power cap)")
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "ms_per_layer": round(ms_step / L, 4), "higher_is_better": True,
            "scaling": "strong" if (ulysses or refcp) else "weak",
            "vs_baseline": None, "dtype": "e4m3 (QK, PV; fp32 accumulate)" if args.fp8 else "bf16",
            "data": "synthetic (seeded N(0,1)/sqrt(D), RoPE-3D)",
            "config": bench_config(args, cfg, world, flop_tiles, flop_exact),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "traffic": NCU_TRAFFIC_BYTES.get(args.config),
                         "algorithmic_bytes": 4 * T * P * H * D * 2 + 4 * nt * H * D * 2,
                         "peak_source": peak_source, "mean_launch_ms": round(kernel_ms, 4)},
            "clocks": clk.summary(),
            "gpu_launches": (4 + L * (7 if args.fp8 else (2 if refcp and nt else
                                                        (len(sched.pieces[0]) + 3 if ulysses else 1)))) * args.steps,
            "e2e": e2e,
        }
        if phase_ms:
            line["ulysses_phases_ms_per_layer"] = phase_ms
            line["nccl"] = {"backend": "nccl", "world": world, "version": ".".join(map(str, torch.cuda.nccl.version()))}
        if args.cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, flop_tiles, budget_s=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_fp8_peak(dev, seconds=4.0, n=8192):
    """Sustained dense E4M3 GEMM rate of this GPU (cuBLASLt through
    torch._scaled_mm, bf16 output), the FP8 roofline denominator."""
    import torch
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)
    mm = lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    for _ in range(3):
        mm()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0, it = time.perf_counter(), 0
    e0.record()
    while time.perf_counter() - t0 < seconds:
        for _ in range(20):
            mm()
        it += 20
        torch.cuda.synchronize()
    e1.record()
    torch.cuda.synchronize()
    return round(2 * n ** 3 * it / (e0.elapsed_time(e1) * 1e-3) / 1e12, 1)


def run_e2e(args, cfg, dev, world, flop_tiles):
    """Public-API path with host tensors (``pipeline.attention_from_host``):
    per layer, H2D of q/k/v(+text) from pinned memory, the attention call, D2H
    of the output, all in the timed region; the copies of neighbouring layers
    overlap the kernel on separate streams."""
    import torch
    from longvideosparseattention_b200 import build_block_mask
    from longvideosparseattention_b200.pipeline import attention_from_host
    L, nt = cfg["layers"], cfg["n_text"]
    host = []
    for i in range(2):  # two distinct pinned layer inputs, cycled
        lay = seeded_layer(cfg, 10_000 + i, dev)
        host.append([x.cpu().pin_memory() for x in lay])
        del lay
    out_h = torch.empty(host[0][0].shape, dtype=torch.bfloat16).pin_memory()
    tout_h = torch.empty(host[0][3].shape, dtype=torch.bfloat16).pin_memory() if nt else None
    stream = torch.cuda.current_stream(dev)
    h2d = sum(x.numel() * x.element_size() for x in host[0])
    d2h = out_h.numel() * 2 + (tout_h.numel() * 2 if nt else 0)

    def step():
        mask = build_block_mask(cfg["T"], cfg["P"], cfg["W"], cfg["n_first"], cfg["kfi"],
                                cfg["step"] % cfg["kfi"], True, nt, device=dev)
        ins = [tuple(host[i & 1]) if nt else tuple(host[i & 1][:3]) + (None, None, None) for i in range(L)]
        attention_from_host(ins, mask, [(out_h, tout_h)] * L, dev)
        return mask

    steps = max(1, min(args.steps, 3))
    for _ in range(max(1, min(args.warmup, 3))):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    val = flop_tiles * L * steps * world / (ms * 1e-3) / 1e12
    return {"value": round(val, 2), "unit": "TFLOP/s", "ms_per_layer": round(ms / steps / L, 3),
            "h2d_bytes_per_step": h2d * L, "d2h_bytes_per_step": d2h * L, "steps": steps}


def run_e2e_ulysses(args, cfg, dev, world, rank, flop_tiles, sizes, sched, local_attn):
    """Ulysses through the public calls with this rank's token shard in pinned
    host memory: per layer, H2D of the q/k/v (+text) shard, the head-parallel
    layer (both all-to-alls inside), D2H of the output shard, neighbouring
    layers' copies overlapped (``pipeline.attention_from_host``); all in the
    timed region, max over ranks."""
    import torch
    import torch.distributed as dist
    from longvideosparseattention_b200.pipeline import attention_from_host
    from longvideosparseattention_b200.ulysses import ulysses_attention
    L, nt = cfg["layers"], cfg["n_text"]
    a0 = sum(sizes[:rank])
    host = []
    for i in range(2):
        lay = seeded_layer(cfg, 10_000 + i, dev)
        lay[:3] = [x[:, a0:a0 + sizes[rank]] for x in lay[:3]]
        host.append([x.cpu().pin_memory() for x in lay])
        del lay
    out_h = torch.empty(host[0][0].shape, dtype=torch.bfloat16).pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in host[0])
    d2h = out_h.numel() * 2 + (host[0][3].numel() * 2 if nt else 0)
    tout_h = torch.empty(host[0][3].shape, dtype=torch.bfloat16).pin_memory() if nt else None

    def layer(q, k, v, tq, tk, tv):
        return ulysses_attention(q, k, v, sizes, local_attn, tq, tk, tv, schedule=sched)

    def step():
        ins = [tuple(host[i & 1]) if nt else tuple(host[i & 1][:3]) + (None, None, None) for i in range(L)]
        attention_from_host(ins, None, [(out_h, tout_h)] * L, dev, layer_fn=layer)

    steps = max(1, min(args.steps, 2))
    step()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": round(flop_tiles * L * steps / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "ms_per_layer": round(ms / steps / L, 3), "h2d_bytes_per_step": h2d * L * world,
            "d2h_bytes_per_step": d2h * L * world, "steps": steps,
            "path": "ulysses_attention on per-rank pinned host shards through pipeline.attention_from_host "
                    "(H2D of layer i+1 and D2H of layer i-1 overlap layer i)"}


_CPU_INPUTS = {}


def _cpu_setup(cfg, threads):
    import torch
    from oracle import lvsa_oracle as O
    T, P, H, D, nt = cfg["T"], cfg["P"], cfg["H"], cfg["D"], cfg["n_text"]
    key = (T, P, H, D, nt)
    torch.set_num_threads(threads)
    if key not in _CPU_INPUTS:
        g = torch.Generator().manual_seed(0)
        sc = 1.0 / math.sqrt(D)
        mk = lambda n: torch.randn(1, n, H, D, generator=g) * sc
        _CPU_INPUTS[key] = (mk(T * P), mk(T * P), mk(T * P), mk(nt) if nt else None, mk(nt) if nt else None)
    fp = O.frame_pattern(T, P, cfg["W"], cfg["n_first"], cfg["kfi"], cfg["step"] % cfg["kfi"])
    return _CPU_INPUTS[key], fp


def frame_flops(cfg, fp, f):
    """Useful FLOPs of query frame f on the CPU path: 4 D H P x (its keys)."""
    P, H, D, nt = cfg["P"], cfg["H"], cfg["D"], cfg["n_text"]
    lo, hi = (int(x) for x in fp["window_bounds"][f])
    win = [w for w in range(lo, hi + 1) if w not in fp["global_set"]]
    keys = (len(fp["global_indices"]) + len(win)) * P + nt
    return 4 * D * H * P * keys


def cpu_sample(cfg, frames, threads):
    """Time the reference's CPU arithmetic (oracle restatement of lvsa_sdpa:
    per-frame K/V concat + torch fp32 SDPA) for `frames` query frames;
    returns (seconds, useful FLOPs of those frames)."""
    from oracle import lvsa_oracle as O
    (q, k, v, tk, tv), fp = _cpu_setup(cfg, threads)
    t0 = time.perf_counter()
    O.attention_torch_cpu(q, k, v, fp, tk, tv, frames=frames)
    return time.perf_counter() - t0, sum(frame_flops(cfg, fp, f) for f in frames)


def _spread(T, n, phase=0):
    """n query frames spread over [0, T), shifted by `phase`."""
    n = max(1, min(T, n))
    return sorted({(int(round(i * T / n)) + phase) % T for i in range(n)})


def cpu_baseline(cfg, flop_tiles, budget_s=15.0):
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    T = cfg["T"]
    t1, _ = cpu_sample(cfg, [T // 2], threads)
    frames = _spread(T, int(budget_s / max(t1, 1e-3)))
    t, fl = cpu_sample(cfg, frames, threads)
    # The CPU computes exactly the attended keys: time a layer at that rate
    # (its exact FLOPs), then report the layer's FLOP_tiles over that time,
    # the unit of the GPU arm's value.
    _, flop_exact = flops_for(cfg)
    layer_s = flop_exact / (fl / t)
    return {"value": round(flop_tiles / layer_s / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "ms_per_layer_extrapolated": round(layer_s * 1e3, 1),
            "sample": f"{len(frames)} of {T} query frames x all heads of one {cfg['desc']} layer "
                      f"({t:.1f} s): lvsa_sdpa restated (K/V concat + torch fp32 CPU SDPA); "
                      "value = the layer's FLOP_tiles / (its exact FLOPs at the measured rate)"}


def run_reference(args, cfg):
    """The reference's CPU implementation of the path (lvsa_sdpa's per-frame
    K/V concat + torch fp32 SDPA, restated by the oracle port) on all host
    cores.  Each step times K_FRAMES query frames (all heads) of one layer,
    a different spread of frames per step.  ``ms_per_step`` is the time
    actually measured per step; ``ms_per_layer`` extrapolates it to the
    layer (its exact FLOPs at the measured rate) and ``value`` is the
    layer's FLOP_tiles over that time, the GPU arm's unit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    K_FRAMES = 3
    flop_tiles, flop_exact = flops_for(cfg)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    T = cfg["T"]
    secs, flops = [], []
    for s in range(args.warmup + args.steps):
        dt, fl = cpu_sample(cfg, _spread(T, K_FRAMES, phase=5 * s), threads)
        if s >= args.warmup:
            secs.append(dt)
            flops.append(fl)
    layer_s = flop_exact / (sum(flops) / sum(secs))   # exact keys at the measured rate
    val = flop_tiles / layer_s / 1e12                   # in the GPU arm's unit (FLOP_tiles / time)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {"impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(secs) * 1e3, 1),
            "ms_per_layer": round(layer_s * 1e3, 1), "extrapolated": True,
            "extrapolation": f"ms_per_layer = the layer's exact FLOPs / the measured rate; each timed step is "
                             f"{K_FRAMES} of {T} query frames",
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1)/sqrt(D))",
            "config": bench_config(args, cfg, world, flop_tiles, flop_exact),
            "cpu_baseline": {"value": round(val, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"{K_FRAMES} query frames (all heads) of one layer per step"},
            "e2e": {"value": round(val, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def bench_config(args, cfg, world, flop_tiles, flop_exact, parallelism=None):
    """The `config` object both arms print (same keys and values for one N)."""
    T, P, H, D, nt = cfg["T"], cfg["P"], cfg["H"], cfg["D"], cfg["n_text"]
    if parallelism is None:
        parallelism = _parallelism(args, world, H)
    return {"workload": args.config, "desc": cfg["desc"], "layers_per_step": cfg["layers"],
            "tokens": T * P + nt, "heads": H, "head_dim": D, "tile": "128x128",
            "flop_tiles_per_layer": flop_tiles, "flop_exact_per_layer": flop_exact,
            "l2": "30 distinct layer inputs (35 GB) cycled: inputs exceed L2, no flush",
            "parallelism": parallelism}


def _parallelism(args, world, H):
    if world > 1 and args.parallel == "ulysses":
        return (f"ulysses x{world} (NCCL all-to-all of q/k/v and of the output; "
                + ("whole heads per rank)" if H % world == 0
                   else "(head, tile-row) units balanced by key-tile count)"))
    if world > 1 and args.parallel == "cp":
        return (f"reference CP x{world} (token shards, global frames by NCCL all-reduce, "
                "rank-local windows; FLOPs of that pattern)")
    return f"replicas x{world} (independent layers per rank)"


def run_prologue(args, cfg):
    """--prologue: the fused QK prologue (norm + rotary, one pass per tensor)
    on q and k of the configuration's shape, against the unfused torch path
    the adapters run otherwise (module norm, then the rotation).  HBM-bound:
    algorithmic bytes = read + write of q and k, plus the rotary tables."""
    import torch
    from longvideosparseattention_b200.prologue import qk_norm_rope
    dev = torch.device("cuda", 0)
    S, H, D = cfg["T"] * cfg["P"], cfg["H"], cfg["D"]
    per_head = args.config != "cfg2" and args.config != "cfg3"
    norm = ("layer_head" if args.config == "cfg5" else "rms_head") if per_head else "rms_row"
    g = torch.Generator(device=dev).manual_seed(7)
    xs = [torch.randn(1, S, H, D, device=dev, generator=g).bfloat16() for _ in range(2)]
    w = (1 + 0.1 * torch.randn(D if per_head else H * D, device=dev, generator=g)).bfloat16()
    b = torch.zeros(D, device=dev, dtype=torch.bfloat16) if norm == "layer_head" else None
    ang = torch.rand(S, D // 2, device=dev, generator=g) * 6.0
    cs, sn = torch.cos(ang), torch.sin(ang)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > L2 between steps

    def fused():
        for x in xs:
            qk_norm_rope(x, norm, w, b, 1e-6, cs, sn)

    cos_full, sin_full = cs.repeat_interleave(2, -1)[None, :, None, :], sn.repeat_interleave(2, -1)[None, :, None, :]

    def unfused():
        for x in xs:
            if norm == "rms_row":
                y = torch.nn.functional.rms_norm(x.flatten(2), (H * D,), w, 1e-6).unflatten(2, (H, D))
            elif norm == "rms_head":
                y = torch.nn.functional.rms_norm(x, (D,), w, 1e-6)
            else:
                y = torch.nn.functional.layer_norm(x, (D,), w, b, 1e-6)
            x1, x2 = y.unflatten(-1, (-1, 2)).unbind(-1)
            out = torch.empty_like(y)
            out[..., 0::2] = x1 * cos_full[..., 0::2] - x2 * sin_full[..., 1::2]
            out[..., 1::2] = x1 * sin_full[..., 1::2] + x2 * cos_full[..., 0::2]
            x.copy_(out)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        times = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        return sorted(times)[len(times) // 2]

    with ClockSampler(0) as sampler:
        ms = timed(fused)
    clocks = sampler.summary()
    ms_unfused = timed(unfused)
    nbytes = 2 * (2 * S * H * D * 2) + 2 * S * (D // 2) * 4 * 2  # q, k read + write; cos/sin per tensor
    pk, src = peaks()
    gbs = nbytes / ms / 1e6
    print(json.dumps({
        "metric": "qk-prologue (norm + RoPE of q and k) GB/s", "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.config} q,k prologue", "tokens": S, "heads": H, "head_dim": D,
                   "norm": norm, "l2": "256 MB written between steps (flush)"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": None, "algorithmic_bytes": nbytes,
                     "peak_source": f"{src} hbm_gbs"},
        "unfused_torch_ms": round(ms_unfused, 4), "speedup_vs_unfused": round(ms_unfused / ms, 2),
        "clocks": clocks, "gpu_launches": 2 * args.steps}), flush=True)


def run_out_proj(args, cfg):
    """--out-proj: the to_out projection of the configuration's attention
    output (tokens x H*D -> H*D, Wan / HunyuanVideo / CogVideoX model dim)
    on the tcgen05 GEMM (lvsa_out_proj), against torch's Linear (cuBLAS) on
    the same operands.  Inputs larger than L2 (the attention output)."""
    import torch
    import torch.nn.functional as F
    from longvideosparseattention_b200.out_proj import out_projection
    dev = torch.device("cuda", 0)
    S, H, D = cfg["T"] * cfg["P"], cfg["H"], cfg["D"]
    K = Nout = H * D
    g = torch.Generator(device=dev).manual_seed(3)
    o = torch.randn(1, S, H, D, device=dev, generator=g).bfloat16()
    w = (torch.randn(Nout, K, device=dev, generator=g) / K ** 0.5).bfloat16()
    b = torch.randn(Nout, device=dev, generator=g).bfloat16()
    y = torch.empty(S, Nout, device=dev, dtype=torch.bfloat16)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    with ClockSampler(0) as clk:
        ms = timed(lambda: out_projection(o, w, b, out=y))
    ms_torch = timed(lambda: F.linear(o.view(S, K), w, b))
    flop = 2.0 * S * K * Nout
    pk, src = peaks()
    tf = flop / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": "to_out projection TFLOP/s", "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.config} to_out", "m": S, "k": K, "n": Nout, "bias": True},
        "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": pk.get("bf16_tflops"), "unit": "TFLOP/s",
                     "frac": round(tf / pk.get("bf16_tflops"), 4), "traffic": None,
                     "peak_source": f"{src} bf16_tflops (burst: a short kernel timed alone)"},
        "torch_linear_ms": round(ms_torch, 4), "torch_linear_tflops": round(flop / (ms_torch * 1e-3) / 1e12, 1),
        "clocks": clk.summary(), "gpu_launches": args.steps}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--layers", type=int, default=None, help="override layers per step")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--fp8", action="store_true",
                    help="E4M3 QK/PV with per-tile scales (quantisation inside the timed step)")
    ap.add_argument("--parallel", default="ulysses", choices=["replicas", "ulysses", "cp"],
                    help="N>1: Ulysses head parallelism over one set of layers (default, strong "
                         "scaling), the reference's own sequence-shard pattern (cp, strong scaling), "
                         "or independent layers per rank (replicas, weak scaling)")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-peak", action="store_true", help="--fp8: skip the in-run E4M3 GEMM peak measurement")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--out-proj", action="store_true",
                    help="time the to_out projection GEMM (tcgen05) against torch's Linear")
    ap.add_argument("--prologue", action="store_true",
                    help="time the fused QK prologue (norm + RoPE) instead of the attention step")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg["layers"] = args.layers
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 or args.gpus > 1:
        args.cpu_baseline = False
    if args.prologue:
        run_prologue(args, cfg)
    elif args.out_proj:
        run_out_proj(args, cfg)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_b200(args, cfg)


if __name__ == "__main__":
    main()
