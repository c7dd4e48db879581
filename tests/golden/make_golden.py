"""Generate golden vectors by importing the UNMODIFIED reference LVSA package.

Run in a container where the reference checkout exists:

    python tests/golden/make_golden.py /path/to/LongVideoSparseAttention

It writes ``patterns.npz`` (frame-level ``LVSAMetadata.build`` outputs),
``attn_*.npz`` (seeded bf16-representable inputs with the reference's fp32
``lvsa_sdpa`` output and dense text-query rows) and ``rope.npz`` (the
reference's ``apply_rotary_emb`` / ``slice_rotary_emb`` on seeded inputs)
and ``adapters.npz`` (the reference HunyuanVideo / CogVideoX adapters on
seeded mock modules) and ``cp.npz`` (the reference's world > 1 path, per
rank) and ``cfg1.npz`` (BASELINE configs[0] at full size, fp32, sampled
rows); ``--only rope|adapters|cp|cfg1`` writes just one of them.  The fixtures are committed;
the tests never need the reference at run time.
"""

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, T, P, W, n_first, kfi, offset, expand, rank, world)
PATTERN_CASES = [
    ("cfg1", 9, 1560, 1, 1, 4, 3, True, 0, 1),
    ("cfg2", 81, 1560, 2, 1, 4, 0, True, 0, 1),
    ("cfg3_s0", 121, 1560, 2, 1, 4, 0, True, 0, 1),
    ("cfg3_s1", 121, 1560, 2, 1, 4, 1, True, 0, 1),
    ("cfg3_s2", 121, 1560, 2, 1, 4, 2, True, 0, 1),
    ("cfg3_s3", 121, 1560, 2, 1, 4, 3, True, 0, 1),
    ("cfg4", 49, 1590, 2, 1, 4, 0, True, 0, 1),
    ("cfg5", 49, 1350, 1, 1, 3, 0, True, 0, 1),
    ("w0", 21, 16, 0, 1, 5, 0, True, 0, 1),
    ("noexpand", 21, 16, 3, 1, 5, 2, False, 0, 1),
    ("kfi_none", 17, 8, 2, 4, None, 0, True, 0, 1),
    ("t1", 1, 8, 1, 1, 4, 0, True, 0, 1),
    ("small_T", 5, 4, 3, 1, 2, 1, True, 0, 1),
    ("nfirst3", 33, 12, 2, 3, 7, 5, True, 0, 1),
    ("big_off", 30, 6, 2, 1, 4, 11, True, 0, 1),
    ("wide_w", 40, 10, 9, 2, 6, 4, True, 0, 1),
    ("kfi1", 12, 8, 1, 1, 1, 0, True, 0, 1),
    ("cp_r0", 20, 10, 2, 1, 5, 0, True, 0, 2),
    ("cp_r1", 20, 10, 2, 1, 5, 0, True, 1, 2),
    ("cp_r2of4", 21, 8, 1, 1, 4, 2, True, 2, 4),
]

# (name, T, P, H, Hkv, D, W, n_first, kfi, offset, n_text, B, seed)
ATTN_CASES = [
    ("a_small", 9, 8, 2, 2, 64, 1, 1, 4, 3, 0, 1, 1),
    ("a_text", 7, 12, 2, 2, 128, 1, 1, 3, 1, 10, 1, 2),
    ("a_gqa", 6, 16, 4, 2, 64, 1, 1, 2, 0, 5, 2, 3),
    ("a_w0", 8, 10, 2, 2, 64, 0, 1, 3, 2, 0, 1, 4),
    ("a_p130", 5, 130, 2, 2, 128, 1, 1, 2, 1, 0, 1, 5),
    ("a_t1", 1, 20, 2, 2, 64, 1, 1, 4, 0, 3, 1, 6),
    ("a_d128", 10, 40, 3, 3, 128, 2, 1, 4, 2, 17, 1, 7),
]


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from lvsa.sparse_attention import LVSAMetadata, lvsa_sdpa, compute_boundary_guard_frames
    from lvsa.lvsa_processor import DistributedLVSAProcessor

    pats = {}
    meta_json = {}
    for name, T, P, W, nf, kfi, off, exp, rank, world in PATTERN_CASES:
        guards = (compute_boundary_guard_frames(T, T * P // world, P, world, W)
                  if world > 1 else None)
        m = LVSAMetadata.build(total_latent_frames=T, num_patches=P, window_size=W,
                               n_first_frames=nf, key_frame_interval=kfi, rank=rank,
                               world=world, expand_window=exp, keyframe_offset=off,
                               boundary_guards=guards)
        pats[f"{name}.global_indices"] = np.asarray(m.global_indices, dtype=np.int32)
        pats[f"{name}.global_frame_mask"] = m.global_frame_mask.numpy()
        pats[f"{name}.window_bounds"] = m.window_bounds.numpy()
        pats[f"{name}.attended_indices"] = m.attended_indices.numpy()
        pats[f"{name}.fi_indptr"] = m.fi_indptr.numpy()
        pats[f"{name}.fi_indices"] = m.fi_indices.numpy()
        pats[f"{name}.local_frames"] = np.asarray(m.local_frames, dtype=np.int64)
        wc = [(f, s, e) for f, parts in sorted(m.window_ctx.items()) for s, e in parts]
        pats[f"{name}.window_ctx"] = np.asarray(wc, dtype=np.int64).reshape(-1, 3)
        meta_json[name] = dict(T=T, P=P, W=W, n_first=nf, kfi=kfi, offset=off, expand=exp,
                               rank=rank, world=world, guards=guards or [],
                               local_seq=m.local_seq, fi_MB=m.fi_MB,
                               fi_compact_n=m.fi_compact_n, attended_C=m.attended_C)
    np.savez_compressed(os.path.join(HERE, "patterns.npz"), **pats)
    with open(os.path.join(HERE, "patterns.json"), "w") as fh:
        json.dump(meta_json, fh, indent=1, sort_keys=True)

    for name, T, P, H, Hkv, D, W, nf, kfi, off, nt, B, seed in ATTN_CASES:
        g = torch.Generator().manual_seed(seed)
        N = T * P
        q = bf16_round(torch.randn(B, N, H, D, generator=g))
        k = bf16_round(torch.randn(B, N, Hkv, D, generator=g))
        v = bf16_round(torch.randn(B, N, Hkv, D, generator=g))
        tq = bf16_round(torch.randn(B, nt, H, D, generator=g))
        tk = bf16_round(torch.randn(B, nt, Hkv, D, generator=g))
        tv = bf16_round(torch.randn(B, nt, Hkv, D, generator=g))
        m = LVSAMetadata.build(total_latent_frames=T, num_patches=P, window_size=W,
                               n_first_frames=nf, key_frame_interval=kfi, rank=0, world=1,
                               expand_window=True, keyframe_offset=off)
        # global K/V as lvsa_processor._build_global_kv (world=1) + text appended (:545-549)
        gi = torch.tensor(m.global_indices, dtype=torch.long)
        idx = (gi[:, None] * P + torch.arange(P)[None, :]).flatten()
        kg = torch.cat([k[:, idx], tk], dim=1)
        vg = torch.cat([v[:, idx], tv], dim=1)
        out = lvsa_sdpa(q, k, v, kg, vg, m)
        arrays = dict(q=q.numpy(), k=k.numpy(), v=v.numpy(), out=out.numpy(),
                      text_q=tq.numpy(), text_k=tk.numpy(), text_v=tv.numpy())
        if nt > 0:
            if Hkv != H:
                rep = H // Hkv
                fk = torch.cat([k, tk], 1).repeat_interleave(rep, dim=2)
                fv = torch.cat([v, tv], 1).repeat_interleave(rep, dim=2)
            else:
                fk, fv = torch.cat([k, tk], 1), torch.cat([v, tv], 1)
            arrays["text_out"] = DistributedLVSAProcessor._compute_full_attention(
                None, tq, fk, fv).numpy()
        arrays["params"] = np.asarray([T, P, H, Hkv, D, W, nf, kfi, off, nt, B, seed],
                                      dtype=np.int64)
        np.savez_compressed(os.path.join(HERE, f"attn_{name}.npz"), **arrays)
        print("wrote", name)


def rope_golden(ref_root: str) -> None:
    """lvsa/rope.py:10-28 (apply_rotary_emb) and :31-57 (slice_rotary_emb)."""
    sys.path.insert(0, ref_root)
    from lvsa.rope import apply_rotary_emb, slice_rotary_emb
    g = torch.Generator().manual_seed(4242)
    arrays = {}
    for name, (S, H, D) in {"d128": (24, 3, 128), "d64": (17, 2, 64)}.items():
        x = bf16_round(torch.randn(1, S, H, D, generator=g))
        ang = torch.rand(S, D // 2, generator=g) * 6.0
        # Wan layout [1, S, 1, D]: each pair angle repeated in the even and odd slot.
        cos = torch.cos(ang).repeat_interleave(2, -1)[None, :, None, :]
        sin = torch.sin(ang).repeat_interleave(2, -1)[None, :, None, :]
        arrays[f"{name}.x"] = x.numpy()
        arrays[f"{name}.cos"] = cos.numpy()
        arrays[f"{name}.sin"] = sin.numpy()
        arrays[f"{name}.out"] = apply_rotary_emb(x, cos, sin).numpy()
        c1, s1 = slice_rotary_emb((cos, sin), S // 3, 1, 3)
        arrays[f"{name}.slice_cos"] = c1.numpy()
        arrays[f"{name}.slice_sin"] = s1.numpy()
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **arrays)
    print("wrote rope")


CP_CASES = [  # name, T, P, H, Hkv, D, W, n_first, kfi, offset, n_text, world, seed
    ("cp_w2", 9, 40, 2, 2, 64, 1, 1, 4, 1, 17, 2, 71),
    ("cp_w3_mid", 9, 50, 2, 1, 64, 2, 1, 3, 2, 0, 3, 72),   # rank splits inside frames, GQA
    ("cp_w4_d128", 12, 30, 2, 2, 128, 1, 1, 5, 0, 9, 4, 73),
]


def cp_golden(ref_root: str) -> None:
    """The reference's world > 1 path on each rank: LVSAMetadata.build with the
    processor's boundary guards, the global K/V _build_global_kv assembles
    (all global frames, text appended), lvsa_sdpa; text queries attend the
    rank's video keys + text (lvsa/lvsa_processor.py:586-591)."""
    sys.path.insert(0, ref_root)
    from lvsa.sparse_attention import LVSAMetadata, compute_boundary_guard_frames, lvsa_sdpa
    from lvsa.lvsa_processor import DistributedLVSAProcessor
    arrays = {}
    for name, T, P, H, Hkv, D, W, nf, kfi, off, nt, world, seed in CP_CASES:
        g = torch.Generator().manual_seed(seed)
        N = T * P
        q = bf16_round(torch.randn(1, N, H, D, generator=g))
        k = bf16_round(torch.randn(1, N, Hkv, D, generator=g))
        v = bf16_round(torch.randn(1, N, Hkv, D, generator=g))
        tq = bf16_round(torch.randn(1, nt, H, D, generator=g))
        tk = bf16_round(torch.randn(1, nt, Hkv, D, generator=g))
        tv = bf16_round(torch.randn(1, nt, Hkv, D, generator=g))
        arrays.update({f"{name}.q": q.numpy(), f"{name}.k": k.numpy(), f"{name}.v": v.numpy(),
                       f"{name}.text_q": tq.numpy(), f"{name}.text_k": tk.numpy(), f"{name}.text_v": tv.numpy(),
                       f"{name}.params": np.asarray([T, P, H, Hkv, D, W, nf, kfi, off, nt, world, seed])})
        S_r = N // world
        guards = compute_boundary_guard_frames(T, S_r, P, world, W)
        for r in range(world):
            m = LVSAMetadata.build(total_latent_frames=T, num_patches=P, window_size=W, n_first_frames=nf,
                                   key_frame_interval=kfi, rank=r, world=world, expand_window=True,
                                   keyframe_offset=off, boundary_guards=guards)
            gi = torch.tensor(m.global_indices, dtype=torch.long)
            idx = (gi[:, None] * P + torch.arange(P)[None, :]).flatten()
            kg, vg = k[:, idx], v[:, idx]
            if nt:
                kg, vg = torch.cat([kg, tk], 1), torch.cat([vg, tv], 1)
            sl = slice(r * S_r, (r + 1) * S_r)
            out = lvsa_sdpa(q[:, sl], k[:, sl], v[:, sl], kg, vg, m)
            arrays[f"{name}.out{r}"] = out.numpy()
            arrays[f"{name}.globals{r}"] = np.asarray(m.global_indices)
            if nt:
                fk, fv = torch.cat([k[:, sl], tk], 1), torch.cat([v[:, sl], tv], 1)
                if Hkv != H:
                    fk, fv = fk.repeat_interleave(H // Hkv, 2), fv.repeat_interleave(H // Hkv, 2)
                arrays[f"{name}.text_out{r}"] = DistributedLVSAProcessor._compute_full_attention(
                    None, tq, fk, fv).numpy()
    np.savez_compressed(os.path.join(HERE, "cp.npz"), **arrays)
    print("wrote cp")


def adapters_golden(ref_root: str) -> None:
    """The reference HunyuanVideo / CogVideoX adapters (lvsa/adapters/
    hunyuan_video.py, cogvideox.py) on seeded mock modules: extract_qkv,
    extract_encoder_qkv, apply_rotary (its RoPE fallback, lvsa/rope.py),
    output_projection and format_output."""
    import importlib.util
    sys.path.insert(0, ref_root)
    from lvsa.adapters import get_adapter
    spec = importlib.util.spec_from_file_location("adapter_mocks", os.path.join(os.path.dirname(HERE),
                                                                                "adapter_mocks.py"))
    mocks = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mocks)
    MockAttn, rope_pair = mocks.MockAttn, mocks.rope_pair
    arrays = {}
    for name, norm, dual in (("hunyuan_video", "rms", True), ("cogvideox", "ln", False)):
        dim, heads, S, St = 256, 4, 24, 7
        attn = MockAttn(dim, heads, norm, dual, seed=len(name))
        g = torch.Generator().manual_seed(99 + len(name))
        hs = torch.randn(1, S, dim, generator=g)
        ehs = torch.randn(1, St, dim, generator=g)
        cos, sin = rope_pair(S, dim // heads, seed=5)
        ad = get_adapter(name)
        with torch.no_grad():
            q, k, v = ad.extract_qkv(attn, hs, ehs)
            q2, k2 = ad.apply_rotary(q, k, (cos, sin), S, 0, 1)
            eq, ek, ev = ad.extract_encoder_qkv(attn, ehs)
            o = torch.randn(1, S, heads, dim // heads, generator=g)
            eo = torch.randn(1, St, heads, dim // heads, generator=g)
            hp = ad.output_projection(attn, o, torch.float32)
            fo = ad.format_output(attn, hp, eo, St, torch.float32)
        for key, t in dict(hs=hs, ehs=ehs, cos=cos, sin=sin, q=q2, k=k2, v=v, eq=eq, ek=ek, ev=ev,
                           o=o, eo=eo, out_video=fo[0], out_text=fo[1]).items():
            arrays[f"{name}.{key}"] = t.numpy()
        arrays[f"{name}.ppf"] = np.asarray([ad.patches_per_frame(480, 832, _Pipe(name)),
                                            ad.latent_frames(121, _Pipe(name)),
                                            ad.reference_latent_frames(_Pipe(name))])
    np.savez_compressed(os.path.join(HERE, "adapters.npz"), **arrays)
    print("wrote adapters")


# B=1, 12 heads, head_dim 128, fp32 q/k/v ~ N(0,1),
# 9 latent frames x 1560 tokens, W=1, one anchor, kfi 4, step 3.
CFG1 = dict(T=9, P=1560, H=12, D=128, W=1, n_first=1, kfi=4, step=3, seed=9001, rows_per_frame=24)


def cfg1_inputs():
    """The full-size fp32 inputs, regenerated from the seed (torch's CPU
    generator is deterministic for a given torch build)."""
    c = CFG1
    g = torch.Generator().manual_seed(c["seed"])
    N = c["T"] * c["P"]
    return tuple(torch.randn(1, N, c["H"], c["D"], generator=g) for _ in range(3))


def cfg1_rows():
    """Sampled query rows: rows_per_frame seeded token positions in every frame."""
    c = CFG1
    rng = np.random.default_rng(c["seed"])
    return np.concatenate([f * c["P"] + np.sort(rng.choice(c["P"], c["rows_per_frame"], replace=False))
                           for f in range(c["T"])]).astype(np.int64)


def cfg1_golden(ref_root: str) -> None:
    """configs[0] at full size through the reference's own lvsa_sdpa in fp32
    (lvsa/sparse_attention.py:643-706), global K/V as _build_global_kv at
    world 1.  The output is kept on sampled rows (all heads) with checksums
    of the inputs, so the test can regenerate them and detect a drift."""
    sys.path.insert(0, ref_root)
    from lvsa.sparse_attention import LVSAMetadata, lvsa_sdpa
    c = CFG1
    q, k, v = cfg1_inputs()
    m = LVSAMetadata.build(total_latent_frames=c["T"], num_patches=c["P"], window_size=c["W"],
                           n_first_frames=c["n_first"], key_frame_interval=c["kfi"], rank=0, world=1,
                           expand_window=True, keyframe_offset=c["step"] % c["kfi"])
    gi = torch.tensor(m.global_indices, dtype=torch.long)
    idx = (gi[:, None] * c["P"] + torch.arange(c["P"])[None, :]).flatten()
    out = lvsa_sdpa(q, k, v, k[:, idx], v[:, idx], m)
    rows = cfg1_rows()
    np.savez_compressed(os.path.join(HERE, "cfg1.npz"), rows=rows, out=out[0, rows].numpy(),
                        checksums=np.asarray([float(x.double().sum()) for x in (q, k, v)]),
                        params=np.asarray([c[x] for x in ("T", "P", "H", "D", "W", "n_first", "kfi", "step",
                                                          "seed", "rows_per_frame")]))
    print("wrote cfg1")


class _Pipe:
    """Minimal pipeline stand-in for the geometry helpers."""

    def __init__(self, name: str):
        class _Cfg:
            patch_size = 2 if name != "hunyuan_video" else [1, 1, 1]
            patch_size_t = None

        class _Tr:
            config = _Cfg()
        self.transformer = _Tr()
        self.vae_scale_factor_spatial = 16 if name == "hunyuan_video" else 8
        self.vae_scale_factor_temporal = 4


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = args[0] if args else os.environ.get("LVSA_REFERENCE_ROOT", ".")
    if "--only" in sys.argv:
        which = sys.argv[sys.argv.index("--only") + 1]
        {"rope": rope_golden, "adapters": adapters_golden, "cp": cp_golden, "cfg1": cfg1_golden}[which](root)
    else:
        main(root)
        rope_golden(root)
        adapters_golden(root)
        cp_golden(root)
        cfg1_golden(root)
