"""Helpers shared by the GPU parity tests."""

import numpy as np
import torch

# bf16 output vs fp32 oracle on the same (bf16-representable) inputs.
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3


def seeded(shape, seed, dtype=torch.bfloat16, scale=1.0, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    return x.to(dtype).to(device)


def to_np(x):
    return x.detach().float().cpu().numpy()


def assert_close(got, want, max_abs=MAX_ABS_TOL, mean_abs=MEAN_ABS_TOL, what=""):
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    sel = ~np.isnan(want)
    d = np.abs(got[sel] - want[sel])
    assert np.isfinite(got[sel]).all(), f"{what}: non-finite output"
    assert d.max() <= max_abs, f"{what}: max-abs {d.max():.3e} > {max_abs}"
    assert d.mean() <= mean_abs, f"{what}: mean-abs {d.mean():.3e} > {mean_abs}"
