"""LVSAConfig (mirror of lvsa-vllm-omni/lvsa_vllm_omni/config.py:9-144).

Frame-valued fields are in VIDEO frames and are divided by
``vae_temporal_factor`` to get latent frames.  ``backend`` is accepted for
compatibility; every value runs the same sm_100a kernel.
"""

import json
import os
from dataclasses import dataclass, fields
from typing import List, Optional


@dataclass
class LVSAConfig:
    window_size: int = 12
    n_first_frames: int = 4
    key_frame_interval: int = 16
    auto_keyframes: bool = True
    rotate_keyframes: bool = False
    expand_window: bool = True
    backend: str = "sdpa"
    vae_temporal_factor: int = 4
    total_latent_frames: Optional[int] = None
    sparsity_scale: float = 1.0
    reference_latent_frames: int = 21

    @classmethod
    def from_env(cls) -> "LVSAConfig":
        """``LVSA_CONFIG`` (JSON) if set, else the individual ``LVSA_*`` variables."""
        js = os.environ.get("LVSA_CONFIG")
        if js:
            return cls.from_json(js)
        env = os.environ

        def b(key, d):
            v = env.get(key)
            return d if v is None else v.lower() in ("1", "true", "yes")
        tl = env.get("LVSA_TOTAL_LATENT_FRAMES")
        return cls(window_size=int(env.get("LVSA_WINDOW_SIZE", 12)),
                   n_first_frames=int(env.get("LVSA_N_FIRST_FRAMES", 4)),
                   key_frame_interval=int(env.get("LVSA_KEY_FRAME_INTERVAL", 16)),
                   auto_keyframes=b("LVSA_AUTO_KEYFRAMES", True),
                   rotate_keyframes=b("LVSA_ROTATE_KEYFRAMES", False),
                   expand_window=b("LVSA_EXPAND_WINDOW", True),
                   backend=env.get("LVSA_BACKEND", "sdpa"),
                   vae_temporal_factor=int(env.get("LVSA_VAE_TEMPORAL_FACTOR", 4)),
                   total_latent_frames=int(tl) if tl else None,
                   sparsity_scale=float(env.get("LVSA_SPARSITY_SCALE", 1.0)),
                   reference_latent_frames=int(env.get("LVSA_REFERENCE_LATENT_FRAMES", 21)))

    @classmethod
    def from_json(cls, s: str) -> "LVSAConfig":
        data = json.loads(s)
        names = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in names})

    @property
    def latent_window_size(self) -> int:
        return self.window_size // self.vae_temporal_factor

    @property
    def latent_n_first_frames(self) -> int:
        return self.n_first_frames // self.vae_temporal_factor

    @property
    def latent_key_frame_interval(self) -> int:
        return self.key_frame_interval // self.vae_temporal_factor


DEFAULT_PATCHES_PER_FRAME = 1560


def candidate_patches_per_frame() -> List[int]:
    """P candidates for geometry detection: ``LVSA_PATCHES_PER_FRAME`` (list),
    else derived from ``LVSA_VIDEO_HEIGHT/WIDTH`` (+ VAE spatial factor and
    patch size), else 1560."""
    ov = os.environ.get("LVSA_PATCHES_PER_FRAME")
    if ov:
        try:
            return [int(x) for x in ov.split(",") if x.strip()]
        except ValueError:
            pass
    try:
        h = int(os.environ.get("LVSA_VIDEO_HEIGHT", "0"))
        w = int(os.environ.get("LVSA_VIDEO_WIDTH", "0"))
        sf = int(os.environ.get("LVSA_VAE_SPATIAL_FACTOR", "8"))
        ps = int(os.environ.get("LVSA_PATCH_SIZE", "2"))
        if h > 0 and w > 0 and sf > 0 and ps > 0:
            ph, pw = (h // sf) // ps, (w // sf) // ps
            if ph > 0 and pw > 0:
                return [ph * pw]
    except ValueError:
        pass
    return [DEFAULT_PATCHES_PER_FRAME]
