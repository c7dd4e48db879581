"""vllm-omni plugin entry point (interface of
lvsa-vllm-omni/lvsa_vllm_omni/register.py:18-133).

``register_lvsa_backend()`` adds LVSA to vllm-omni's diffusion attention
backends and installs the block-level hooks their environment variables ask
for (``LVSA_HUNYUAN_HOOK``, ``LVSA_WAN_HOOK``, ``LVSA_COSMOS3_HOOK`` = 1, with
``LVSA_TOTAL_LATENT_FRAMES``).  Nothing of vllm-omni is imported before a
function is called."""

import os

_TRUE = ("1", "true", "yes")


def register_lvsa_backend() -> None:
    from aenum import extend_enum
    from vllm_omni.diffusion.attention.backends.registry import (
        DiffusionAttentionBackendEnum,
        register_diffusion_backend,
    )
    path = "longvideosparseattention_b200.vllm_omni.backend.LVSABackend"
    if not hasattr(DiffusionAttentionBackendEnum, "LVSA"):
        extend_enum(DiffusionAttentionBackendEnum, "LVSA", path)
    register_diffusion_backend(DiffusionAttentionBackendEnum.LVSA, path)
    maybe_install_hunyuan_hook()
    maybe_install_wan_hook()
    maybe_install_cosmos3_hook()


def _maybe_install(env: str, name: str, install) -> None:
    if os.environ.get(env, "").lower() not in _TRUE:
        return
    t_lat = os.environ.get("LVSA_TOTAL_LATENT_FRAMES")
    if not t_lat:
        print(f"[LVSA] Warning: {env}=1 but LVSA_TOTAL_LATENT_FRAMES not set")
        return
    try:
        install()(total_latent_frames=int(t_lat))
    except Exception as e:  # reported, not raised: the server keeps its dense path
        print(f"[LVSA] {name} installation failed: {e}")


def maybe_install_hunyuan_hook() -> None:
    def f():
        from .hunyuan_hook import install_hunyuan_lvsa_hook
        return install_hunyuan_lvsa_hook
    _maybe_install("LVSA_HUNYUAN_HOOK", "Hook", f)


def maybe_install_wan_hook() -> None:
    def f():
        from .wan_hook import install_wan_lvsa_hook
        return install_wan_lvsa_hook
    _maybe_install("LVSA_WAN_HOOK", "Wan hook", f)


def maybe_install_cosmos3_hook() -> None:
    def f():
        from .cosmos3_hook import install_cosmos3_lvsa_hook
        return install_cosmos3_lvsa_hook
    _maybe_install("LVSA_COSMOS3_HOOK", "Cosmos3 hook", f)
