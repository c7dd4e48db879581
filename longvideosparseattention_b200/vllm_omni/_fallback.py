"""One-time warnings when the plugin falls back to dense attention
(interface of lvsa-vllm-omni/lvsa_vllm_omni/_fallback.py:17-57).

Printed once per (origin, reason, seq_len); ``LVSA_WARN_FALLBACK=0`` (read at
import) silences them."""

import os
from typing import Optional, Set

_FALLBACK_WARN = os.environ.get("LVSA_WARN_FALLBACK", "1").lower() in ("1", "true", "yes")
_seen_warnings: Set[str] = set()


def warn_fallback(origin: str, reason: str, seq_len: int = -1, extra: Optional[dict] = None) -> None:
    if not _FALLBACK_WARN:
        return
    key = f"{origin}:{reason}:{seq_len}"
    if key in _seen_warnings:
        return
    _seen_warnings.add(key)
    detail = "".join(f", {k}={v}" for k, v in (extra or {}).items())
    print(f"[LVSA-FALLBACK] origin={origin} reason={reason} seq_len={seq_len}{detail.replace(', ', ' ', 1)} "
          f"-- falling back to DENSE attention (set LVSA_WARN_FALLBACK=0 to silence)", flush=True)


def reset_warnings() -> None:
    _seen_warnings.clear()
