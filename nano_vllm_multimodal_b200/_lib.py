"""Loads the in-tree native libraries. There is no fallback: if the CUDA
extension is missing or cannot be built, every op raises."""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libnib_b200.so"
SHIM_PATH = PKG / "_nib_torch.so"

_LOCK = threading.Lock()
_LOADED = False


def load_ops() -> None:
    """Register ``torch.ops.nanoinfer_b200`` / ``torch.ops.nanovllm_paged_kv``.

    Rebuilds first when the sources changed since the last build (the build
    stamp covers every source, header and flag).
    """
    global _LOADED
    if _LOADED:
        return
    with _LOCK:
        if _LOADED:
            return
        import torch

        from nano_vllm_multimodal_b200 import _build

        try:
            if not _build.up_to_date():
                # one process builds at a time (ranks of a multi-GPU run start together);
                # the others find the stamp current once they hold the lock
                import fcntl
                with open(PKG / ".build.lock", "w") as lock:
                    fcntl.flock(lock, fcntl.LOCK_EX)
                    if not _build.up_to_date():
                        _build.build()
        except Exception as exc:  # pragma: no cover - exercised only on broken toolchains
            raise RuntimeError(
                "nano_vllm_multimodal_b200: building the sm_100a CUDA extension failed; "
                f"there is no CPU fallback. Original error: {exc}") from exc
        if not SHIM_PATH.exists():
            raise RuntimeError(f"nano_vllm_multimodal_b200: {SHIM_PATH} is missing")
        torch.ops.load_library(str(SHIM_PATH))
        _LOADED = True


def cdll() -> ctypes.CDLL:
    """The C ABI library itself (``include/nib_b200.h``), for FFI callers."""
    if not LIB_PATH.exists():
        raise RuntimeError(f"nano_vllm_multimodal_b200: {LIB_PATH} is missing; build it first")
    return ctypes.CDLL(str(LIB_PATH))
