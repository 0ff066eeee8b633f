"""Device gate and runtime report for the B200 path (replaces the
reference's ROCm/gfx1151 probe, rdna35_block_attention/diagnostics.py:22-157).

The product kernels live in the in-tree C-ABI library loaded by b200_pisa;
this module only answers "is the current CUDA device an sm_100 GPU" and
describes the runtime for the diagnostics node."""
from __future__ import annotations

import importlib
from typing import Any

import torch

REQUIRED_MAJOR = 10  # sm_100 (B200)


def b200_device_index() -> tuple[int | None, str | None]:
    """(device index, None) for a usable sm_100 device, else (None, reason)."""
    if not torch.cuda.is_available() or torch.version.cuda is None:
        return None, "PyTorch CUDA device is unavailable"
    try:
        index = torch.cuda.current_device()
        major, minor = torch.cuda.get_device_capability(index)
    except (RuntimeError, AssertionError) as exc:
        return None, f"could not query the current CUDA device ({type(exc).__name__}: {exc})"
    if major != REQUIRED_MAJOR:
        return None, f"sm_100 (B200) is required, got sm_{major}{minor}"
    return index, None


def native_module():
    """The B200 native module; raises ImportError when the library is missing."""
    return importlib.import_module("b200_pisa")


def has_native() -> tuple[bool, str]:
    try:
        module = native_module()
    except (ImportError, OSError) as exc:
        return False, f"{type(exc).__name__}: {exc}"
    return True, f"api={module.build_info().get('api')}"


def detect_runtime() -> dict[str, Any]:
    ok, info = has_native()
    index, reason = b200_device_index()
    name = torch.cuda.get_device_name(index) if index is not None else None
    return {
        "torch_version": torch.__version__,
        "torch_version_cuda": torch.version.cuda,
        "torch_cuda_is_available": torch.cuda.is_available(),
        "device": name,
        "device_index": index,
        "device_reason": reason,
        "native_available": ok,
        "native_info": info,
    }


def explain_dispatch() -> str:
    runtime = detect_runtime()
    lines = ["RDNA35-Attention B200 runtime"]
    lines += [f"{key}: {value}" for key, value in runtime.items()]
    if runtime["device_index"] is None or not runtime["native_available"]:
        lines.append("optimized kernels: unavailable (calls chain to the previous attention backend)")
    else:
        lines.append("optimized kernels: tcgen05/TMA/TMEM attention, PISA statistics/routing, layout kernels")
    return "\n".join(lines)
