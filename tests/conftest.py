import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
for p in (ROOT / "comfyui-rdna35-attention_b200", ROOT / "oracle", ROOT / "tests", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run on the B200 box)")


def pytest_sessionstart(session):
    """Build the in-tree C-ABI library (nvcc cross-compiles without a GPU)
    when it is missing, so the CPU suite can load it."""
    lib = ROOT / "comfyui-rdna35-attention_b200" / "b200_pisa" / "lib" / "libb200attn.so"
    if not lib.exists():
        import build_native

        build_native.build()
