"""Build the in-tree C-ABI library libb200attn.so for sm_100a with nvcc.

Usage: python build_native.py [--debug]
The library lands next to this file in b200_pisa/lib/ so it travels with the
package; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT_DIR = HERE / "b200_pisa" / "lib"
LIB = OUT_DIR / "libb200attn.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and pathlib.Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; CUDA 12.9 is required to build libb200attn.so")


def sources() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cu"))


def build(debug: bool = False, verbose: bool = False) -> pathlib.Path:
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                    "-I", str(HERE.parent / "include")]
    if debug:
        flags += ["-DB2_DEBUG=1"]
    objects = []
    procs = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        objects.append(obj)
        deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [HERE.parent / "include" / "b200attn.h"]
        if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
            continue
        cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            failed.append(f"{src.name}:\n{out}")
        elif verbose and out.strip():
            print(out)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    link = [nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objects)]
    if verbose:
        print(" ".join(link))
    subprocess.run(link, check=True)
    return LIB


if __name__ == "__main__":
    path = build(debug="--debug" in sys.argv, verbose=True)
    print(path)
