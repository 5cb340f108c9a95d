"""In-tree build of the sm_100a C-ABI library (explicit nvcc, no JIT cache).

The kernels are written for B200 only: ``-gencode arch=compute_100a,code=sm_100a``.
nvcc cross-compiles without a GPU, so this runs on a CPU-only host too.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import List, Optional

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"  # aether_b200.h: the sources include it, so drift fails to compile
SOURCES = ["capi.cu", "tq.cu", "compat.cu", "csa_decode_api.cu", "csa_decode_cta.cu", "csa_prefill.cu", "csa_prefill_attn.cu", "cp_exchange.cu"]
OUT = PKG / "libaether_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def find_nvcc() -> Optional[str]:
    nv = shutil.which("nvcc")
    if nv:
        return nv
    for root in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if root and (Path(root) / "bin" / "nvcc").is_file():
            return str(Path(root) / "bin" / "nvcc")
    return None


def needs_build() -> bool:
    if not OUT.exists():
        return True
    mtime = OUT.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False, extra: Optional[List[str]] = None) -> Path:
    """Compile every source to an object in parallel, then link the library.

    Objects go to ``_build/`` beside the package (git-ignored); only the
    linked ``libaether_b200.so`` is loaded.
    """
    if not force and not needs_build():
        return OUT
    nvcc = find_nvcc()
    if nvcc is None:
        raise RuntimeError("nvcc was not found; cannot build the Aether sm_100a kernels")
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]

    def compile_one(src: str) -> Path:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc, *compile_flags, "-I", str(INCLUDE), *(extra or []), "-c", "-o", str(obj), str(CSRC / src)]
        if verbose:
            print(" ".join(cmd))
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src} ({res.returncode}):\n{res.stdout}\n{res.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=max(1, min(len(SOURCES), os.cpu_count() or 1))) as pool:
        objs = list(pool.map(compile_one, SOURCES))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
           "-o", str(tmp), *[str(o) for o in objs]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, OUT)
    return OUT

if __name__ == "__main__":
    print(build(force=True, verbose=True))
