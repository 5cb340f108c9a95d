"""Kernel loader with the reference's interface (aether_kernels/loader.py:24-157).

``load_aether_cuda_kernels()`` returns an object exposing the reference
extension's four ops (bindings.cpp:124-141) backed by the in-tree sm_100a
C-ABI library instead of a JIT-compiled pybind module.  The environment
probes keep the reference's names, keys and messages so its tests and its
serving code (``CudaSparseAttentionBackend``) work unchanged.
"""
from __future__ import annotations

import os
import shutil
from functools import lru_cache
from pathlib import Path
from typing import Dict, Optional

import torch

from . import _lib, ops

try:  # CUDA_HOME as torch resolves it (import has no side effects)
    from torch.utils.cpp_extension import CUDA_HOME
except Exception:  # pragma: no cover
    CUDA_HOME = os.environ.get("CUDA_HOME")


def cuda_build_environment() -> Dict[str, object]:
    """Same seven keys as the reference (loader.py:24-64)."""
    conda_prefix = os.environ.get("CONDA_PREFIX")
    target_include = target_lib = runtime_lib = None
    if conda_prefix:
        base = Path(conda_prefix) / "targets" / "x86_64-linux"
        if (base / "include").exists():
            target_include = str(base / "include")
        if (base / "lib").exists():
            target_lib = str(base / "lib")
        rt = Path(conda_prefix) / "lib" / "python3.10" / "site-packages" / "nvidia" / "cuda_runtime" / "lib"
        if rt.exists():
            runtime_lib = str(rt)
    nvcc = shutil.which("nvcc")
    if nvcc is None:
        for root in (CUDA_HOME, "/usr/local/cuda", "/usr/local/cuda-12"):
            if root and (Path(root) / "bin" / "nvcc").is_file():
                nvcc = str(Path(root) / "bin" / "nvcc")
                break
    return {
        "torch_cuda_built": torch.backends.cuda.is_built(),
        "torch_cuda_available": torch.cuda.is_available(),
        "cuda_home": CUDA_HOME,
        "nvcc": nvcc,
        "conda_target_include": target_include,
        "conda_target_lib": target_lib,
        "cuda_runtime_lib": runtime_lib,
    }


def cuda_extension_unavailable_reason(require_device: bool = False) -> Optional[str]:
    """None when the kernels can be used (loader.py:67-77).  The prebuilt
    in-tree library replaces the reference's nvcc requirement: nvcc is only
    needed when the library has not been built yet."""
    env = cuda_build_environment()
    if not env["torch_cuda_built"]:
        return "PyTorch was built without CUDA support."
    if require_device and not env["torch_cuda_available"]:
        return "No CUDA device is available for executing the custom kernels."
    if not _lib.library_path().exists():
        if env["cuda_home"] is None:
            return "CUDA_HOME is not set; install a CUDA toolkit that matches the PyTorch build."
        if env["nvcc"] is None:
            return "nvcc was not found on PATH; install the CUDA toolkit compiler."
    if require_device:
        major, minor = torch.cuda.get_device_capability()
        if (major, minor) != (10, 0):
            return f"The Aether kernels are built for sm_100a (B200); this device is sm_{major}{minor}."
    return None


class AetherKernels:
    """Object with the reference extension's method names and signatures."""

    def __init__(self) -> None:
        self.lib = _lib.load()

    @staticmethod
    def sparse_sink_attention(q, kv, topk_indices, sink, softmax_scale):
        return ops.sparse_sink_attention(q, kv, topk_indices, sink, softmax_scale)

    @staticmethod
    def tiled_prefill_attention(q, kv, sink, softmax_scale, tile_size=256):
        return ops.tiled_prefill_attention(q, kv, sink, softmax_scale, tile_size)

    @staticmethod
    def csa_indexer_topk(index_q, index_kv, index_weight, k):
        return ops.csa_indexer_topk(index_q, index_kv, index_weight, k)

    @staticmethod
    def hca_compress(buffer_c, buffer_z):
        return ops.hca_compress(buffer_c, buffer_z)


@lru_cache(maxsize=1)
def load_aether_cuda_kernels(verbose: bool = False, build_directory: Optional[str] = None):
    """Return the kernel object; builds the in-tree library first if needed.

    ``build_directory`` / ``AETHER_KERNEL_BUILD_DIR`` are accepted for
    signature compatibility; the library is always built next to this file
    so that it ships with the package."""
    reason = cuda_extension_unavailable_reason(require_device=False)
    if reason is not None:
        raise RuntimeError(f"Aether CUDA kernels are unavailable: {reason}")
    if not _lib.library_path().exists():
        from . import _build

        _build.build(verbose=verbose)
    return AetherKernels()
