"""Test infrastructure: build the reference's own CUDA extension for sm_100a.

Compiles the reference checkout's aether_kernels/csrc sources where they lie
(bindings.cpp and the four .cu kernels) with the flags of the reference's
loader (aether_kernels/loader.py:128-150: -O3, --use_fast_math, the half /
bf16 conversion undefines, relaxed constexpr, extended lambdas), for sm_100a,
into oracle/_ref/aether_ref_kernels.so.  Nothing is copied into this
repository; the built module is git-ignored and travels to GPU boxes with the
tree.  Only the tests import it, as a second reference for the drop-in
kernels (aether_kernels.sparse_attention).

    python oracle/build_ref.py <reference checkout>
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "_ref"
NAME = "aether_ref_kernels"


def module_path() -> Path:
    return OUT / f"{NAME}.so"


def build(reference_root: str | os.PathLike, verbose: bool = False) -> Path:
    csrc = Path(reference_root) / "aether_kernels" / "csrc"
    sources = [str(csrc / "bindings.cpp")] + sorted(str(p) for p in csrc.glob("*.cu"))
    if not all(Path(s).exists() for s in sources) or len(sources) < 2:
        raise FileNotFoundError(f"reference extension sources not found under {csrc}")
    OUT.mkdir(exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    load(name=NAME, sources=sources, extra_cflags=["-O3"],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo", "-U__CUDA_NO_HALF_OPERATORS__",
                            "-U__CUDA_NO_HALF_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
                            "--expt-relaxed-constexpr", "--expt-extended-lambda",
                            "-gencode", "arch=compute_100a,code=sm_100a"],
         extra_include_paths=[str(csrc)], build_directory=str(OUT), with_cuda=True, verbose=verbose)
    return module_path()


def load_built():
    """Import the built module (torch must be importable), or return None."""
    path = module_path()
    if not path.exists():
        return None
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    loader = importlib.machinery.ExtensionFileLoader(NAME, str(path))
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AETHER_REFERENCE")
    if not root:
        sys.exit("usage: build_ref.py <reference checkout>")
    print(build(root, verbose=True))
