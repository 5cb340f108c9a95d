"""CPU checks of the C-ABI boundary: the header compiles as C, and the
in-tree library loads and exports every function the header declares (no
kernel is launched, so no GPU is needed)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "aether_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(aether_\w+)\s*\(", text)))


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "aether_b200.h"\nint main(void) { return aether_abi_version(); }\n')
    res = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-c", str(src), "-I", str(HEADER.parent), "-o",
                          str(tmp_path / "t.o")], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_library_exports_header_symbols():
    from aether_kernels import _build, _lib

    if not _lib.library_path().exists():
        try:
            _build.build()
        except RuntimeError as e:  # no nvcc on this host
            pytest.skip(str(e))
    lib = ctypes.CDLL(str(_lib.library_path()))
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes table covers the same functions
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)
    assert lib.aether_abi_version() == 1


def test_invalid_argument_reports_error():
    from aether_kernels import _lib

    lib = _lib.load()
    rc = lib.aether_tq_encode(None, 0, 4, 96, 8, None, None, None, None, None)
    assert rc == 1
    assert "64 or 128" in _lib.last_error()


def _prototypes():
    """name -> (return type, parameter count) of every function the header declares."""
    text = re.sub(r"/\*.*?\*/", " ", HEADER.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    out = {}
    for ret, name, params in re.findall(r"([A-Za-z_][\w\s\*]*?)\s*\b(aether_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        params = " ".join(params.split())
        n = 0 if params in ("", "void") else params.count(",") + 1
        out[name] = (" ".join(ret.split()).split()[-1].rstrip("*") or ret, n)
    return out


def test_ctypes_table_matches_header_prototypes():
    """Every ctypes signature has the header prototype's parameter count and
    a void return exactly where the header returns void (the sources include
    the header, so the definitions match it at compile time)."""
    from aether_kernels import _lib

    protos = _prototypes()
    assert len(protos) == len(declared_functions())
    bad = []
    for name, (ret, n) in protos.items():
        restype, argtypes = _lib.SIGNATURES[name]
        if len(argtypes) != n:
            bad.append(f"{name}: header {n} parameters, ctypes {len(argtypes)}")
        if (ret == "void") != (restype is None):
            bad.append(f"{name}: header returns {ret}, ctypes {restype}")
    assert not bad, bad
