"""CPU test: the C-ABI library loads and exports every function include/*.h declares."""

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[\w\s\*]+?\b(skinny_\w+)\s*\(", text, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_library_exports_declared_symbols():
    from skinny_mlx_b200 import build, _lib

    build.build()
    handle = ctypes.CDLL(str(build.LIB))
    names = declared_functions()
    assert len(names) >= 7
    missing = [n for n in names if not hasattr(handle, n)]
    assert not missing, missing
    # the Python binding declares a signature for every exported entry point
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_host_side_calls_without_gpu():
    """Calls that need no device: version, status text, sizes, argument validation."""
    from skinny_mlx_b200 import _lib

    L = _lib.lib()
    assert L.skinny_version() >= 100
    assert b"token" in L.skinny_strerror(-3)
    assert L.skinny_repack_bytes(9728, 2560) == 76 * 40 * 4608
    assert L.skinny_repack_bytes(8224, 2560) == 65 * 40 * 4608
    assert L.skinny_repack_bytes(100, 100) == 0  # K not a multiple of 64
    # invalid arguments are rejected on the host before any launch
    assert L.skinny_qmm_w4g64(None, 64, None, None, 8, 1, 8, 64, None, 0, None) == -1
    assert L.skinny_repack_w4g64(None, None, None, None, 8, 64, None) == -1
