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


def test_peer_sync_descriptors_are_checked_on_the_host():
    """The sharded step's synchronisation descriptor (skinny_peer_sync) is validated before any
    launch: an error word is required, 1..8 ranks, a wait or a signal, a flag address per rank for
    a signal, at most 8 mirrors and each 16-byte aligned.  (The pointers here are never touched.)"""
    from skinny_mlx_b200 import _lib

    L = _lib.lib()
    fake = 0x10000

    def prep_with(s):
        return L.skinny_prep(2, ctypes.c_void_p(fake), 64, None, 0, 0, None, None, 0, None, ctypes.c_float(0.0), 1, 64,
                             ctypes.c_void_p(fake), None, ctypes.byref(s), None)

    def good():
        s = _lib.PeerSync()
        s.epoch, s.counter, s.err, s.n_ranks = fake, fake, fake, 2
        s.signal_flags[0], s.signal_flags[1] = fake, fake + 4
        return s

    bad = []
    s = good(); s.err = None; bad.append(s)
    s = good(); s.n_ranks = 0; bad.append(s)
    s = good(); s.n_ranks = 9; bad.append(s)
    s = good(); s.counter = None; bad.append(s)  # neither a wait nor a signal
    s = good(); s.signal_flags[1] = None; bad.append(s)
    s = good(); s.n_mirror = 9; bad.append(s)
    s = good(); s.n_mirror, s.mirror[0] = 1, fake + 4; bad.append(s)  # misaligned mirror
    s = good(); s.n_mirror = 1; bad.append(s)  # a mirror slot left empty
    for s in bad:
        assert prep_with(s) == -1
    # rotary widths the half-warp rotation cannot pair are rejected as a shape error
    f = ctypes.c_void_p(fake)
    assert L.skinny_attn_fused(f, 1024, f, f, f, 48, 0, ctypes.c_float(1e-6), f, f, 0, None, 1, 4, 4, 64, f, 1 << 20,
                               f, None, None, None) == -2
