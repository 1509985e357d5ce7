"""The drop-in boundary: the native library loads without a GPU and exports every function include/panvram_b200.h
declares (no compute call is made here)."""
import ctypes
import os
import re
import subprocess

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "panvram_b200.h")
LIB = os.path.join(ROOT, "panvram_b200", "libpanvram_b200.so")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pv_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    for want in ("pv_core_open", "pv_core_pools", "pv_windows", "pv_windows_ex", "pv_core_fasta_xxh3", "pv_last_error"):
        assert want in names


def test_library_exports_every_declared_symbol():
    if not os.path.exists(LIB):
        subprocess.run(["python", os.path.join(ROOT, "panvram_b200", "build.py")], check=True)
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (pv_\w+)$", out, flags=re.M))
    assert set(declared()) <= exported


def test_last_error_without_gpu():
    lib = ctypes.CDLL(LIB)
    lib.pv_last_error.restype = ctypes.c_char_p
    lib.pv_windows_launches.restype = ctypes.c_int
    lib.pv_windows_launches.argtypes = [ctypes.c_int64, ctypes.c_int64]
    assert lib.pv_last_error() is not None
    assert lib.pv_windows_launches(0, 10) == 0 and lib.pv_windows_launches(5, 0) == 0 and lib.pv_windows_launches(5, 10) == 3    # decode, emission, general path


def test_sample_coords_refuses_bad_arguments_without_launching():
    """pv_sample_coords checks its arguments before any CUDA call: a negative count, an empty contig table, an unknown
    strand mode and missing pointers are refused (PV_EARG) with a message; an empty call with no status word is a no-op."""
    from panvram_b200 import _C
    lib = _C._lib
    P = ctypes.c_void_p(16)
    def call(n, nctg=3, mode=0, ptrs=True, r=None, rc=None):
        p = P if ptrs else None
        return lib.pv_sample_coords(p, p, p, p, p, nctg, p, r, 0.5, mode, n, p, p, rc, None, None, None)
    assert call(-1) == _C.PV_EARG
    assert call(4, nctg=0) == _C.PV_EARG
    assert call(4, mode=3) == _C.PV_EARG
    assert call(4, ptrs=False) == _C.PV_EARG
    assert call(4, mode=2, rc=P) == _C.PV_EARG                  # strand from draws without the draws
    assert call(4, mode=1) == _C.PV_EARG                        # strand output missing
    assert b"NULL" in lib.pv_kernels_last_error()
    assert call(0, ptrs=False) == _C.PV_OK


def test_windows_refuses_bad_decode_lanes_without_launching():
    """pv_windows_ex checks its flags before any CUDA call: PV_WIN_DEC_LANES above 32 is refused (PV_EARG)."""
    from panvram_b200 import _C
    lib = _C._lib
    dev = _C.DevCohort()
    for f in ("ref", "payload", "blocks", "asms", "tabs", "low"):
        setattr(dev, f, 16)
    dev.Q, dev.nasm, dev.tab_max = 4096, 1, 1024
    P = ctypes.c_void_p(16)
    rc = lib.pv_windows_ex(ctypes.byref(dev), P, P, 8, 100, None, 0, 1, _C.PV_WIN_SPLIT | _C.PV_WIN_DEC_LANES(33), P, P, None,
                           P, 1 << 30, None)
    assert rc == _C.PV_EARG and b"lanes" in lib.pv_kernels_last_error()


def test_windows_form_rule():
    """pv_windows_form reports the launches a call takes without a GPU: the fused kernel for few items, the split form
    beyond (4,608 items; 3,072 at Q = 16,384), with about 3,072 decode warps (at most 32 items per warp); flags pin it."""
    from panvram_b200 import _C
    assert _C.windows_form(4096, 1024, 8192) == (1, 0)              # config 1: 3,072 items
    assert _C.windows_form(4096, 1536, 8192) == (3, 2)              # 4,608 items
    assert _C.windows_form(16384, 1024, 8192) == (1, 0)             # 2,048 items
    assert _C.windows_form(16384, 4096, 8192) == (3, 3)             # config 2: 8,192 items
    assert _C.windows_form(4096, 131072, 512) == (3, 32)
    assert _C.windows_form(4096, 1024, 8192, _C.PV_WIN_SPLIT) == (3, 1)
    assert _C.windows_form(16384, 4096, 8192, _C.PV_WIN_FUSED) == (1, 0)
    assert _C.windows_form(4096, 9999, 8192, _C.PV_WIN_SPLIT | _C.PV_WIN_DEC_LANES(7)) == (3, 7)
    assert _C.windows_form(4096, 0, 8192) == (0, 0)
    import pytest
    with pytest.raises(ValueError):
        _C.windows_form(3000, 10, 10)


def test_torch_draw_geometry_without_gpu():
    """pv_torch_draw_geometry restates torch's launch for sample()'s draws (256-thread blocks, at most SMs x 8 of them;
    each thread's curand4 call gives 2 values for randint ranges of 2^28 or more, else 4, and 4 for rand; the Philox
    offset advances 4 per call a thread makes): known cases on a 148-SM, 2,048-thread-per-SM device."""
    from panvram_b200 import _C
    import pytest
    assert _C.torch_draw_geometry(1024, 198_000_000_000, 2, 148, 2048) == (1024, 4, 8)
    assert _C.torch_draw_geometry(1024, 1000, 0, 148, 2048) == (1024, 4, 4)
    assert _C.torch_draw_geometry(700_000, 1 << 40, 2, 148, 2048) == (303_104, 8, 12)        # randint: 2 passes
    assert _C.torch_draw_geometry(1_300_000, 1000, 2, 148, 2048) == (303_104, 8, 16)         # both: 2 passes
    assert _C.torch_draw_geometry(0, 5, 2, 148, 2048) == (0, 0, 0)                           # no draws, no advance
    with pytest.raises(ValueError):
        _C.torch_draw_geometry(10, 0, 0, 148, 2048)


def test_new_entry_points_refuse_bad_arguments_without_launching():
    """The host-coordinate gather and the status read accept only pinned host memory, and the in-kernel draws check
    their sizes, all before any launch: ordinary (pageable) host memory, a zero range or a negative count are refused
    with PV_EARG and a message."""
    import numpy as np
    from panvram_b200 import _C
    lib = _C._lib
    a = np.zeros(8, dtype=np.int64)
    s = np.zeros(8, dtype=np.int64)
    P = ctypes.c_void_p(16)
    assert lib.pv_coords_from_host(a.ctypes.data, s.ctypes.data, None, 8, P, P, None, None) == _C.PV_EARG
    assert b"pinned" in lib.pv_kernels_last_error()
    assert lib.pv_coords_from_host(None, None, None, 0, None, None, None, None) == _C.PV_OK          # nothing to do
    w = np.zeros(1, dtype=np.int32)
    assert lib.pv_status_to_host(P, w.ctypes.data, None) == _C.PV_EARG
    for n, total in ((-1, 10), (4, 0)):
        assert lib.pv_sample_draw_coords(P, P, P, P, P, 1, total, None, 0, 0, 0.5, 2, n, P, P, P, None, None, None, None, None) == _C.PV_EARG
