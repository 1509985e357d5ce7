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
    assert lib.pv_windows_launches(0, 10) == 0 and lib.pv_windows_launches(5, 0) == 0 and lib.pv_windows_launches(5, 10) == 1
