"""Build panvram_b200's native library in-tree: panvram_b200/libpanvram_b200.so (the C ABI of
include/panvram_b200.h) from csrc/pv_host.cpp (host reader, pooling) and csrc/pv_kernels.cu (sm_100a kernels).

    python panvram_b200/build.py [--force] [--ptxas-info]

nvcc cross-compiles for sm_100a (B200) without a GPU; the CUDA runtime is linked statically so the library does not
depend on which libcudart the host process (torch) loaded. Rebuilds only what changed."""
import argparse
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INC = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build", "panvram_b200")
LIB = os.path.join(PKG, "libpanvram_b200.so")
SYNTH_LIB = os.path.join(PKG, "synth", "libpvsynth.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
LIBDIR = "/usr/lib/x86_64-linux-gnu"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HEADERS = [os.path.join(INC, "panvram_b200.h")] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".h")]


def _stale(target, deps):
    return not os.path.exists(target) or any(os.path.getmtime(d) > os.path.getmtime(target) for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build failed: " + " ".join(cmd[:3]))
    return r.stdout + r.stderr


def build(force=False, verbose=False, ptxas_info=False):
    os.makedirs(BUILD, exist_ok=True)
    objs, log = [], ""
    for src in sorted(os.listdir(CSRC)):
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        if src.endswith(".cu"):
            cmd = [os.path.join(CUDA, "bin", "nvcc"), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-I" + INC, "-I" + CSRC, "-c", path, "-o", obj] + (["-Xptxas", "-v"] if ptxas_info else [])
        elif src.endswith(".cpp"):
            cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-Wall", "-I" + INC, "-I" + CSRC, "-I" + os.path.join(CUDA, "include"),
                   "-c", path, "-o", obj]
        else:
            continue
        objs.append(obj)
        if force or ptxas_info or _stale(obj, [path] + HEADERS):
            log += _run(cmd, verbose)
    if force or _stale(LIB, objs):
        _run(["g++", "-shared", "-o", LIB, *objs, "-L" + os.path.join(CUDA, "lib64"), "-lcudart_static", "-ldl", "-lrt", "-lpthread",
              os.path.join(LIBDIR, "libzstd.so.1"), os.path.join(LIBDIR, "libxxhash.so.0"), os.path.join(LIBDIR, "libcrypto.so.3")], verbose)
    # the cohort synthesizer (test and benchmark data; not linked into the decode library)
    src = os.path.join(PKG, "synth", "pv_synth.cpp")
    if force or _stale(SYNTH_LIB, [src] + HEADERS):
        _run(["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-Wall", "-I" + INC, "-I" + CSRC, src, "-o", SYNTH_LIB, "-lpthread",
              os.path.join(LIBDIR, "libzstd.so.1"), os.path.join(LIBDIR, "libxxhash.so.0"), os.path.join(LIBDIR, "libcrypto.so.3")], verbose)
    return LIB, log


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    lib, log = build(a.force, a.v, a.ptxas_info)
    if log.strip():
        print(log)
    print(lib)


if __name__ == "__main__":
    main()
