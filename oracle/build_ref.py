"""Build the reference's own code from its sources, where they lie, into oracle/_ref/ (test infrastructure).

    python oracle/build_ref.py [--reference /path/to/panvram] [--cuda]

Products (oracle/_ref/, git-ignored, shipped to the GPU box with the working tree):
  panvram_ref_C.so   the reference's CPU extension (csrc/pv_core.cpp): Core, Core.windows (the CPU decoder), fasta,
                     fasta_xxh3 - the golden-vector generator here and bench.py's `--impl reference` arm on the box.
  refrel3v1          the reference's archive encoder (tools/rr3bench/refrel3v1.cpp), used to encode config 0.
  panvram_ref_Ccu.so (--cuda) the same extension with the reference's CUDA kernel (csrc/pv_cuda.cu) for sm_100a.

The image lacks zstd's header and the aceapex library; oracle/shim/ declares the five zstd prototypes the sources
call and stubs aceapex_decompress_region (reached only by the encoder's pre-v1 container paths). Nothing is copied:
the compiler reads the sources under the reference checkout.
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
SHIM = os.path.join(HERE, "shim")
LIBDIR = "/usr/lib/x86_64-linux-gnu"


def _stale(target, sources):
    return not os.path.exists(target) or any(os.path.getmtime(s) > os.path.getmtime(target) for s in sources)


def build_ext(ref, cuda=False, verbose=False):
    import torch.utils.cpp_extension as ce
    name = "panvram_ref_Ccu" if cuda else "panvram_ref_C"
    csrc = os.path.join(ref, "csrc")
    srcs = [os.path.join(csrc, "pv_core.cpp")] + ([os.path.join(csrc, "pv_cuda.cu")] if cuda else [])
    target = os.path.join(OUT, name + ".so")
    if not _stale(target, srcs):
        return target
    bdir = os.path.join(OUT, "build_" + name)
    os.makedirs(bdir, exist_ok=True)
    kw = dict(name=name, sources=srcs, extra_include_paths=[csrc, SHIM], build_directory=bdir,
              extra_cflags=["-O3"] + (["-DPV_WITH_CUDA=1"] if cuda else []),
              extra_ldflags=[os.path.join(LIBDIR, "libzstd.so.1")], verbose=verbose, is_python_module=False)
    if cuda:
        kw["extra_cuda_cflags"] = ["-O3", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a"]
        kw["with_cuda"] = True
    ce.load(**kw)
    os.replace(os.path.join(bdir, name + ".so"), target)
    return target


def build_encoder(ref):
    rr = os.path.join(ref, "tools", "rr3bench")
    src = os.path.join(rr, "refrel3v1.cpp")
    target = os.path.join(OUT, "refrel3v1")
    if not _stale(target, [src]):
        return target
    cmd = ["g++", "-std=c++17", "-O3", "-march=x86-64-v3", "-funroll-loops", "-w", "-I" + rr, "-I" + os.path.join(ref, "csrc"),
           "-I" + SHIM, src, os.path.join(SHIM, "aceapex_stub.cpp"), os.path.join(LIBDIR, "libzstd.so.1"), "-lpthread", "-o", target]
    subprocess.run(cmd, check=True)
    return target


def main():
    ap = argparse.ArgumentParser()
    # the reference checkout: $PANVRAM_REFERENCE, else a directory named "reference" beside this repository
    ap.add_argument("--reference", default=os.environ.get("PANVRAM_REFERENCE") or
                    os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference"))
    ap.add_argument("--cuda", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    if not os.path.isdir(os.path.join(a.reference, "csrc")):
        sys.exit(f"no reference checkout at {a.reference}")
    os.makedirs(OUT, exist_ok=True)
    print(build_ext(a.reference, verbose=a.v))
    print(build_encoder(a.reference))
    if a.cuda:
        print(build_ext(a.reference, cuda=True, verbose=a.v))


if __name__ == "__main__":
    main()
