"""Synthetic cohorts for the tests and the benchmark (the configs of this build's workload definition): a generated
reference plus assemblies derived from it, written as refrel3 v1 archives by pv_synth.cpp (a generator-aware encoder
of the same format; see its header). Deterministic for a seed; a finished cohort directory carries a manifest and is
reused when asked again with the same parameters.

    from panvram_b200.synth import make_cohort
    path = make_cohort("/tmp/cohorts/cfg1", "cfg1")          # reference.fa + <name>.q4k.rr3 ...
"""
import ctypes
import hashlib
import json
import os
import sys
import time

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpvsynth.so")

# CHM13-like chromosome lengths (25 contigs, 248 Mbp down to a 16.5 kbp mitochondrion; about 3.1 Gbp)
CHM13_LIKE = [248387328, 242696752, 201105948, 193574945, 182045439, 172126628, 160567428, 146259331, 150617247, 134758134,
              135127769, 133324548, 113566686, 101161492, 99753195, 96330493, 84276897, 80542538, 61707364, 66210255,
              45090682, 51324926, 154259566, 62460029, 16569]

BASE = dict(snv=1e-3, indel=1.5e-4, indel_mean=3.0, indel_cap=50, n_sv=20, sv_min=10_000, sv_max=50_000,
            ctg_min=50, ctg_max=500, ctg_sigma=1.0, rc_frac=0.3, low_frac=0.05, low_mean=300.0, iupac=2e-7, block_hashes=1, zlevel=3)
CONFIGS = {
    # config 0: 4 contigs, 8 Mbp; 4 assemblies (SNV 1e-3, indel 1e-4, two SVs, 3-10 contigs), q4k
    "cfg0": dict(ref_lens=[3_000_000, 2_500_000, 1_500_000, 1_000_000], nasm=4, Q=4096, seed=0,
                 asm=dict(BASE, indel=1e-4, n_sv=2, ctg_min=3, ctg_max=10)),
    # config 1: CHM13-like 3.1 Gbp reference; 64 assemblies (SNV 1e-3, indel 1.5e-4, 20 SVs, 50-500 contigs), q4k
    "cfg1": dict(ref_lens=CHM13_LIKE, nasm=64, Q=4096, seed=1, asm=dict(BASE)),
    # config 2: 558 assemblies from the config-1 generator, SNV rate ~ U(0.8e-3, 1.5e-3), q16k
    "cfg2": dict(ref_lens=CHM13_LIKE, nasm=558, Q=16384, seed=2, asm=dict(BASE), snv_range=(0.8e-3, 1.5e-3)),
}
REF_LW = 80
_lib = None


class Spec(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("Q", ctypes.c_uint32), ("snv", ctypes.c_double), ("indel", ctypes.c_double),
                ("indel_mean", ctypes.c_double), ("indel_cap", ctypes.c_uint32), ("n_sv", ctypes.c_uint32), ("sv_min", ctypes.c_uint32),
                ("sv_max", ctypes.c_uint32), ("ctg_min", ctypes.c_uint32), ("ctg_max", ctypes.c_uint32), ("ctg_sigma", ctypes.c_double),
                ("rc_frac", ctypes.c_double), ("low_frac", ctypes.c_double), ("low_mean", ctypes.c_double), ("iupac", ctypes.c_double),
                ("block_hashes", ctypes.c_int32), ("zlevel", ctypes.c_int32)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing; build: python panvram_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        L.pvs_last_error.restype = ctypes.c_char_p
        L.pvs_ref_generate.restype = P
        L.pvs_ref_generate.argtypes = [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int, ctypes.c_double, ctypes.c_uint64,
                                       ctypes.c_double, ctypes.c_double, ctypes.c_int]
        L.pvs_ref_free.argtypes = [P]
        L.pvs_ref_n.restype, L.pvs_ref_n.argtypes = ctypes.c_uint64, [P]
        L.pvs_ref_sha256.argtypes = [P, ctypes.c_char_p]
        L.pvs_ref_write_fasta.restype, L.pvs_ref_write_fasta.argtypes = ctypes.c_int, [P, ctypes.c_char_p, ctypes.c_uint32]
        L.pvs_make_archives.restype = ctypes.c_int
        L.pvs_make_archives.argtypes = [P, ctypes.POINTER(Spec), ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                        ctypes.POINTER(ctypes.c_char_p), ctypes.c_char_p, ctypes.c_int]
        _lib = L
    return _lib


def _mix(*xs):
    h = hashlib.sha256(repr(xs).encode()).digest()
    return int.from_bytes(h[:8], "little")


def plan(config, Q=None, nasm=None, scale=1.0):
    """The full parameter set of a cohort (what its manifest records): reference lengths and one spec per assembly."""
    cfg = CONFIGS[config] if isinstance(config, str) else config
    Q = int(Q or cfg["Q"])
    n = int(nasm or cfg["nasm"])
    lens = [max(1000, int(x * scale)) for x in cfg["ref_lens"]]
    specs = []
    for i in range(n):
        a = dict(cfg["asm"])
        a["seed"] = _mix(cfg["seed"], "asm", i)
        if "snv_range" in cfg:
            lo, hi = cfg["snv_range"]
            a["snv"] = lo + (hi - lo) * ((_mix(cfg["seed"], "snv", i) >> 11) / 2.0 ** 53)
        if scale != 1.0:
            a["sv_min"], a["sv_max"] = max(100, int(a["sv_min"] * min(1.0, scale * 10))), max(200, int(a["sv_max"] * min(1.0, scale * 10)))
        a["Q"] = Q
        specs.append(a)
    return {"config": config if isinstance(config, str) else "custom", "ref_seed": _mix(cfg["seed"], "ref"), "ref_lens": lens,
            "n_frac": 0.01, "n_run": 1000, "low_frac": 0.05, "low_mean": 300.0, "Q": Q, "specs": specs,
            "names": [f"asm{i:04d}" for i in range(n)], "format": "refrel3 v1", "generator": "pv_synth 1"}


def dataset_of(Q):
    return f"q{Q // 1024}k"


def make_cohort(out_dir, config="cfg0", Q=None, nasm=None, scale=1.0, threads=0, write_fasta=False, verbose=False):
    """Write (or reuse) a synthetic cohort in out_dir: reference.fa and <name>.q<Q/1024>k.rr3 per assembly. Returns
    out_dir. write_fasta also writes <name>.fa, the assembly FASTA each archive encodes (for cross-checks)."""
    P = plan(config, Q, nasm, scale)
    os.makedirs(out_dir, exist_ok=True)
    man = os.path.join(out_dir, "manifest.json")
    ds = dataset_of(P["Q"])
    paths = [os.path.join(out_dir, f"{nm}.{ds}.rr3") for nm in P["names"]]
    if os.path.exists(man):
        with open(man) as f:
            old = json.load(f)
        if old.get("plan") == P and all(os.path.exists(p) for p in paths) and (not write_fasta or old.get("fasta")):
            return out_dir
    threads = threads or os.cpu_count() or 4
    L = lib()
    t0 = time.time()
    ref_path = os.path.join(out_dir, "reference.fa")
    lens = (ctypes.c_uint64 * len(P["ref_lens"]))(*P["ref_lens"])
    r = L.pvs_ref_generate(P["ref_seed"], lens, len(P["ref_lens"]), P["n_frac"], P["n_run"], P["low_frac"], P["low_mean"], threads)
    try:
        if L.pvs_ref_write_fasta(r, os.fsencode(ref_path), REF_LW):
            raise OSError(L.pvs_last_error().decode())
        t1 = time.time()
        specs = (Spec * len(P["specs"]))(*[Spec(**{k: s[k] for k, _ in Spec._fields_}) for s in P["specs"]])
        cpaths = (ctypes.c_char_p * len(paths))(*[os.fsencode(p) for p in paths])
        fpaths = None
        if write_fasta:
            fpaths = (ctypes.c_char_p * len(paths))(*[os.fsencode(os.path.join(out_dir, nm + ".fa")) for nm in P["names"]])
        if L.pvs_make_archives(r, specs, len(paths), cpaths, fpaths, b"reference.fa", int(threads)):
            raise OSError(L.pvs_last_error().decode())
        sha = ctypes.create_string_buffer(32)
        L.pvs_ref_sha256(r, sha)
    finally:
        L.pvs_ref_free(r)
    t2 = time.time()
    with open(man, "w") as f:
        json.dump({"plan": P, "reference_sha256": sha.raw.hex(), "fasta": bool(write_fasta), "seconds_reference": round(t1 - t0, 2),
                   "seconds_archives": round(t2 - t1, 2), "threads": threads}, f)
    if verbose:
        print(f"cohort {out_dir}: reference {t1 - t0:.1f} s, {len(paths)} archives {t2 - t1:.1f} s on {threads} threads",
              file=sys.stderr, flush=True)
    return out_dir
