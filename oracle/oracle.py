"""TEST INFRASTRUCTURE ONLY: Python access to the oracle (oracle/pv_oracle.c, the CPU restatement of the reference's
refrel3 v1 reader and decoder) and to the reference's own compiled CPU extension (oracle/_ref/panvram_ref_C.so).
Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg only; never by the product."""
import ctypes
import importlib.machinery
import importlib.util
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libpvoracle.so")
REF_EXT = os.path.join(HERE, "_ref", "panvram_ref_C.so")
REF_EXT_CUDA = os.path.join(HERE, "_ref", "panvram_ref_Ccu.so")
REF_ENCODER = os.path.join(HERE, "_ref", "refrel3v1")

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        P, U64, I64, I32, U32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int, ctypes.c_uint32
        sig = {
            "pvo_ref_load": (I32, [ctypes.c_char_p, ctypes.POINTER(P), ctypes.c_char_p, ctypes.c_size_t]),
            "pvo_ref_free": (None, [P]), "pvo_ref_n": (U64, [P]), "pvo_ref_bases": (P, [P]),
            "pvo_ref_sha256": (None, [P, ctypes.c_char_p]),
            "pvo_arc_open": (I32, [ctypes.c_char_p, P, ctypes.POINTER(P), ctypes.c_char_p, ctypes.c_size_t]),
            "pvo_arc_free": (None, [P]), "pvo_arc_q": (U32, [P]), "pvo_arc_nbases": (U64, [P]), "pvo_arc_nblocks": (U64, [P]),
            "pvo_arc_payload_bytes": (U64, [P]), "pvo_arc_block_payload": (U64, [P, U64]), "pvo_arc_fasta_xxh3": (U64, [P]),
            "pvo_arc_block_state": (I32, [P, U64, ctypes.POINTER(U64), ctypes.POINTER(U32)]),
            "pvo_arc_freq": (U32, [P, I32, I32]),
            "pvo_arc_ncontigs": (U64, [P]), "pvo_arc_nlow": (U64, [P]),
            "pvo_arc_contig": (I32, [P, U64, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(U32)]),
            "pvo_block": (I32, [P, P, U64, P, I32]),
            "pvo_window": (I32, [P, P, U64, U64, I32, I32, I32, I32, P]),
            "pvo_windows": (I32, [P, I64, P, I64, P, P, U64, P, I32, I32, I32, I32, P]),
            "pvo_fasta": (I32, [P, P, I32, P, U64, ctypes.POINTER(U64)]),
            "pvo_fasta_xxh3": (U64, [P, P]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


class OracleError(Exception):
    pass


class Reference:
    def __init__(self, path):
        L, h, e = lib(), ctypes.c_void_p(), ctypes.create_string_buffer(512)
        if L.pvo_ref_load(os.fsencode(path), ctypes.byref(h), e, 512):
            raise OracleError(e.value.decode())
        self.h, self.path, self._free = h, path, L.pvo_ref_free

    def __del__(self):
        if getattr(self, "h", None):
            self._free(self.h)
            self.h = None

    @property
    def n(self):
        return lib().pvo_ref_n(self.h)

    def sha256(self):
        b = ctypes.create_string_buffer(32)
        lib().pvo_ref_sha256(self.h, b)
        return b.raw.hex()


class Archive:
    def __init__(self, path, ref):
        L, h, e = lib(), ctypes.c_void_p(), ctypes.create_string_buffer(512)
        if L.pvo_arc_open(os.fsencode(path), ref.h, ctypes.byref(h), e, 512):
            raise OracleError(e.value.decode())
        self.h, self.ref, self.path, self._free = h, ref, path, L.pvo_arc_free

    def __del__(self):
        if getattr(self, "h", None):
            self._free(self.h)
            self.h = None

    Q = property(lambda s: lib().pvo_arc_q(s.h))
    nbases = property(lambda s: lib().pvo_arc_nbases(s.h))
    nblocks = property(lambda s: lib().pvo_arc_nblocks(s.h))
    payload_bytes = property(lambda s: lib().pvo_arc_payload_bytes(s.h))
    fasta_xxh3 = property(lambda s: "%016x" % lib().pvo_arc_fasta_xxh3(s.h))

    def block_payload(self, b):
        return lib().pvo_arc_block_payload(self.h, b)

    def freq(self):
        """model frequencies [61, 104] (uint16 as the reference's R3Tab.freq)."""
        L = lib()
        return np.array([[L.pvo_arc_freq(self.h, c, s) for s in range(104)] for c in range(61)], dtype=np.uint32)

    def block_state(self, b):
        """(c, dir) start diagonal of block b, c as the unsigned 64-bit value the reference keeps."""
        c, d = ctypes.c_uint64(), ctypes.c_uint32()
        if lib().pvo_arc_block_state(self.h, b, ctypes.byref(c), ctypes.byref(d)):
            raise OracleError(f"block {b}")
        return c.value, d.value

    def contigs(self):
        """[(name, header, length, base offset, line width)] as the reference's Core.contigs."""
        L, out = lib(), []
        for i in range(L.pvo_arc_ncontigs(self.h)):
            hb = ctypes.create_string_buffer(1 << 16)
            n, o, w = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint32()
            L.pvo_arc_contig(self.h, i, hb, 1 << 16, ctypes.byref(n), ctypes.byref(o), ctypes.byref(w))
            hdr = hb.value.decode()
            name = hdr.replace("\t", " ").split(" ")[0]
            out.append((name, hdr, n.value, o.value, w.value))
        return out

    def block(self, b, verify=False):
        out = np.zeros(self.Q, np.uint8)
        e = lib().pvo_block(self.h, self.ref.h, b, out.ctypes.data, int(verify))
        if e:
            raise OracleError(f"block {b}: code {e}")
        return out

    def window(self, s, W, rc=False, tokens=False, apply_case=True, verify=False):
        out = np.zeros(max(W, 1), np.uint8)
        e = lib().pvo_window(self.h, self.ref.h, s, W, int(rc), int(tokens), int(apply_case), int(verify), out.ctypes.data)
        if e:
            raise OracleError(f"window ({s}, {W}): code {e}")
        return out[:W]

    def fasta(self, verify=True):
        L, sz = lib(), ctypes.c_uint64()
        L.pvo_fasta(self.h, self.ref.h, 0, None, 0, ctypes.byref(sz))
        out = np.zeros(max(sz.value, 1), np.uint8)
        e = L.pvo_fasta(self.h, self.ref.h, int(verify), out.ctypes.data, sz.value, ctypes.byref(sz))
        if e:
            raise OracleError(f"{self.path}: fasta code {e}")
        return out[:sz.value].tobytes()

    def fasta_xxh3_of(self, bases):
        b = np.ascontiguousarray(bases, dtype=np.uint8)
        return "%016x" % lib().pvo_fasta_xxh3(self.h, b.ctypes.data)


def windows(arcs, ref, asm, start, W, rc=None, tokens=False, apply_case=True, verify=False, threads=1):
    """The reference CPU decoder's Core.windows, restated: uint8 [n, W]."""
    asm = np.ascontiguousarray(asm, dtype=np.int64)
    start = np.ascontiguousarray(start, dtype=np.int64)
    n = len(asm)
    out = np.zeros((n, W), np.uint8)
    if n == 0:
        return out
    hs = (ctypes.c_void_p * len(arcs))(*[a.h.value for a in arcs])
    rcp = None
    if rc is not None:
        rcb = np.ascontiguousarray(rc, dtype=np.uint8)
        rcp = rcb.ctypes.data
    e = lib().pvo_windows(hs, len(arcs), ref.h, n, asm.ctypes.data, start.ctypes.data, W, rcp, int(tokens), int(apply_case),
                          int(verify), int(threads), out.ctypes.data)
    if e:
        raise OracleError(f"windows: code {e}")
    return out


def reference_extension(cuda=False):
    """The reference's compiled extension (panvram._C built from its own sources), or None when absent. cuda: the build
    with its GPU kernels (pv_cuda.cu, sm_100a), which adds windows_cuda / windows_cuda2."""
    path, name = (REF_EXT_CUDA, "panvram_ref_Ccu") if cuda else (REF_EXT, "panvram_ref_C")
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the extension links libtorch)
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


class ReferenceGPU:
    """The reference's own GPU path on a cohort directory: its Core, its pools copied to the device as its Cohort does
    (panvram/cohort.py:25-38), its windows_cuda (pv_cuda.cu:153-161) and its sample() arithmetic
    (panvram/cohort.py:165-194, restated with the same torch calls). Test infrastructure: the comparison side for the
    reference's kernel, never part of panvram_b200."""

    def __init__(self, ext, reference, paths, device, threads=0):
        import torch
        self.torch, self.ext, self.device = torch, ext, torch.device(device)
        self.core = ext.Core(reference, list(paths), threads)
        pools = self.core.pools()
        self.dev = {k: v.to(self.device) for k, v in pools.items() if isinstance(v, torch.Tensor) and not k.startswith("ctg_")}
        self.ctg = {k: pools[k].to(self.device) for k in ("ctg_asm", "ctg_local", "ctg_boff", "ctg_len")}
        self.valid = {}

    def windows(self, asm, start, W, rc=None, tokens=False):
        d = self.dev
        return self.ext.windows_cuda(d["P"], d["pay_base"], d["off"], d["st"], d["tab"], d["blk_base"], d["nbases"], d["low_s"],
                                     d["low_l"], d["low_base"], d["low_cnt"], d["ref"], self.core.Q, asm, start, int(W), rc, tokens, True)

    def sample(self, n, W, generator, reverse_complement=False, tokens=False):
        torch = self.torch
        if W not in self.valid:
            v = (self.ctg["ctg_len"] - W + 1).clamp_min(0)
            self.valid[W] = (torch.cumsum(v, 0), v)
        cum, v = self.valid[W]
        total = int(cum[-1].item())
        gdev = generator.device
        u = torch.randint(0, total, (n,), generator=generator, device=gdev, dtype=torch.int64).to(self.device)
        k = torch.searchsorted(cum, u, right=True)
        pos = u - (cum[k] - v[k])
        asm = self.ctg["ctg_asm"][k]
        start = self.ctg["ctg_boff"][k] + pos
        rc = None
        if reverse_complement is True:
            rc = torch.ones(n, dtype=torch.bool, device=self.device)
        elif reverse_complement:
            rc = (torch.rand(n, generator=generator, device=gdev) < float(reverse_complement)).to(self.device)
        out, status = self.windows(asm, start, W, rc, tokens)
        strand = rc.to(torch.int64) if rc is not None else torch.zeros(n, dtype=torch.int64, device=self.device)
        return out, status, torch.stack([asm, self.ctg["ctg_local"][k], pos, strand], 1)
