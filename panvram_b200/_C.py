"""panvram_b200._C - the binding of the native library (include/panvram_b200.h) under the names of the reference's
extension module panvram._C (pv_core.cpp:195-220): Core, FormatError, with_cuda, sha256_file_bases, and the window
launch that replaces windows_cuda / windows_cuda2 (pv_cuda.cu:153-179).

The binding is ctypes over the C ABI: tensors cross as device pointers plus torch's current CUDA stream. There is no
CPU decoder and no fallback: if the native library is missing, importing this module raises."""
import ctypes
import os

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpanvram_b200.so")
if not os.path.exists(LIB_PATH):
    raise ImportError(f"panvram_b200 native library missing ({LIB_PATH}); build it: python panvram_b200/build.py")
_lib = ctypes.CDLL(LIB_PATH)

PV_OK, PV_EFORMAT, PV_EARG, PV_ECUDA, PV_EIO = 0, 1, 2, 3, 4
PV_TAB_MAX_BYTES = 8208
with_cuda = True


class FormatError(ValueError):
    """An archive or reference refused (the reference's panvram.FormatError, a ValueError)."""


class AsmRec(ctypes.Structure):
    _fields_ = [("nbases", ctypes.c_uint64), ("blk_base", ctypes.c_uint64), ("nb", ctypes.c_uint64), ("low_base", ctypes.c_uint64),
                ("low_cnt", ctypes.c_uint64), ("tab_off", ctypes.c_uint64), ("tab_bytes", ctypes.c_uint64), ("grp_base", ctypes.c_uint64)]


class DevCohort(ctypes.Structure):
    _fields_ = [("ref", ctypes.c_void_p), ("ref_n", ctypes.c_uint64), ("payload", ctypes.c_void_p), ("blocks", ctypes.c_void_p),
                ("asms", ctypes.c_void_p), ("tabs", ctypes.c_void_p), ("tab_max", ctypes.c_uint64), ("low", ctypes.c_void_p),
                ("cache", ctypes.c_void_p), ("nasm", ctypes.c_int64),
                ("Q", ctypes.c_uint32), ("pad", ctypes.c_uint32),
                ("pref", ctypes.c_void_p), ("pruns", ctypes.c_void_p), ("pidx", ctypes.c_void_p), ("pnruns", ctypes.c_uint64),
                ("groups", ctypes.c_void_p), ("btab", ctypes.c_void_p), ("bexc", ctypes.c_void_p),
                ("packed", ctypes.c_uint32), ("compact", ctypes.c_uint32),
                ("ckpt", ctypes.c_void_p), ("ckpt_shift", ctypes.c_uint32), ("pad2", ctypes.c_uint32), ("brun", ctypes.c_void_p),
                ("rcref", ctypes.c_void_p)]


class HostPools(ctypes.Structure):
    _fields_ = [(k, t) for k, t in (
        ("ref_padded", ctypes.c_void_p), ("ref_padded_bytes", ctypes.c_uint64), ("payload", ctypes.c_void_p), ("payload_bytes", ctypes.c_uint64),
        ("blocks", ctypes.c_void_p), ("blocks_bytes", ctypes.c_uint64), ("asms", ctypes.c_void_p), ("asms_bytes", ctypes.c_uint64),
        ("tabs", ctypes.c_void_p), ("tabs_bytes", ctypes.c_uint64), ("tab_max", ctypes.c_uint64), ("low", ctypes.c_void_p),
        ("low_bytes", ctypes.c_uint64),
        ("ctg_asm", ctypes.c_void_p), ("ctg_local", ctypes.c_void_p), ("ctg_boff", ctypes.c_void_p), ("ctg_len", ctypes.c_void_p),
        ("ncontigs", ctypes.c_uint64),
        ("pref", ctypes.c_void_p), ("pref_bytes", ctypes.c_uint64), ("pruns", ctypes.c_void_p), ("pruns_bytes", ctypes.c_uint64),
        ("pnruns", ctypes.c_uint64), ("pidx", ctypes.c_void_p), ("pidx_bytes", ctypes.c_uint64),
        ("groups", ctypes.c_void_p), ("groups_bytes", ctypes.c_uint64), ("btab", ctypes.c_void_p), ("btab_bytes", ctypes.c_uint64),
        ("bexc", ctypes.c_void_p), ("bexc_bytes", ctypes.c_uint64), ("packed", ctypes.c_uint32), ("compact", ctypes.c_uint32))]

# pv_blk_group (include/panvram_b200.h) as a numpy record
BLK_GROUP = np.dtype([("off", "<u8"), ("state", "<i8"), ("exc_mask", "<u4"), ("exc_base", "<u4"), ("cache_mask", "<u4"),
                      ("cache_base", "<u4")])
PV_BLK_GROUP = 32
PV_CODE_EXC = -32768


class AsmInfo(ctypes.Structure):
    _fields_ = [("Q", ctypes.c_uint32), ("block_hashes", ctypes.c_uint32), ("bases", ctypes.c_uint64), ("blocks", ctypes.c_uint64),
                ("file_bytes", ctypes.c_uint64), ("payload_bytes", ctypes.c_uint64), ("contigs", ctypes.c_uint64),
                ("lower_case_runs", ctypes.c_uint64), ("fasta_xxh3", ctypes.c_uint64), ("bases_xxh3", ctypes.c_uint64)]


_P, _I64, _U64, _I32, _U32, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t
for _name, _res, _args in (
        ("pv_last_error", ctypes.c_char_p, []),
        ("pv_kernels_last_error", ctypes.c_char_p, []),
        ("pv_core_open", _I32, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), _I64, _I32, _I32, _I32, ctypes.POINTER(_P)]),
        ("pv_core_free", None, [_P]),
        ("pv_core_n", _I64, [_P]), ("pv_core_q", _U32, [_P]), ("pv_core_ref_bases", _U64, [_P]),
        ("pv_core_ref_sha256", None, [_P, ctypes.c_char_p]),
        ("pv_core_pools", _I32, [_P, ctypes.POINTER(HostPools)]),
        ("pv_core_release_uploaded", None, [_P]),
        ("pv_core_info", _I32, [_P, _I64, ctypes.POINTER(AsmInfo)]),
        ("pv_core_info_strings", _I32, [_P, _I64, ctypes.c_char_p, _SZ, ctypes.c_char_p, _SZ]),
        ("pv_core_ncontigs", _I64, [_P, _I64]),
        ("pv_core_contig", _I32, [_P, _I64, _I64, ctypes.c_char_p, _SZ, ctypes.c_char_p, _SZ, ctypes.POINTER(_U64), ctypes.POINTER(_U64),
                                  ctypes.POINTER(_U32)]),
        ("pv_core_fasta_xxh3", _I32, [_P, _I64, _P, _U64, ctypes.POINTER(_U64)]),
        ("pv_core_fasta_write", _I32, [_P, _I64, _P, _U64, _P, _U64, ctypes.POINTER(_U64)]),
        ("pv_core_check_block_hashes", _I32, [_P, _I64, _P, _U64, ctypes.POINTER(_I64)]),
        ("pv_core_apply_case", _I32, [_P, _I64, _P, _U64]),
        ("pv_sha256_file_bases", _I32, [ctypes.c_char_p, ctypes.c_char_p]),
        ("pv_windows", _I32, [ctypes.POINTER(DevCohort), _P, _P, _I64, _I64, _P, _I32, _I32, _P, _P, _P, _SZ, _P]),
        ("pv_windows_ex", _I32, [ctypes.POINTER(DevCohort), _P, _P, _I64, _I64, _P, _I32, _I32, _U32, _P, _P, _P, _P, _SZ, _P]),
        ("pv_windows_work_bytes", _SZ, [ctypes.POINTER(DevCohort), _I64, _I64]),
        ("pv_windows_noalloc", _I32, [ctypes.POINTER(DevCohort), _P, _P, _I64, _I64, _P, _I32, _I32, _P, _P, _P]),
        ("pv_windows_ids", _I32, [ctypes.POINTER(DevCohort), _P, _P, _I64, _I64, _P, ctypes.POINTER(ctypes.c_int64), _P, _P, _P, _SZ, _P]),
        ("pv_sample_coords", _I32, [_P, _P, _P, _P, _P, _I64, _P, _P, ctypes.c_float, _I32, _I64, _P, _P, _P, _P, _P, _P]),
        ("pv_windows_launches", _I32, [_I64, _I64]),
        ("pv_status_to_host", _I32, [_P, _P, _P]),
        ("pv_coords_from_host", _I32, [_P, _P, _P, _I64, _P, _P, _P, _P]),
        ("pv_windows_form", _I32, [_U32, _I64, _I64, _U32, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(_U32)]),
        ("pv_core_device_check_work_bytes", _SZ, [_P, _I64]),
        ("pv_core_fasta_xxh3_device", _I32, [_P, _I64, _P, _U64, _U64, _P, _SZ, _P, ctypes.POINTER(_U64)]),
        ("pv_core_fasta_write_device", _I32, [_P, _I64, _P, _U64, _P, _U64, _P, _SZ, _P, ctypes.POINTER(_U64)]),
        ("pv_core_check_block_hashes_device", _I32, [_P, _I64, _P, _U64, _P, _SZ, _P, ctypes.POINTER(_I64)]),
        ("pv_apply_case_device", _I32, [ctypes.POINTER(DevCohort), _I64, _U64, _P, _U64, _P]),
        ("pv_xxh3_64_long_host", _I32, [_P, _U64, ctypes.POINTER(_U64)]),
        ("pv_sample_draw_coords", _I32, [_P, _P, _P, _P, _P, _I64, _U64, _P, _U64, _U64, ctypes.c_float, _I32, _I64, _P, _P, _P, _P, _P, _P,
                                         _P, _P]),
        ("pv_torch_draw_geometry", _I32, [_I64, _U64, _I32, _I32, _I32, ctypes.POINTER(_U64), ctypes.POINTER(_U64), ctypes.POINTER(_U64)]),
        ("pv_index_bytes", _SZ, [_U32, _U64, _U32]),
        ("pv_windows_items", _SZ, [ctypes.POINTER(DevCohort), _I64, _I64]),
        ("pv_rc_reference", _I32, [_P, _U64, _P, _P]),
        ("pv_windows_trace", _I32, [ctypes.POINTER(DevCohort), _P, _P, _I64, _I64, _P, _I32, _I32, _U32, _P, _P, _P, _SZ, _P, _SZ, _P]),
        ("pv_index_build", _I32, [ctypes.POINTER(DevCohort), _U64, _U32, _P, _P, _P, _P, _P])):
    _f = getattr(_lib, _name)
    _f.restype, _f.argtypes = _res, _args


def _err(code):
    msg = (_lib.pv_last_error() or b"").decode(errors="replace")
    if code == PV_EFORMAT:
        return FormatError(msg)
    if code == PV_EARG:
        return RuntimeError(msg)
    return RuntimeError(f"panvram_b200: {msg or 'error ' + str(code)}")


def _check(code):
    if code:
        raise _err(code)


def _host_array(ptr, nbytes, dtype):
    if not nbytes:
        return np.zeros(0, dtype)
    buf = (ctypes.c_uint8 * nbytes).from_address(ptr)
    return np.frombuffer(buf, dtype=dtype)


class Core:
    """The opened cohort on the host (the reference's panvram._C.Core): reference + archives, every check done,
    arrays pooled in the device layout (pools()) for the caller to move to its GPU."""

    def __init__(self, reference, paths, threads=0, packed_reference=False, compact_blocks=False):
        h = ctypes.c_void_p()
        arr = (ctypes.c_char_p * len(paths))(*[os.fsencode(p) for p in paths])
        _check(_lib.pv_core_open(os.fsencode(reference), arr, len(paths), int(threads), int(bool(packed_reference)),
                                 int(bool(compact_blocks)), ctypes.byref(h)))
        self._h, self._free = h, _lib.pv_core_free
        self.packed_reference, self.compact_blocks = bool(packed_reference), bool(compact_blocks)

    def __del__(self):
        if getattr(self, "_h", None):
            self._free(self._h)
            self._h = None

    Q = property(lambda self: int(_lib.pv_core_q(self._h)))
    n = property(lambda self: int(_lib.pv_core_n(self._h)))
    ref_bases = property(lambda self: int(_lib.pv_core_ref_bases(self._h)))

    @property
    def ref_sha256(self):
        b = ctypes.create_string_buffer(65)
        _lib.pv_core_ref_sha256(self._h, b)
        return b.value.decode()

    def release_uploaded(self):
        """Free the host copies of the reference and the pooled payload once they are on the device (pools() then
        gives them empty; views taken before dangle)."""
        _lib.pv_core_release_uploaded(self._h)

    def pools(self):
        """Host arrays in the device layout (numpy views of the core's memory), keyed by component."""
        p = HostPools()
        _check(_lib.pv_core_pools(self._h, ctypes.byref(p)))
        n = p.ncontigs
        return {
            "ref_padded": _host_array(p.ref_padded, p.ref_padded_bytes, np.uint8),
            "payload": _host_array(p.payload, p.payload_bytes, np.uint8),
            "blocks": _host_array(p.blocks, p.blocks_bytes, np.uint64),
            "asms": _host_array(p.asms, p.asms_bytes, np.uint8),
            "tabs": _host_array(p.tabs, p.tabs_bytes, np.uint8), "tab_max": int(p.tab_max),
            "low": _host_array(p.low, p.low_bytes, np.uint64),
            "ctg_asm": _host_array(p.ctg_asm, n * 8, np.int64), "ctg_local": _host_array(p.ctg_local, n * 8, np.int64),
            "ctg_boff": _host_array(p.ctg_boff, n * 8, np.int64), "ctg_len": _host_array(p.ctg_len, n * 8, np.int64),
            "pref": _host_array(p.pref, p.pref_bytes, np.uint32), "pruns": _host_array(p.pruns, p.pruns_bytes, np.uint8),
            "pnruns": int(p.pnruns), "pidx": _host_array(p.pidx, p.pidx_bytes, np.uint32),
            "groups": _host_array(p.groups, p.groups_bytes, np.uint8), "btab": _host_array(p.btab, p.btab_bytes, np.uint32),
            "bexc": _host_array(p.bexc, p.bexc_bytes, np.int64),
        }

    def _asm_check(self, i):
        i = int(i)
        if not 0 <= i < self.n:
            raise FormatError("assembly index out of range")
        return i

    def info(self, i):
        i = self._asm_check(i)
        a = AsmInfo()
        _check(_lib.pv_core_info(self._h, i, ctypes.byref(a)))
        path, refname = ctypes.create_string_buffer(4096), ctypes.create_string_buffer(65536)
        _check(_lib.pv_core_info_strings(self._h, i, path, 4096, refname, 65536))
        return {"path": path.value.decode(), "Q": a.Q, "bases": a.bases, "blocks": a.blocks, "file_bytes": a.file_bytes,
                "payload_bytes": a.payload_bytes, "block_hashes": bool(a.block_hashes), "fasta_xxh3": "%016x" % a.fasta_xxh3,
                "contigs": a.contigs, "lower_case_runs": a.lower_case_runs, "reference_name": refname.value.decode()}

    def contigs(self, i):
        """[(name, header, length, offset in the base stream, line width)] (pv_core.cpp:160)."""
        i = self._asm_check(i)
        out = []
        for k in range(_lib.pv_core_ncontigs(self._h, i)):
            hdr, name = ctypes.create_string_buffer(1 << 16), ctypes.create_string_buffer(1 << 16)
            ln, bo, lw = _U64(), _U64(), _U32()
            _check(_lib.pv_core_contig(self._h, i, k, hdr, 1 << 16, name, 1 << 16, ctypes.byref(ln), ctypes.byref(bo), ctypes.byref(lw)))
            out.append((name.value.decode(), hdr.value.decode(), ln.value, bo.value, lw.value))
        return out

    @staticmethod
    def _host_u8(bases):
        if not isinstance(bases, torch.Tensor) or bases.device.type != "cpu" or bases.dtype != torch.uint8:
            raise FormatError("bases: uint8 CPU tensor of the assembly's length")
        return bases.contiguous()

    def fasta_xxh3(self, i, bases):
        """XXH3 of the FASTA rebuilt from a decoded base stream (case applied), "%016x" (pv_core.cpp:167-176)."""
        i, b = self._asm_check(i), self._host_u8(bases)
        h = _U64()
        code = _lib.pv_core_fasta_xxh3(self._h, i, b.data_ptr(), b.numel(), ctypes.byref(h))
        if code:
            raise FormatError((_lib.pv_last_error() or b"").decode())
        return "%016x" % h.value

    def fasta_bytes(self, i, bases):
        """The FASTA file's bytes rebuilt from a decoded base stream (case applied) and the contig table."""
        i, b = self._asm_check(i), self._host_u8(bases)
        sz = _U64()
        _check(_lib.pv_core_fasta_write(self._h, i, b.data_ptr(), b.numel(), None, 0, ctypes.byref(sz)))
        buf = ctypes.create_string_buffer(max(1, sz.value))
        _check(_lib.pv_core_fasta_write(self._h, i, b.data_ptr(), b.numel(), ctypes.cast(buf, ctypes.c_void_p), sz.value, ctypes.byref(sz)))
        return buf.raw[:sz.value]

    def first_bad_block(self, i, upper_bases):
        i, b = self._asm_check(i), self._host_u8(upper_bases)
        r = _I64()
        _check(_lib.pv_core_check_block_hashes(self._h, i, b.data_ptr(), b.numel(), ctypes.byref(r)))
        return r.value

    def apply_case(self, i, bases):
        i, b = self._asm_check(i), self._host_u8(bases)
        if not b.is_contiguous():
            raise FormatError("bases must be contiguous")
        _check(_lib.pv_core_apply_case(self._h, i, b.data_ptr(), b.numel()))
        return b

    # ---- the same checks over a decoded stream in device memory (kernels on torch's current stream of its device)
    @staticmethod
    def _dev_u8(bases):
        if not isinstance(bases, torch.Tensor) or bases.device.type != "cuda" or bases.dtype != torch.uint8 or not bases.is_contiguous():
            raise FormatError("bases: contiguous uint8 CUDA tensor of the assembly's length")
        return bases

    def _dev_call(self, fn, i, b, *args):
        work = torch.empty(max(16, _lib.pv_core_device_check_work_bytes(self._h, i)), dtype=torch.uint8, device=b.device)
        code = fn(self._h, i, b.data_ptr(), b.numel(), *args[:-1], work.data_ptr(), work.numel(),
                  torch.cuda.current_stream(b.device).cuda_stream, args[-1])
        if code:
            msg = (_lib.pv_kernels_last_error() or b"").decode(errors="replace")
            raise (RuntimeError if code == PV_ECUDA else FormatError)(msg)

    def fasta_xxh3_device(self, i, bases, chunk_blocks=0):
        """fasta_xxh3 of a decoded stream (case applied) in device memory: the FASTA is read over the stream on the
        device (nothing copied back but XXH3's per-block sums, chunk_blocks of them per round trip; 0: 65,536),
        "%016x"."""
        i, b = self._asm_check(i), self._dev_u8(bases)
        h = _U64()
        with torch.cuda.device(b.device):
            self._dev_call(_lib.pv_core_fasta_xxh3_device, i, b, int(chunk_blocks), ctypes.byref(h))
        return "%016x" % h.value

    def fasta_device(self, i, bases):
        """The FASTA file's bytes rebuilt on the device from a decoded stream (case applied) -> uint8 CUDA tensor."""
        i, b = self._asm_check(i), self._dev_u8(bases)
        sz = _U64()
        _check(_lib.pv_core_fasta_write_device(self._h, i, None, b.numel(), None, 0, None, 0, None, ctypes.byref(sz)))
        out = torch.empty(max(1, sz.value), dtype=torch.uint8, device=b.device)
        with torch.cuda.device(b.device):
            self._dev_call(_lib.pv_core_fasta_write_device, i, b, out.data_ptr(), out.numel(), ctypes.byref(sz))
        return out[:sz.value]

    def first_bad_block_device(self, i, upper_bases):
        """first_bad_block of a decoded upper-case stream in device memory (per-block XXH3 on the device)."""
        i, b = self._asm_check(i), self._dev_u8(upper_bases)
        r = _I64()
        with torch.cuda.device(b.device):
            self._dev_call(_lib.pv_core_check_block_hashes_device, i, b, ctypes.byref(r))
        return r.value


def xxh3_64_long_host(data):
    """XXH3_64bits of bytes longer than 240, by the block sums, scramble chain and finish the device path splits."""
    b = bytes(data)
    h = _U64()
    buf = ctypes.create_string_buffer(b, len(b))
    code = _lib.pv_xxh3_64_long_host(ctypes.cast(buf, ctypes.c_void_p), len(b), ctypes.byref(h))
    if code:
        raise ValueError((_lib.pv_kernels_last_error() or b"").decode())
    return h.value


def apply_case_device(dev, a, runs, bases):
    """Lower-case runs of assembly a (as uploaded in the DevCohort dev) applied in place to its device stream."""
    code = _lib.pv_apply_case_device(ctypes.byref(dev), int(a), int(runs), bases.data_ptr(), bases.numel(),
                                     torch.cuda.current_stream(bases.device).cuda_stream)
    if code:
        raise RuntimeError("panvram_b200 apply_case: " + (_lib.pv_kernels_last_error() or b"").decode())
    return bases


def sha256_file_bases(path):
    b = ctypes.create_string_buffer(65)
    _check(_lib.pv_sha256_file_bases(os.fsencode(path), b))
    return b.value.decode()


PV_WIN_BLOCK_PATH = 1
PV_WIN_FUSED = 2          # force the one-kernel form
PV_WIN_SPLIT = 4          # force the decode + emission pair
PV_WIN_TEST_WAIT = 16     # make every kernel's bounded copy wait expire (status 4), for testing that path


def PV_WIN_DEC_LANES(k):
    """flag: the split form's decode kernel runs k items per warp (1..32) instead of its size rule's choice"""
    return int(k) << 8
PV_BLOCK_CACHED = 0xFFFFFE




def work_bytes(dev, n, W):
    """Bytes of device scratch a window call with these sizes needs (pv_windows_work_bytes)."""
    return int(_lib.pv_windows_work_bytes(ctypes.byref(dev), int(n), int(W)))


def work_buffer(dev, device, n, W):
    """Fresh device scratch for one window call, from torch's caching allocator on the current stream (so calls on
    different streams never share it, and a captured graph keeps the one it was captured with alive)."""
    need = work_bytes(dev, n, W)
    return (torch.empty(need, dtype=torch.uint8, device=device) if need else None), need


def windows_cuda(dev, wasm, wstart, W, rc=None, tokens=False, apply_case=True, out=None, status=None, flags=0, wstatus=None, ids=None,
                 work=None):
    """out uint8 [n, W] (int64 [n, W] of ids when ids are given), status int32 [1] on the cohort's device: the window
    decode (pv_windows_ex / pv_windows_ids).
    dev: the DevCohort of device pointers; wasm / wstart: int64 device tensors [n]; rc: None or a [n] bool/uint8 device
    tensor; wstatus: None or a zeroed uint8 device tensor of at least n bytes rounded up to 4 (per-window status).
    Asynchronous on torch's current stream of that device."""
    n, W = int(wasm.numel()), int(W)
    if wstart.numel() != n:
        raise RuntimeError("assembly and start counts differ")
    if W < 0 or W >= (1 << 31):
        raise RuntimeError("W")
    device = wasm.device
    if out is None:
        out = torch.empty((n, W), dtype=torch.int64 if ids is not None else torch.uint8, device=device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=device)
    rp = None
    if rc is not None:
        if rc.numel() != n:
            raise RuntimeError("reverse_complement mask size")
        rp = rc.data_ptr()
    stream = torch.cuda.current_stream(device).cuda_stream
    if wstatus is not None and wstatus.numel() < (n + 3) // 4 * 4:
        raise RuntimeError("wstatus: n bytes rounded up to a multiple of 4")
    if work is None:
        work, need = work_buffer(dev, device, n, W)
    else:
        need = work_bytes(dev, n, W)
        if work.numel() < need:
            raise RuntimeError("scratch buffer too small")
    if ids is not None:
        if len(ids) != 5 or out.dtype != torch.int64:
            raise RuntimeError("token ids: five values, int64 output")
        idv = (ctypes.c_int64 * 5)(*[int(x) for x in ids])
        code = _lib.pv_windows_ids(ctypes.byref(dev), wasm.data_ptr(), wstart.data_ptr(), n, W, rp, idv, out.data_ptr(), status.data_ptr(),
                                   work.data_ptr() if work is not None else None, need, stream)
        if code:
            raise RuntimeError("panvram_b200 window launch: " + (_lib.pv_kernels_last_error() or b"").decode())
        return out, status
    code = _lib.pv_windows_ex(ctypes.byref(dev), wasm.data_ptr(), wstart.data_ptr(), n, W, rp, int(bool(tokens)), int(bool(apply_case)),
                              int(flags), out.data_ptr(), status.data_ptr(), wstatus.data_ptr() if wstatus is not None else None,
                              work.data_ptr() if work is not None else None, need, stream)
    if code:
        msg = (_lib.pv_kernels_last_error() or b"").decode()
        raise RuntimeError(f"panvram_b200 window launch: {msg}")
    return out, status


def sample_coords(cum, valid, ctg, u, r, p, rc_mode, asm, start, rc=None, coords=None, status=None):
    """sample()'s coordinate arithmetic in one launch (pv_sample_coords): writes asm / start (int64 [n]), rc (uint8
    [n], rc_mode 1 or 2), coords (int64 [n, 4]) when given, and zeroes status when given. cum / valid: the per-W
    prefix sums and valid-start counts of the contigs; ctg: the cohort's contig arrays; u: int64 draws; r: the float
    draws (rc_mode 2, strand = r < p). Asynchronous on torch's current stream of u's device."""
    n = int(u.numel())
    ptr = lambda t: t.data_ptr() if t is not None else None
    code = _lib.pv_sample_coords(cum.data_ptr(), valid.data_ptr(), ctg["ctg_asm"].data_ptr(), ctg["ctg_boff"].data_ptr(),
                                 ctg["ctg_local"].data_ptr(), int(cum.numel()), u.data_ptr(), ptr(r), float(p), int(rc_mode), n,
                                 asm.data_ptr(), start.data_ptr(), ptr(rc), ptr(coords), ptr(status),
                                 torch.cuda.current_stream(u.device).cuda_stream)
    if code:
        raise RuntimeError("panvram_b200 sample coordinates: " + (_lib.pv_kernels_last_error() or b"").decode())


def sample_draw_coords(cum, valid, ctg, total, rng, p, rc_mode, n, asm, start, rc=None, coords=None, status=None, u_out=None,
                       r_out=None, seed=0, offset=0):
    """sample_coords with the draws made in the same launch exactly as torch.randint(0, total, (n,)) and (rc_mode 2)
    torch.rand(n) would make them on a CUDA generator whose seed and Philox offset are in rng (int64 [3] on the device:
    seed, offset, 0; the launch advances rng's offset as those calls advance the generator's) or, with rng None, are
    seed and offset (the caller advances its generator). u_out / r_out: the draws, when given. Asynchronous on torch's
    current stream of asm's device."""
    ptr = lambda t: t.data_ptr() if t is not None else None
    code = _lib.pv_sample_draw_coords(cum.data_ptr(), valid.data_ptr(), ctg["ctg_asm"].data_ptr(), ctg["ctg_boff"].data_ptr(),
                                      ctg["ctg_local"].data_ptr(), int(cum.numel()), int(total), ptr(rng), int(seed) & ((1 << 64) - 1),
                                      int(offset), float(p), int(rc_mode), int(n), asm.data_ptr(), start.data_ptr(), ptr(rc), ptr(coords),
                                      ptr(status), ptr(u_out), ptr(r_out), torch.cuda.current_stream(asm.device).cuda_stream)
    if code:
        raise RuntimeError("panvram_b200 sample draws: " + (_lib.pv_kernels_last_error() or b"").decode())


def torch_draw_geometry(n, total, rc_mode, sm_count, threads_per_sm):
    """(threads, offset consumed by randint, by randint and rand) of torch's draws for sample() on such a device."""
    t, a, b = _U64(), _U64(), _U64()
    if _lib.pv_torch_draw_geometry(int(n), int(total), int(rc_mode), int(sm_count), int(threads_per_sm), ctypes.byref(t), ctypes.byref(a),
                                   ctypes.byref(b)):
        raise ValueError((_lib.pv_kernels_last_error() or b"").decode())
    return t.value, a.value, b.value


def coords_from_host(asm, start, rc, device):
    """Pinned host coordinates (int64 asm / start, uint8 rc or None) -> device tensors, gathered by a kernel through the
    host arrays' mapped addresses (pv_coords_from_host) on the current stream; None if an array is not pinned."""
    n = int(asm.numel())
    a = torch.empty(n, dtype=torch.int64, device=device)
    s = torch.empty(n, dtype=torch.int64, device=device)
    r = torch.empty(n, dtype=torch.uint8, device=device) if rc is not None else None
    code = _lib.pv_coords_from_host(asm.data_ptr(), start.data_ptr(), rc.data_ptr() if rc is not None else None, n, a.data_ptr(),
                                    s.data_ptr(), r.data_ptr() if r is not None else None,
                                    torch.cuda.current_stream(device).cuda_stream)
    if code == PV_EARG:
        return None
    if code:
        raise RuntimeError("panvram_b200 coordinates from host: " + (_lib.pv_kernels_last_error() or b"").decode())
    return a, s, r


PV_CKPT_BAD = 1
PV_CKPT_CACHED = 2
TRACE_PHASES = ("start", "located", "decode_start", "decoded", "emit_start", "header_copied", "emitted")


def windows_trace(dev, wasm, wstart, W, rc=None, tokens=False, apply_case=True, flags=0):
    """windows_cuda with the per-item %globaltimer trace (pv_windows_trace) -> (out, status, trace): trace a numpy
    uint64 [items, 8] array, read after the call (one sync)."""
    n, W = int(wasm.numel()), int(W)
    device = wasm.device
    items = int(_lib.pv_windows_items(ctypes.byref(dev), n, W))
    out = torch.empty((n, W), dtype=torch.uint8, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    trace = torch.zeros((max(1, items), 8), dtype=torch.int64, device=device)
    work, need = work_buffer(dev, device, n, W)
    code = _lib.pv_windows_trace(ctypes.byref(dev), wasm.data_ptr(), wstart.data_ptr(), n, W, rc.data_ptr() if rc is not None else None,
                                 int(bool(tokens)), int(bool(apply_case)), int(flags), out.data_ptr(), status.data_ptr(),
                                 work.data_ptr() if work is not None else None, need, trace.data_ptr(), items,
                                 torch.cuda.current_stream(device).cuda_stream)
    if code:
        raise RuntimeError("panvram_b200 traced window launch: " + (_lib.pv_kernels_last_error() or b"").decode())
    return out, status, trace[:items].cpu().numpy().view(np.uint64)


def trace_summary(trace):
    """Per-phase durations (ns) of the items that were decoded (state 1 = decoded and emitted): mean, median, p99 and
    max of each phase, the items' span from the call's first start to their end, and the decode's bases and ops."""
    t = trace.astype(np.int64)
    info = trace[:, 7]
    state = (info >> np.uint64(8)) & np.uint64(15)
    form = (info >> np.uint64(12)) & np.uint64(3)
    ok = (state == 1) & (t[:, 6] > 0)
    r = {"items": int(len(t)), "decoded": int(ok.sum()),
         "states": {int(k): int(v) for k, v in zip(*np.unique(state, return_counts=True))}}
    hv = (state == 2) & (t[:, 6] > 0)               # the general path's items (pv_heavy_kernel): their whole time
    if hv.any():
        h0 = t[hv, 0]
        r["heavy_ns"] = {"count": int(hv.sum()), "max_end": float((t[hv, 6] - t[:, 0][t[:, 0] > 0].min()).max()),
                         "max_span": float((t[hv, 6] - h0).max())}
    if not ok.any():
        return r
    t, info, form = t[ok], info[ok], form[ok]
    t0 = t[:, 0][t[:, 0] > 0].min()
    split = form == 2

    def stats(x):
        x = np.asarray(x, dtype=np.float64)
        return {"mean": float(x.mean()), "p50": float(np.median(x)), "p99": float(np.percentile(x, 99)), "max": float(x.max())}
    r["locate_ns"] = stats(t[:, 1] - t[:, 0])
    r["wait_ns"] = stats(t[:, 2] - t[:, 1])
    r["decode_ns"] = stats(t[:, 3] - t[:, 2])
    emit0 = np.where(split, t[:, 5], t[:, 3])
    r["emit_ns"] = stats(t[:, 6] - emit0)
    if split.any():
        r["emit_queue_ns"] = stats((t[:, 4] - t[:, 3])[split])
        r["emit_header_ns"] = stats((t[:, 5] - t[:, 4])[split])
    r["end_ns"] = stats(t[:, 6] - t0)
    r["call_ns"] = float(t[:, 6].max() - t0)
    r["bases_decoded"] = stats(info >> np.uint64(48))
    r["ops"] = stats((info >> np.uint64(16)) & np.uint64(0xFFFF))
    r["sms"] = int(len(np.unique(info & np.uint64(0xFF))))
    return r




def index_build(dev, nblocks, ckpt_shift, device):
    """The cohort's checkpoint index on `device` (pv_index_build: every block decoded once on the device; blocks in the
    block cache skipped) -> (uint8 tensor of pv_ckpt records, int32 tensor of each block's first lower-case run, number
    of blocks that failed to decode, int32 tensor of each block's decode cost: events + literal bytes of its costliest
    stride cell). Waits for it."""
    nbytes = int(_lib.pv_index_bytes(int(dev.Q), int(nblocks), int(ckpt_shift)))
    if not nbytes:
        raise ValueError(f"checkpoint stride 2^{ckpt_shift}: a power of two from 256 to the block size {dev.Q}")
    out = torch.empty(nbytes, dtype=torch.uint8, device=device)
    brun = torch.empty(max(1, int(nblocks)), dtype=torch.int32, device=device)
    nbad = torch.zeros(1, dtype=torch.int64, device=device)
    cost = torch.zeros(max(1, int(nblocks)), dtype=torch.int16, device=device)
    with torch.cuda.device(device):
        code = _lib.pv_index_build(ctypes.byref(dev), int(nblocks), int(ckpt_shift), out.data_ptr(), nbad.data_ptr(), brun.data_ptr(),
                                   cost.data_ptr(), torch.cuda.current_stream(device).cuda_stream)
        if code:
            raise RuntimeError("panvram_b200 index: " + (_lib.pv_kernels_last_error() or b"").decode())
        torch.cuda.current_stream(device).synchronize()
    return out, brun, int(nbad.item()), cost.to(torch.int32) & 0xFFFF


def rc_reference(ref_padded, n, device):
    """The reverse-complement reference (pv_rc_reference) of a device reference (ref_padded: the uint8 tensor with 64
    bytes before the first base), in a tensor with the same 64-byte padding on each side."""
    out = torch.zeros(int(n) + 128, dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        code = _lib.pv_rc_reference(ref_padded.data_ptr() + 64, int(n), out.data_ptr() + 64, torch.cuda.current_stream(device).cuda_stream)
    if code:
        raise RuntimeError("panvram_b200 reverse-complement reference: " + (_lib.pv_kernels_last_error() or b"").decode())
    return out


def read_status(status):
    """The int32 status word (a CUDA tensor) after the work queued before this call on the current stream, as an int:
    stored by one device thread into a pinned host word (pv_status_to_host), then the stream waited for - so the read
    never queues behind other device-to-host copies, as status.item() would."""
    h = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    stream = torch.cuda.current_stream(status.device)
    if _lib.pv_status_to_host(status.data_ptr(), h.data_ptr(), stream.cuda_stream):
        raise RuntimeError("panvram_b200 status read: " + (_lib.pv_kernels_last_error() or b"").decode())
    stream.synchronize()
    return int(h[0])


def launches_per_call(n, W):
    return int(_lib.pv_windows_launches(int(n), int(W)))


def windows_form(cell, n, W, flags=0):
    """(kernel launches, decode items per warp) of a window call with these sizes: (1, 0) the fused kernel, (2, k) the
    split form with k items per decode warp, (0, 0) an empty call. cell: the cohort's checkpoint stride when it has an
    index (Cohort.item_cell), else its block size."""
    L, k = ctypes.c_int(), _U32()
    if _lib.pv_windows_form(int(cell), int(n), int(W), int(flags), ctypes.byref(L), ctypes.byref(k)):
        raise ValueError((_lib.pv_kernels_last_error() or b"").decode())
    return L.value, k.value
