"""panvram_b200.Cohort - the reference's public API (panvram/cohort.py:21-234) over the B200 decode path.

A cohort of refrel3 v1 archives against one decoded reference, resident on one GPU; windows and coordinate slices are
decoded on the card by the one-kernel window decode (include/panvram_b200.h pv_windows). Same methods, arguments,
coordinates, errors and status text as the reference. Differences, by design:
  * GPU only: device="cpu" is refused (the reference's CPU decoder is this repository's test oracle, not a product
    path); fasta() decodes on the GPU and rebuilds / verifies the FASTA on the host.
  * sample() keeps the reference's torch call sequence (same generator, same coordinates) but caches the per-W
    valid-start total, so a call makes no host sync unless check=True.
"""
import glob
import os
import re

import torch

from . import _C

DATASETS = ("q4k", "q16k")
STATUS_TEXT = "GPU decode failed (status {}: 1 corrupt block, 4 bounded wait expired, 8 window outside an assembly)"


def _arch_ok(device):
    cap = torch.cuda.get_device_capability(device)
    if cap < (10, 0):
        raise RuntimeError(f"panvram_b200 is built for sm_100a (B200); {torch.cuda.get_device_name(device)} is sm_{cap[0]}{cap[1]}")


class Cohort:
    """Open with Cohort.open(dir, device=...). Coordinates are 0-based; a contig is its FASTA header up to the first
    space or tab, or its index in the assembly; an assembly is its name (archive file name without .<dataset>.rr3) or
    its index."""

    def __init__(self, core, names, device):
        self._core, self.names, self.device = core, list(names), torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("panvram_b200 decodes on the GPU only: open the cohort with device='cuda' or 'cuda:N'")
        if not torch.cuda.is_available():
            raise RuntimeError("panvram_b200 needs a CUDA device (none is visible)")
        _arch_ok(self.device)
        self._index = {n: i for i, n in enumerate(self.names)}
        self._ctg_names = [{c[0]: k for k, c in enumerate(core.contigs(i))} for i in range(core.n)]
        pools = core.pools()
        with torch.cuda.device(self.device):
            self._dev = {k: torch.from_numpy(v).to(self.device) for k, v in pools.items() if not k.startswith("ctg_")}
            self._ctg = {k: torch.from_numpy(pools[k]).to(self.device) for k in ("ctg_asm", "ctg_local", "ctg_boff", "ctg_len")}
        d = self._dev
        self._devc = _C.DevCohort(ref=d["ref_padded"].data_ptr() + 64, ref_n=core.ref_bases, payload=d["payload"].data_ptr(),
                                  blocks=d["blocks"].data_ptr(), asms=d["asms"].data_ptr(), tabs=d["tabs"].data_ptr(),
                                  low=d["low"].data_ptr(), nasm=core.n, Q=core.Q, pad=0)
        self._valid = {}
        self._info = [core.info(i) for i in range(core.n)]
        # a list to collect (start, end) CUDA events around each window-kernel launch (measurement); None = off
        self.kernel_events = None

    @classmethod
    def open(cls, path, device="cuda", dataset="q4k", reference=None, threads=0, assemblies=None,
             packed_reference=False, compact_blocks=False):
        """Open the cohort directory `path`: every `*.<dataset>.rr3` in it (sorted by name; `assemblies` = a list of
        names to take only those) and the reference they were encoded against - `reference` if given, else
        `path/reference.fa`, else the file named in the archives' header in `path`. Every archive is checked before
        any decode (header XXH3, reference SHA-256 and size, sections, tables). One block size per cohort.
        device: "cuda" or "cuda:N"."""
        if dataset is not None and not re.fullmatch(r"q\d+k", dataset):
            raise ValueError(f"dataset: {DATASETS} (or another q<N>k suffix), or None for every *.rr3")
        pat = f"*.{dataset}.rr3" if dataset else "*.rr3"
        files = sorted(glob.glob(os.path.join(path, pat)))
        suffix = f".{dataset}.rr3" if dataset else ".rr3"
        names = [os.path.basename(f)[: -len(suffix)] for f in files]
        if assemblies is not None:
            want = list(assemblies)
            have = dict(zip(names, files))
            missing = [a for a in want if a not in have]
            if missing:
                raise FileNotFoundError(f"not in {path}: {missing[:5]}")
            names, files = want, [have[a] for a in want]
        if not files:
            raise FileNotFoundError(f"no {pat} in {path}")
        if reference is None:
            cand = os.path.join(path, "reference.fa")
            if not os.path.exists(cand):
                with open(files[0], "rb") as f:
                    h = f.read(138 + 65535)
                nl = h[136] | h[137] << 8
                cand = os.path.join(path, h[138:138 + nl].decode())
            reference = cand
        if not os.path.exists(reference):
            raise FileNotFoundError(f"reference {reference} not found (pass reference=)")
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("panvram_b200 decodes on the GPU only: open the cohort with device='cuda' or 'cuda:N'")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        core = _C.Core(os.fspath(reference), [os.fspath(f) for f in files], int(threads), bool(packed_reference), bool(compact_blocks))
        return cls(core, names, device)

    # ------------------------------------------------------------------ description
    def __len__(self):
        return len(self.names)

    @property
    def block_size(self):
        return self._core.Q

    @property
    def reference_sha256(self):
        return self._core.ref_sha256

    def info(self, assembly):
        return dict(self._info[self._asm(assembly)])

    def contigs(self, assembly):
        """[(name, header, length, offset in the base stream, line width)] of an assembly."""
        return self._core.contigs(self._asm(assembly))

    def resident_bytes(self):
        """Bytes of the cohort on its device (reference included), by component. Keys follow the reference's where
        the component is the same (P payload, tab model tables, ref reference); blocks is the block table (the
        reference's off + st), low the lower-case runs (low_s + low_l), asm the per-assembly records."""
        d = self._dev
        r = {"P": d["payload"].numel(), "blocks": d["blocks"].numel() * 8, "tab": d["tabs"].numel(), "low": d["low"].numel() * 8,
             "ref": d["ref_padded"].numel(), "asm": d["asms"].numel()}
        r["total"] = sum(r.values())
        return r

    # ------------------------------------------------------------------ decode
    def _asm(self, a):
        if isinstance(a, str):
            if a not in self._index:
                raise KeyError(f"no assembly {a}")
            return self._index[a]
        a = int(a)
        if not 0 <= a < len(self.names):
            raise IndexError(f"assembly index {a}")
        return a

    def _contig(self, a, c):
        if isinstance(c, str):
            if c not in self._ctg_names[a]:
                raise KeyError(f"no contig {c} in {self.names[a]}")
            return self._ctg_names[a][c]
        c = int(c)
        if not 0 <= c < len(self._ctg_names[a]):
            raise IndexError(f"contig index {c}")
        return c

    def _launch(self, asm, start, W, reverse_complement, tokens, apply_case, out=None, status=None, flags=0):
        dev = self.device
        with torch.cuda.device(dev):
            asm = torch.as_tensor(asm).to(dev, torch.int64).contiguous()
            start = torch.as_tensor(start).to(dev, torch.int64).contiguous()
            rc = None
            if reverse_complement is not None:
                rc = torch.as_tensor(reverse_complement).to(dev, torch.uint8).contiguous()
            if self.kernel_events is None:
                return _C.windows_cuda(self._devc, asm, start, W, rc, tokens, apply_case, out=out, status=status, flags=flags)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            out = torch.empty((asm.numel(), int(W)), dtype=torch.uint8, device=dev) if out is None else out
            status = torch.zeros(1, dtype=torch.int32, device=dev) if status is None else status
            a.record()
            r = _C.windows_cuda(self._devc, asm, start, W, rc, tokens, apply_case, out=out, status=status, flags=flags)
            b.record()
            self.kernel_events.append((a, b))
            return r

    def windows(self, asm, start, W, reverse_complement=None, tokens=False, check=True):
        """Bases [start, start + W) of assembly asm[i] (start = offset in the assembly's base stream: contigs
        concatenated in file order) for every i -> uint8 [n, W] on the cohort's device. reverse_complement: None or a
        bool tensor [n]. tokens: A/a 0, C/c 1, G/g 2, T/t 3, anything else 4; else the FASTA's bytes, case kept.
        check: wait for the kernel and raise if any block failed to decode (one device sync)."""
        out, status = self._launch(asm, start, int(W), reverse_complement, tokens, True)
        if check:
            s = int(status.item())
            if s:
                raise RuntimeError(STATUS_TEXT.format(s))
        return out

    def sample(self, n, W, generator=None, reverse_complement=False, tokens=False, return_coords=False, check=True):
        """n windows of W bases, uniform over every (assembly, contig, start) with start + W <= contig length (a
        window never crosses contigs) -> uint8 [n, W] on the cohort's device. generator: a torch.Generator (its device
        draws the numbers). reverse_complement: False, True, or p in (0, 1) - each window reverse-complemented with
        probability p. return_coords: also an int64 [n, 4] tensor (assembly, contig index, start in the contig,
        reverse-complemented 0/1)."""
        n, W = int(n), int(W)
        if W <= 0 or n < 0:
            raise ValueError("W must be positive, n non-negative")
        if W not in self._valid:
            v = (self._ctg["ctg_len"] - W + 1).clamp_min(0)
            cum = torch.cumsum(v, 0)
            self._valid[W] = (cum, v, int(cum[-1].item()) if cum.numel() else 0)
        cum, v, total = self._valid[W]
        if total == 0:
            raise ValueError(f"no contig of {W} bases or more")
        gdev = generator.device if generator is not None else self.device
        u = torch.randint(0, total, (n,), generator=generator, device=gdev, dtype=torch.int64).to(self.device)
        k = torch.searchsorted(cum, u, right=True)
        pos = u - (cum[k] - v[k])
        asm = self._ctg["ctg_asm"][k]
        start = self._ctg["ctg_boff"][k] + pos
        if reverse_complement is True:
            rc = torch.ones(n, dtype=torch.bool, device=self.device)
        elif reverse_complement is False or reverse_complement is None or reverse_complement == 0:
            rc = None
        else:
            p = float(reverse_complement)
            if not 0 < p <= 1:
                raise ValueError("reverse_complement: False, True or a probability")
            rc = (torch.rand(n, generator=generator, device=gdev) < p).to(self.device)
        x = self.windows(asm, start, W, rc, tokens, check)
        if not return_coords:
            return x
        strand = rc.to(torch.int64) if rc is not None else torch.zeros(n, dtype=torch.int64, device=self.device)
        return x, torch.stack([asm, self._ctg["ctg_local"][k], pos, strand], 1)

    def fetch(self, assembly, contig, start, length, reverse_complement=False, tokens=False):
        """Bases [start, start + length) of a contig (0-based) -> uint8 [length] on the cohort's device."""
        a = self._asm(assembly)
        c = self._contig(a, contig)
        name, _, clen, boff, _ = self._core.contigs(a)[c]
        start, length = int(start), int(length)
        if start < 0 or length < 0 or start + length > clen:
            raise IndexError(f"{self.names[a]} {name}:{start}+{length} outside the contig ({clen} bases)")
        asm = torch.tensor([a], dtype=torch.int64)
        st = torch.tensor([boff + start], dtype=torch.int64)
        rc = torch.tensor([bool(reverse_complement)]) if reverse_complement else None
        return self.windows(asm, st, length, rc, tokens)[0]

    def _decode(self, a, chunk, out, apply_case):
        n = self._info[a]["bases"]
        if out is None or out.numel() < n:
            out = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        out = out[:n]
        asm = torch.tensor([a], dtype=torch.int64)
        for s in range(0, n, chunk):
            k = min(chunk, n - s)
            x, status = self._launch(asm, torch.tensor([s], dtype=torch.int64), k, None, False, apply_case)
            st = int(status.item())
            if st:
                raise RuntimeError(STATUS_TEXT.format(st))
            out[s:s + k].copy_(x[0], non_blocking=False)
        return out

    def decode(self, assembly, chunk=1 << 28, out=None):
        """The whole base stream of an assembly (contigs concatenated, case as in the FASTA) decoded on the cohort's
        device in chunks of `chunk` bases -> uint8 [bases] on the host (pinned; `out` reused if given)."""
        return self._decode(self._asm(assembly), int(chunk), out, True)

    def check_full(self, assembly, out=None):
        """Full decode on the cohort's device, the FASTA rebuilt from it (layout from the contig table) hashed with
        XXH3 -> (equal to the header's source XXH3, the hash "%016llx")."""
        a = self._asm(assembly)
        h = self._core.fasta_xxh3(a, self.decode(a, out=out))
        return h == self._info[a]["fasta_xxh3"], h

    def fasta(self, assembly, verify=True):
        """Full decode of an assembly -> the FASTA file's bytes. verify: every block XXH3 (if present) and the XXH3 of
        the rebuilt FASTA against the header's (the source file's). Decoded on the GPU, rebuilt on the host."""
        a = self._asm(assembly)
        path = self._info[a]["path"]
        try:
            b = self._decode(a, 1 << 28, None, False)
        except RuntimeError:
            raise _C.FormatError(path + ": block decode failed")
        if verify and self._core.first_bad_block(a, b) >= 0:
            raise _C.FormatError(path + ": block XXH3 mismatch")
        self._core.apply_case(a, b)
        fa = self._core.fasta_bytes(a, b)
        if verify:
            import xxhash
            if "%016x" % xxhash.xxh3_64_intdigest(fa) != self._info[a]["fasta_xxh3"]:
                raise _C.FormatError(path + ": FASTA XXH3 differs from the header")
        return fa
