"""panvram_b200.Cohort - the reference's public API (panvram/cohort.py:21-234) over the B200 decode path.

A cohort of refrel3 v1 archives against one decoded reference, resident on one GPU; windows and coordinate slices are
decoded on the card by the window kernels (include/panvram_b200.h pv_windows). Same methods, arguments,
coordinates, errors and status text as the reference. Differences, by design:
  * GPU only: device="cpu" is refused (the reference's CPU decoder is this repository's test oracle, not a product
    path); fasta() decodes on the GPU and rebuilds / verifies the FASTA on the host.
  * sample() keeps the reference's draws (the same torch.randint / torch.rand calls on the same generator, so the
    same coordinates) but does the arithmetic from draws to coordinates in one kernel (pv_sample_coords) and caches
    the per-W valid-start total, so a call makes no host sync unless check=True.
"""
import glob
import os
import re

import numpy as np
import torch

from . import _C

DATASETS = ("q4k", "q16k")
# torch releases (major.minor) whose randint / rand CUDA kernels (launch geometry, Philox state per thread, element
# order, transforms) the coordinate kernel's restatement of them was checked against bit for bit
# (tests/test_gpu_coords.py). With any other torch, sample() and Cohort.sampler make the draws with torch's own calls:
# the same coordinates, at the cost of their launches.
TORCH_DRAWS_CHECKED = ("2.11",)


def _native_draws():
    return ".".join(torch.__version__.split("+")[0].split(".")[:2]) in TORCH_DRAWS_CHECKED
STATUS_TEXT = "GPU decode failed (status {}: 1 corrupt block, 4 bounded wait expired, 8 window outside an assembly)"


def _arch_ok(device):
    cap = torch.cuda.get_device_capability(device)
    if cap < (10, 0):
        raise RuntimeError(f"panvram_b200 is built for sm_100a (B200); {torch.cuda.get_device_name(device)} is sm_{cap[0]}{cap[1]}")


def _pinned_coords(asm, start, rc, dev):
    """Coordinates given as contiguous pinned host tensors (int64, and bool / uint8 strands) -> device tensors gathered
    by one kernel through their mapped addresses (no copy engine: a device-to-host copy in flight, such as the previous
    batch's windows, does not delay them); None for any other input."""
    ts = (asm, start) + ((rc,) if rc is not None else ())
    if not all(isinstance(t, torch.Tensor) and t.device.type == "cpu" and t.is_contiguous() for t in ts):
        return None
    if asm.dtype != torch.int64 or start.dtype != torch.int64 or asm.numel() != start.numel():
        return None
    if rc is not None:
        if rc.dtype == torch.bool:
            rc = rc.view(torch.uint8)
        if rc.dtype != torch.uint8 or rc.numel() != asm.numel():
            return None
    if not all(t.is_pinned() for t in ts):
        return None
    return _C.coords_from_host(asm, start, rc, dev)


def _strand_mode(reverse_complement):
    """sample()'s reverse_complement -> (mode, p): 0 none, 1 all, 2 each window with probability p"""
    if reverse_complement is True:
        return 1, 0.0
    if reverse_complement is False or reverse_complement is None or reverse_complement == 0:
        return 0, 0.0
    p = float(reverse_complement)
    if not 0 < p <= 1:
        raise ValueError("reverse_complement: False, True or a probability")
    return 2, p


class Cohort:
    """Open with Cohort.open(dir, device=...). Coordinates are 0-based; a contig is its FASTA header up to the first
    space or tab, or its index in the assembly; an assembly is its name (archive file name without .<dataset>.rr3) or
    its index."""

    CHECKPOINT_STRIDE = 2048

    def __init__(self, core, names, device, block_cache=True, checkpoint_stride=None):
        self._core, self.names, self.device = core, list(names), torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("panvram_b200 decodes on the GPU only: open the cohort with device='cuda' or 'cuda:N'")
        if not torch.cuda.is_available():
            raise RuntimeError("panvram_b200 needs a CUDA device (none is visible)")
        _arch_ok(self.device)
        self._index = {n: i for i, n in enumerate(self.names)}
        self._ctg_tables = {}
        self._ctg_names = [{c[0]: k for k, c in enumerate(core.contigs(i))} for i in range(core.n)]
        pools = core.pools()
        packed, compact = core.packed_reference, core.compact_blocks
        with torch.cuda.device(self.device):
            self._dev = {k: torch.from_numpy(v).to(self.device) for k, v in pools.items()
                         if isinstance(v, np.ndarray) and v.size and not k.startswith("ctg_")}
            self._ctg = {k: torch.from_numpy(pools[k]).to(self.device) for k in ("ctg_asm", "ctg_local", "ctg_boff", "ctg_len")}
        d = self._dev
        ptr = lambda k: d[k].data_ptr() if k in d else None
        self._devc = _C.DevCohort(ref=None if packed else d["ref_padded"].data_ptr() + 64, ref_n=core.ref_bases,
                                  payload=d["payload"].data_ptr(), blocks=None if compact else ptr("blocks"), asms=d["asms"].data_ptr(),
                                  tabs=d["tabs"].data_ptr(), tab_max=pools["tab_max"], low=d["low"].data_ptr(), cache=None,
                                  nasm=core.n, Q=core.Q, pad=0,
                                  pref=ptr("pref") if packed else None, pruns=ptr("pruns") if packed else None,
                                  pidx=ptr("pidx") if packed else None, pnruns=pools["pnruns"],
                                  groups=ptr("groups") if compact else None, btab=ptr("btab") if compact else None,
                                  bexc=ptr("bexc") if compact else None, packed=int(packed), compact=int(compact))
        self._valid = {}
        self._incs = {}
        self._info = [core.info(i) for i in range(core.n)]
        # a list to collect (start, end) CUDA events around each window-kernel launch (measurement); None = off
        self.kernel_events = None
        self._cache, self.cached_blocks = None, 0
        self._fetch_host = self._fetch_rc = None
        # PV_WIN_* flags added to every window launch: _C.PV_WIN_FUSED / PV_WIN_SPLIT pin the kernel form (default: by
        # call size); the output is the same
        self.launch_flags = 0
        self._ckpt, self.checkpoint_stride, self.bad_blocks = None, 0, 0
        stride = self.CHECKPOINT_STRIDE if checkpoint_stride is None else int(checkpoint_stride)
        cost = self._build_index(min(stride, core.Q)) if stride else None
        if block_cache:
            self._build_block_cache(pools, cost)
        # the reference reverse-complemented, for the byte form: the split emission reads reverse-complement copies
        # forward from it (one more copy of the reference, ref_n bytes)
        self._rcref = None
        if not packed:
            self._rcref = _C.rc_reference(self._dev["ref_padded"], core.ref_bases, self.device)
            self._devc.rcref = self._rcref.data_ptr() + 64
        # the host copies of the reference and the payload are on the device now and read for nothing else: free them
        # (at config 2 that is ~12 GB of host memory per process, per GPU)
        torch.cuda.synchronize(self.device)
        del pools
        core.release_uploaded()

    def _build_index(self, stride):
        """The checkpoint index (pv_index_build): every block decoded once on the device, its decoder state kept at the
        last event boundary at or before each multiple of `stride` in the block. Window items then cover one stride
        each: each decodes from its checkpoint to the end of its range only, so a window's serial chains are about a
        stride long instead of a block, and the blocks outside the window's span are not decoded. Decoding every block
        here also validates it: a block that fails is marked, and windows touching it report status 1 exactly as when
        they decoded it in full. Alongside, each block's first lower-case run (4 bytes per block), so an item finds its
        runs in a step or two instead of a binary search of the assembly's runs. -> each block's decode cost (device
        int32: the events and literal bytes of its costliest stride cell), which picks blocks for the block cache."""
        if stride & (stride - 1) or not 256 <= stride <= self._core.Q:
            raise ValueError(f"checkpoint_stride: a power of two from 256 to the block size ({self._core.Q}), or 0")
        shift = stride.bit_length() - 1
        asms = self._dev["asms"].cpu().numpy().view(np.uint64).reshape(-1, 8)
        nblocks = int(asms[:, 2].sum())
        self._ckpt, self._brun, self.bad_blocks, cost = _C.index_build(self._devc, nblocks, shift, self.device)
        self._devc.ckpt, self._devc.ckpt_shift, self._devc.brun = self._ckpt.data_ptr(), shift, self._brun.data_ptr()
        self.checkpoint_stride = stride
        return cost

    @property
    def item_cell(self):
        """The bases one work item of the window kernels covers: the checkpoint stride, or the block size without an
        index."""
        return self.checkpoint_stride or self._core.Q

    CACHE_BYTES = 4 << 30
    # with an index: also cache this fraction of the blocks, the costliest to decode (their costliest stride cell), so
    # that no window item's serial chain is much longer than a typical one's (a call lasts as long as its longest chain)
    CACHE_COSTLY = 0.002

    def _build_block_cache(self, pools, cost=None):
        """Decode once, into an HBM cache, the blocks whose rANS stream is at least Q/32 bytes - literal-heavy novel
        sequence, whose serial decode is many times longer than a typical block's - and, given the index's block costs,
        the CACHE_COSTLY fraction of blocks whose costliest stride cell costs the most; point their block-table entries
        (and their checkpoints) at the cache: windows then copy those bytes instead of decoding them. A block that
        fails to decode stays uncached, so a window touching it still reports status 1. At most CACHE_BYTES (the
        costliest, else the longest streams, first)."""
        Q = self._core.Q
        compact = self._core.compact_blocks
        if compact:
            plen = (pools["btab"][: len(pools["btab"]) - _C.PV_BLK_GROUP] & np.uint32(0xFFFF)).astype(np.int64)
        else:
            plen = (pools["blocks"][0::2] >> np.uint64(40)).astype(np.int64)
        want = (plen >= max(64, Q // 32)) & (plen < _C.PV_BLOCK_CACHED)
        score = plen
        if cost is not None and len(cost) == len(plen) and self.CACHE_COSTLY > 0:
            k = max(1, int(len(cost) * (1.0 - self.CACHE_COSTLY)))
            cut = int(torch.kthvalue(cost.float(), k).values.item())
            c = cost.cpu().numpy()
            want |= (c > max(cut, 0)) & (plen < _C.PV_BLOCK_CACHED)
            score = c
        cand = np.nonzero(want)[0]
        if len(cand) == 0:
            return
        if len(cand) * Q > self.CACHE_BYTES:
            cand = np.sort(cand[np.argsort(-score[cand], kind="stable")[: self.CACHE_BYTES // Q]])
        asms = pools["asms"].view(np.uint64).reshape(-1, 8)
        base, nbases = asms[:, 1].astype(np.int64), asms[:, 0].astype(np.int64)
        a = np.searchsorted(base, cand, side="right") - 1
        start = (cand - base[a]) * Q
        W = np.minimum(Q, nbases[a] - start)
        n = len(cand)
        full = np.nonzero(W == Q)[0]
        dev = self.device
        with torch.cuda.device(dev):
            # row i of the decode is block cand[i] (block order); the surviving blocks take cache slots in that order
            rows = torch.empty((n, Q), dtype=torch.uint8, device=dev)
            ws = torch.zeros((n + 3) // 4 * 4, dtype=torch.uint8, device=dev)
            at = torch.from_numpy(a).to(dev)
            st = torch.from_numpy(start).to(dev)
            if len(full):
                fi = torch.from_numpy(full).to(dev)
                wf = torch.zeros((len(full) + 3) // 4 * 4, dtype=torch.uint8, device=dev)
                out, _ = _C.windows_cuda(self._devc, at[fi], st[fi], Q, None, False, False, wstatus=wf)
                rows[fi] = out
                ws[fi] = wf[:len(full)]
            for i in np.nonzero(W < Q)[0]:
                w4 = torch.zeros(4, dtype=torch.uint8, device=dev)
                _C.windows_cuda(self._devc, at[i:i + 1], st[i:i + 1], int(W[i]), None, False, False,
                                out=rows[i:i + 1, :int(W[i])], wstatus=w4)
                ws[i:i + 1].copy_(w4[:1])
            ok = (ws[:n] == 0).cpu().numpy()
            keep = np.nonzero(ok)[0]
            cache = torch.zeros(64 + len(keep) * Q + 64, dtype=torch.uint8, device=dev)
            if len(keep):
                cache[64:64 + len(keep) * Q].view(len(keep), Q).copy_(rows[torch.from_numpy(keep).to(dev)])
            del rows
            blocks = cand[keep]
            if len(blocks) and compact:
                g = self._dev["groups"].cpu().numpy().view(_C.BLK_GROUP)
                grp_base = asms[:, 7].astype(np.int64)
                ab = a[keep]
                k = blocks - base[ab]
                gi = grp_base[ab] + k // _C.PV_BLK_GROUP
                np.bitwise_or.at(g["cache_mask"], gi, (np.uint32(1) << (k % _C.PV_BLK_GROUP).astype(np.uint32)))
                counts = np.zeros(len(g), np.int64)
                np.add.at(counts, gi, 1)
                g["cache_base"] = (np.cumsum(counts) - counts).astype(np.uint32)
                self._dev["groups"].copy_(torch.from_numpy(g.view(np.uint8)).to(dev))
            elif len(blocks):
                blk = self._dev["blocks"].view(torch.int64)
                vals = torch.from_numpy((np.arange(len(blocks), dtype=np.uint64) | np.uint64(_C.PV_BLOCK_CACHED << 40)).view(np.int64)).to(dev)
                blk[torch.from_numpy(2 * blocks).to(dev)] = vals
            if len(blocks) and self._ckpt is not None:
                # their checkpoints: every cell of a cached block says so, with the block's cache row (as the index
                # build writes them for blocks it finds cached)
                ncell = Q // self.checkpoint_stride
                rec = self._ckpt.view(torch.int32).view(-1, 8)
                rows = (torch.from_numpy(blocks.astype(np.int64)).to(dev)[:, None] * ncell + torch.arange(ncell, device=dev)).reshape(-1)
                new = torch.zeros((len(rows), 8), dtype=torch.int32, device=dev)
                new[:, 1] = torch.arange(len(blocks), dtype=torch.int32, device=dev).repeat_interleave(ncell)
                new[:, 7] = _C.PV_CKPT_CACHED << 16
                rec[rows] = new
            torch.cuda.synchronize(dev)
        self._cache, self.cached_blocks = cache, int(len(keep))
        self._devc.cache = cache.data_ptr() + 64

    @classmethod
    def open(cls, path, device="cuda", dataset="q4k", reference=None, threads=0, assemblies=None,
             packed_reference=False, compact_blocks=False, block_cache=True, checkpoint_stride=None):
        """Open the cohort directory `path`: every `*.<dataset>.rr3` in it (sorted by name; `assemblies` = a list of
        names to take only those) and the reference they were encoded against - `reference` if given, else
        `path/reference.fa`, else the file named in the archives' header in `path`. Every archive is checked before
        any decode (header XXH3, reference SHA-256 and size, sections, tables). One block size per cohort.
        device: "cuda" or "cuda:N". block_cache: decode the long (literal-heavy) blocks once at open and serve them
        from HBM (same output; see _build_block_cache). Opt-in compact resident forms (same archives, same output):
        packed_reference - the reference in 2 bits per base plus its runs of other bytes instead of a byte per base;
        compact_blocks - the block table as 32-byte records per 32 blocks plus 4 bytes per block instead of 16.
        checkpoint_stride: the decoder checkpoint index built on the device at open (see _build_index): a checkpoint
        every this many bases of each block (a power of two from 256 to the block size; None: 2048, capped at the block
        size; 0: no index - every window item then decodes its whole block). Same output either way; 32 bytes per
        checkpoint of device memory."""
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
        return cls(core, names, device, block_cache=block_cache, checkpoint_stride=checkpoint_stride)

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
        a = self._asm(assembly)
        if a not in self._ctg_tables:
            self._ctg_tables[a] = self._core.contigs(a)
        return list(self._ctg_tables[a])

    def resident_bytes(self):
        """Bytes of the cohort on its device (reference included), by component. Keys follow the reference's where
        the component is the same (P payload, tab model tables, ref reference); blocks is the block table (the
        reference's off + st), low the lower-case runs (low_s + low_l), asm the per-assembly records, cache the decoded
        long blocks, index the decoder checkpoints."""
        d = self._dev
        nb = lambda *ks: sum(d[k].numel() * d[k].element_size() for k in ks if k in d)
        r = {"P": nb("payload"), "blocks": nb("blocks", "groups", "btab", "bexc"), "tab": nb("tabs"), "low": nb("low"),
             "ref": nb("ref_padded", "pref", "pruns", "pidx") + (self._rcref.numel() if self._rcref is not None else 0), "asm": nb("asms"),
             "cache": self._cache.numel() if self._cache is not None else 0,
             "index": (self._ckpt.numel() + 4 * self._brun.numel()) if self._ckpt is not None else 0}
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

    def _launch(self, asm, start, W, reverse_complement, tokens, apply_case, out=None, status=None, flags=0, synced=False, ids=None):
        """synced: the caller waits for the stream before it returns (windows with check), so host inputs may be
        copied without a wait of their own."""
        dev = self.device
        with torch.cuda.device(dev):
            g = _pinned_coords(asm, start, reverse_complement, dev) if synced else None
            if g is not None:
                asm, start, rc = g
            else:
                asm = torch.as_tensor(asm).to(dev, torch.int64, non_blocking=synced).contiguous()
                start = torch.as_tensor(start).to(dev, torch.int64, non_blocking=synced).contiguous()
                rc = None
                if reverse_complement is not None:
                    rc = torch.as_tensor(reverse_complement)
                    if rc.dtype == torch.bool:
                        rc = rc.view(torch.uint8)                 # same bytes (0 / 1), no conversion kernel
                    rc = rc.to(dev, torch.uint8, non_blocking=synced).contiguous()
            flags |= self.launch_flags
            if self.kernel_events is None:
                return _C.windows_cuda(self._devc, asm, start, W, rc, tokens, apply_case, out=out, status=status, flags=flags, ids=ids)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            out = torch.empty((asm.numel(), int(W)), dtype=torch.int64 if ids is not None else torch.uint8, device=dev) if out is None else out
            status = torch.zeros(1, dtype=torch.int32, device=dev) if status is None else status
            a.record()
            r = _C.windows_cuda(self._devc, asm, start, W, rc, tokens, apply_case, out=out, status=status, flags=flags, ids=ids)
            b.record()
            self.kernel_events.append((a, b))
            return r

    def windows(self, asm, start, W, reverse_complement=None, tokens=False, check=True, token_ids=None):
        """Bases [start, start + W) of assembly asm[i] (start = offset in the assembly's base stream: contigs
        concatenated in file order) for every i -> uint8 [n, W] on the cohort's device. reverse_complement: None or a
        bool tensor [n]. tokens: A/a 0, C/c 1, G/g 2, T/t 3, anything else 4; else the FASTA's bytes, case kept.
        check: wait for the kernel and raise if any block failed to decode (one device sync).
        token_ids: five ids (for tokens 0..4) -> int64 [n, W] of those ids, mapped in the decode's store (what the
        Megatron adapter does as lut5[windows(tokens=True).long()], tools/megatron/panvram_loader.py:96-97)."""
        ids = None if token_ids is None else [int(x) for x in token_ids]
        if ids is not None and len(ids) != 5:
            raise ValueError("token_ids: five ids, for A C G T and anything else")
        out, status = self._launch(asm, start, int(W), reverse_complement, tokens or ids is not None, True, synced=bool(check), ids=ids)
        if check:
            with torch.cuda.device(self.device):
                s = _C.read_status(status)
            if s:
                raise RuntimeError(STATUS_TEXT.format(s))
        return out

    def trace_windows(self, asm, start, W, reverse_complement=None, tokens=False, flags=0):
        """windows() with a per-item trace of the kernels (pv_windows_trace: %globaltimer at every phase of every work
        item) -> (windows, status, summary dict of the phase times, the raw trace [items, 8]). For measurement; one
        sync. flags: PV_WIN_* (e.g. _C.PV_WIN_FUSED / PV_WIN_SPLIT to trace one kernel form)."""
        dev = self.device
        with torch.cuda.device(dev):
            asm = torch.as_tensor(asm).to(dev, torch.int64).contiguous()
            start = torch.as_tensor(start).to(dev, torch.int64).contiguous()
            rc = None
            if reverse_complement is not None:
                rc = torch.as_tensor(reverse_complement)
                rc = (rc.view(torch.uint8) if rc.dtype == torch.bool else rc).to(dev, torch.uint8).contiguous()
            x, status, tr = _C.windows_trace(self._devc, asm, start, int(W), rc, tokens, True, flags | self.launch_flags)
        return x, int(status.item()), _C.trace_summary(tr), tr

    def _draw(self, n, W, generator, reverse_complement, tokens, return_coords, status=None, rng=None):
        """The sample() sequence without the host check: (windows, coords or None, status tensor). The draws are the
        reference's (torch.randint over all valid starts, then torch.rand for the strand, on the generator's device):
        for a CUDA generator on the cohort's device, outside stream capture, made in the coordinate kernel exactly as
        those torch calls make them (pv_sample_draw_coords; the generator then advanced as they advance it), else by
        the torch calls; the arithmetic from the draws to the decode's coordinates is one kernel (pv_sample_coords). status: None (a
        fresh word, zeroed by that kernel) or an int32 device word the decode ORs into. rng (int64 [3] on the cohort's
        device: a generator's seed and offset, 0): the same draws made inside that kernel from rng, which it advances
        as the two torch calls advance the generator (pv_sample_draw_coords)."""
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
        dev = self.device
        mode, p = _strand_mode(reverse_complement)
        u = r = None
        gen = None
        if (rng is None and gdev.type == "cuda" and (gdev.index or 0) == (dev.index or 0) and not torch.cuda.is_current_stream_capturing()
                and _native_draws()):
            # outside stream capture the draws are made in the coordinate kernel, from the generator's seed and offset,
            # exactly as torch.randint / torch.rand would make them; the generator is then advanced as they would
            gen = generator if generator is not None else torch.cuda.default_generators[dev.index or 0]
        elif rng is None:
            u = torch.randint(0, total, (n,), generator=generator, device=gdev, dtype=torch.int64).to(dev)
            if mode == 2:
                r = torch.rand(n, generator=generator, device=gdev).to(dev)
        with torch.cuda.device(dev):
            asm = torch.empty(n, dtype=torch.int64, device=dev)
            start = torch.empty(n, dtype=torch.int64, device=dev)
            rc = torch.empty(n, dtype=torch.uint8, device=dev) if mode else None
            coords = torch.empty((n, 4), dtype=torch.int64, device=dev) if return_coords else None
            fresh = status is None
            if fresh:
                status = torch.empty(1, dtype=torch.int32, device=dev)
            if gen is not None:
                seed, off = gen.initial_seed(), gen.get_offset()
                _C.sample_draw_coords(cum, v, self._ctg, total, None, p, mode, n, asm, start, rc, coords, status if fresh else None,
                                      seed=seed, offset=off)
                gen.set_offset(off + self._draw_increment(n, total, mode))
            elif rng is None:
                _C.sample_coords(cum, v, self._ctg, u, r, p, mode, asm, start, rc, coords, status if fresh else None)
            else:
                _C.sample_draw_coords(cum, v, self._ctg, total, rng, p, mode, n, asm, start, rc, coords, status if fresh else None)
            x, status = self._launch(asm, start, W, rc, tokens, True, status=status)
        return x, coords, status

    def _draw_increment(self, n, total, mode):
        """the Philox offset torch's randint (and, mode 2, rand) for sample() consume on this device"""
        key = (n, total, mode)
        if key not in self._incs:
            pr = torch.cuda.get_device_properties(self.device)
            self._incs[key] = _C.torch_draw_geometry(n, total, mode, pr.multi_processor_count,
                                                     getattr(pr, "max_threads_per_multi_processor", 2048))[2]
        return self._incs[key]

    def sample(self, n, W, generator=None, reverse_complement=False, tokens=False, return_coords=False, check=True):
        """n windows of W bases, uniform over every (assembly, contig, start) with start + W <= contig length (a
        window never crosses contigs) -> uint8 [n, W] on the cohort's device. generator: a torch.Generator (its device
        draws the numbers). reverse_complement: False, True, or p in (0, 1) - each window reverse-complemented with
        probability p. return_coords: also an int64 [n, 4] tensor (assembly, contig index, start in the contig,
        reverse-complemented 0/1)."""
        x, coords, status = self._draw(int(n), int(W), generator, reverse_complement, tokens, return_coords)
        if check:
            with torch.cuda.device(self.device):
                s = _C.read_status(status)
            if s:
                raise RuntimeError(STATUS_TEXT.format(s))
        return (x, coords) if return_coords else x

    def sampler(self, n, W, generator, reverse_complement=False, tokens=False, return_coords=False):
        """sample(n, W, generator, reverse_complement, tokens, return_coords) captured once as a CUDA graph: calling
        the returned Sampler replays it - the generator's Philox draws, the coordinate arithmetic and the decode kernel
        in one graph launch - and gives the windows (and coordinates) the same successive sample() calls would give.
        The outputs are the graph's static tensors, overwritten by the next call on the stream: consume them in
        stream order, or clone. Each call checks nothing on the host; Sampler.status() reads the OR of the status
        words since the last read (one sync)."""
        return Sampler(self, int(n), int(W), generator, reverse_complement, tokens, return_coords)

    def fetch(self, assembly, contig, start, length, reverse_complement=False, tokens=False):
        """Bases [start, start + length) of a contig (0-based) -> uint8 [length] on the cohort's device."""
        a = self._asm(assembly)
        c = self._contig(a, contig)
        if a not in self._ctg_tables:
            self._ctg_tables[a] = self._core.contigs(a)
        name, _, clen, boff, _ = self._ctg_tables[a][c]
        start, length = int(start), int(length)
        if start < 0 or length < 0 or start + length > clen:
            raise IndexError(f"{self.names[a]} {name}:{start}+{length} outside the contig ({clen} bases)")
        if self._fetch_host is None:                       # one pinned (assembly, start) pair, one copy per call
            self._fetch_host = torch.empty(2, dtype=torch.int64).pin_memory()
            self._fetch_rc = torch.ones(1, dtype=torch.uint8, device=self.device)
        self._fetch_host[0], self._fetch_host[1] = a, boff + start
        with torch.cuda.device(self.device):
            d = self._fetch_host.to(self.device, non_blocking=True)
        # windows() waits for the stream before it returns, so the pinned pair is free again for the next call
        return self.windows(d[0:1], d[1:2], length, self._fetch_rc if reverse_complement else None, tokens)[0]

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

    def _decode_device(self, a, chunk, apply_case):
        """Assembly a's whole base stream decoded into one uint8 CUDA tensor on the cohort's device (chunked
        launches, one status word, one wait); raises on a failed block as windows(check=True) does."""
        n = self._info[a]["bases"]
        out = torch.empty(max(1, n), dtype=torch.uint8, device=self.device)[:n]
        asm = torch.tensor([a], dtype=torch.int64)
        with torch.cuda.device(self.device):
            status = torch.zeros(1, dtype=torch.int32, device=self.device)
            for s in range(0, n, chunk):
                k = min(chunk, n - s)
                self._launch(asm, torch.tensor([s], dtype=torch.int64), k, None, False, apply_case, out=out[s:s + k].view(1, k),
                             status=status)
            st = int(status.item())
        if st:
            raise RuntimeError(STATUS_TEXT.format(st))
        return out

    def decode(self, assembly, chunk=1 << 28, out=None):
        """The whole base stream of an assembly (contigs concatenated, case as in the FASTA) decoded on the cohort's
        device in chunks of `chunk` bases -> uint8 [bases] on the host (pinned; `out` reused if given)."""
        return self._decode(self._asm(assembly), int(chunk), out, True)

    def check_full(self, assembly, out=None):
        """Full decode on the cohort's device, the FASTA rebuilt from it (layout from the contig table) hashed with
        XXH3 -> (equal to the header's source XXH3, the hash "%016llx"). The stream stays on the device: the FASTA is
        read over it there and only XXH3's per-block sums come back (`out`, the reference's host buffer for the stream,
        is accepted and not needed)."""
        a = self._asm(assembly)
        h = self._core.fasta_xxh3_device(a, self._decode_device(a, 1 << 28, True))
        return h == self._info[a]["fasta_xxh3"], h

    def fasta(self, assembly, verify=True):
        """Full decode of an assembly -> the FASTA file's bytes. verify: every block XXH3 (if present) and the XXH3 of
        the rebuilt FASTA against the header's (the source file's). Decode, checks, case and FASTA layout run on the
        cohort's device; the FASTA's bytes are copied back once."""
        a = self._asm(assembly)
        path = self._info[a]["path"]
        try:
            b = self._decode_device(a, 1 << 28, False)
        except RuntimeError:
            raise _C.FormatError(path + ": block decode failed")
        if verify and self._core.first_bad_block_device(a, b) >= 0:
            raise _C.FormatError(path + ": block XXH3 mismatch")
        with torch.cuda.device(self.device):
            _C.apply_case_device(self._devc, a, self._info[a]["lower_case_runs"], b)
        if verify and self._core.fasta_xxh3_device(a, b) != self._info[a]["fasta_xxh3"]:
            raise _C.FormatError(path + ": FASTA XXH3 differs from the header")
        return self._core.fasta_device(a, b).cpu().numpy().tobytes()


class Sampler:
    """A captured sample() call (Cohort.sampler): call k returns what the k-th eager sample() call with the same
    generator would (windows, coordinates, status), and advances the generator as that call would. The graph makes the
    draws itself (pv_sample_draw_coords: torch's randint / rand kernels restated in the coordinate kernel, from a device
    copy of the generator's seed and offset that the graph advances), so a replay needs no generator bookkeeping on the
    device; if the generator is used or reseeded between calls, the next call reloads its state. With a torch release
    that restatement was not checked against (TORCH_DRAWS_CHECKED), the graph captures torch's own randint / rand
    instead, and torch advances the generator at each replay."""

    def __init__(self, cohort, n, W, generator, reverse_complement, tokens, return_coords):
        if generator is None or generator.device.type != "cuda":
            raise ValueError("sampler: a CUDA torch.Generator on the cohort's device")
        self.cohort, self.n, self.W, self.return_coords = cohort, n, W, return_coords
        self.generator = generator
        dev = cohort.device
        mode, _ = _strand_mode(reverse_complement)
        args = (n, W, generator, reverse_complement, tokens, return_coords)
        with torch.cuda.device(dev):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            state = generator.get_state()
            with torch.cuda.stream(side):
                cohort._draw(*args)                              # caches the per-W prefix sums, sizes the scratch
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            generator.set_state(state)                           # the warm-up draws are not part of the stream
            props = torch.cuda.get_device_properties(dev)
            _, _, self._inc = _C.torch_draw_geometry(n, cohort._valid[W][2], mode, props.multi_processor_count,
                                                     getattr(props, "max_threads_per_multi_processor", 2048))
            self.native = _native_draws()
            self._rng = torch.zeros(3, dtype=torch.int64, device=dev)
            self._seed = self._offset = None
            if self.native:
                self._load_rng()
            self.graph = torch.cuda.CUDAGraph()
            if not self.native:                          # torch's draws captured: the graph advances this generator
                self.graph.register_generator_state(generator)
            self._acc = torch.zeros(1, dtype=torch.int32, device=dev)
            events, cohort.kernel_events = cohort.kernel_events, None
            try:
                with torch.cuda.graph(self.graph):
                    self.x, self.coords, _ = cohort._draw(*args, status=self._acc, rng=self._rng if self.native else None)
            finally:
                cohort.kernel_events = events

    def _load_rng(self):
        """The generator's seed and offset into the graph's device copy, when they are not what it holds already."""
        seed, off = self.generator.initial_seed(), self.generator.get_offset()
        if (seed, off) != (self._seed, self._offset):
            w = torch.tensor([seed - (1 << 64) if seed >= 1 << 63 else seed, off, 0], dtype=torch.int64)
            self._rng.copy_(w)
            self._seed, self._offset = seed, off

    def __call__(self):
        with torch.cuda.device(self.cohort.device):
            if not self.native:                          # torch's draws in the graph: torch advances the generator
                self.graph.replay()
                return (self.x, self.coords) if self.return_coords else self.x
            self._load_rng()
            self.graph.replay()
        self._offset += self._inc
        self.generator.set_offset(self._offset)
        return (self.x, self.coords) if self.return_coords else self.x

    def status(self):
        """OR of the decode status words of the calls since the last status() (1 corrupt block, 4 wait expired,
        8 window outside an assembly); one device sync."""
        s = int(self._acc.item())
        self._acc.zero_()
        return s


def global_batch(x, coords=None, group=None):
    """One global batch from every rank's windows: all-gather along dim 0 in rank order (NCCL over NVLink / NVSwitch
    when the tensors are on GPUs; any torch.distributed backend works). The ranks are replicas that never exchange
    data otherwise - call this only when a single global batch is wanted. x: [n, ...] (the same n on every rank);
    coords: None or [n, 4]. Returns (X [world * n, ...], C or None)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)

    def gather(t):
        t = t.contiguous()
        out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t, group=group)
        return out
    return gather(x), (gather(coords) if coords is not None else None)
