"""The opt-in compact resident forms on the host (no GPU): the packed reference unpacks to the byte reference, and the
compact block table walks (the reference's CompactTab::get chain, pv_compact.h:37-48, restated here) to the same
payload offsets, lengths and start states as the full block table."""
import os

import numpy as np
import pytest

from conftest import DATASETS, NAMES


def _core(golden, ds, **kw):
    from panvram_b200 import _C
    return _C.Core(golden["ref"], [os.path.join(golden["dirs"][ds], f"{nm}.{ds}.rr3") for nm in NAMES], 2, **kw)


def _unpack(pools, n):
    """The byte reference from the packed form: 2-bit words, then the runs of other bytes written over."""
    w = pools["pref"]
    q = np.arange(n, dtype=np.int64)
    codes = (w[q >> 4] >> ((q & 15) * 2).astype(np.uint32)) & 3
    out = np.frombuffer(b"ACGT", np.uint8)[codes]
    runs = pools["pruns"].view(np.dtype([("start", "<u8"), ("len", "<u4"), ("byte", "<u4")]))
    assert len(runs) == pools["pnruns"] + 1 and runs[-1]["start"] == np.iinfo(np.uint64).max     # sentinel
    for r in runs[:-1]:
        out[int(r["start"]):int(r["start"]) + int(r["len"])] = r["byte"]
    return out, runs[:-1]


def test_packed_reference_unpacks_to_the_bytes(golden):
    plain = _core(golden, "q4k")
    ref = plain.pools()["ref_padded"][64:64 + plain.ref_bases]
    packed = _core(golden, "q4k", packed_reference=True)
    p = packed.pools()
    assert p["ref_padded"].size == 0 and packed.packed_reference
    got, runs = _unpack(p, packed.ref_bases)
    assert np.array_equal(got, ref)
    # runs: sorted, disjoint, maximal (a run never touches another run of its byte), never A/C/G/T
    s, e = runs["start"].astype(np.int64), runs["start"].astype(np.int64) + runs["len"].astype(np.int64)
    assert (s[1:] >= e[:-1]).all() and not np.isin(runs["byte"], list(b"ACGT")).any()
    assert not ((s[1:] == e[:-1]) & (runs["byte"][1:] == runs["byte"][:-1])).any()
    # the bucket index: the first run ending after each bucket's first position
    idx = p["pidx"]
    for k in range(len(idx)):
        x = k << 12
        want = int(np.searchsorted(e, x, side="right"))
        assert idx[k] == want, k


@pytest.fixture(scope="module")
def synth_cohort(tmp_path_factory):
    """config 0 generated (4 assemblies with SVs, inversions, reverse-complemented contigs): chain breaks to test"""
    import glob
    from panvram_b200 import synth
    d = str(tmp_path_factory.mktemp("cfg0") / "c")
    synth.make_cohort(d, "cfg0")
    return os.path.join(d, "reference.fa"), sorted(glob.glob(os.path.join(d, "*.q4k.rr3")))


@pytest.mark.parametrize("ds", DATASETS + ("synthetic",))
def test_compact_block_table_matches_the_full_one(golden, synth_cohort, ds):
    from panvram_b200 import _C
    if ds == "synthetic":
        full_core = _C.Core(*synth_cohort, 2)
        comp_core = _C.Core(*synth_cohort, 2, compact_blocks=True)
    else:
        full_core = _core(golden, ds)              # pools() are views of the core's memory: keep it alive
        comp_core = _core(golden, ds, compact_blocks=True)
    full = full_core.pools()
    c = comp_core.pools()
    assert c["blocks"].size == 0 and comp_core.compact_blocks
    Q = comp_core.Q
    loc, st = full["blocks"][0::2], full["blocks"][1::2].view(np.int64)
    want_off, want_len = (loc & np.uint64((1 << 40) - 1)).astype(np.int64), (loc >> np.uint64(40)).astype(np.int64)
    g = c["groups"].view(_C.BLK_GROUP)
    btab, bexc = c["btab"], c["bexc"]
    asms = c["asms"].view(np.uint64).reshape(-1, 8)
    for a in range(len(asms)):
        blk_base, nb, grp_base = int(asms[a, 1]), int(asms[a, 2]), int(asms[a, 7])
        for b in range(nb):
            G = g[grp_base + b // 32]
            j = b % 32
            off, s = int(G["off"]), int(G["state"])
            for k in range(1, j + 1):                    # the chain of pv_compact.h:40-46
                v = int(btab[blk_base + b - j + k - 1])
                off += v & 0xFFFF
                code = np.int16(np.uint16(int(btab[blk_base + b - j + k]) >> 16))
                if code == _C.PV_CODE_EXC:
                    s = int(bexc[int(G["exc_base"]) + bin(int(G["exc_mask"]) & ((1 << k) - 1)).count("1")])
                else:
                    pc, pd = s >> 1, s & 1
                    pred = pc - Q if pd else pc + Q
                    s = ((pred + (int(code) >> 1)) << 1) | (int(code) & 1)
            gb = blk_base + b
            assert off == want_off[gb] and (int(btab[gb]) & 0xFFFF) == want_len[gb] and s == int(st[gb]), (a, b)
    if ds == "synthetic":
        assert sum(bin(int(m)).count("1") for m in g["exc_mask"]) > 0      # the chain breaks somewhere


def test_resident_forms_refuse_nothing_else(golden):
    """Both forms together open; info, contigs and the FASTA hashes are those of the plain form."""
    plain = _core(golden, "q16k")
    both = _core(golden, "q16k", packed_reference=True, compact_blocks=True)
    for i in range(plain.n):
        assert plain.info(i) == both.info(i)
        assert plain.contigs(i) == both.contigs(i)
