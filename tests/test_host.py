"""The host side of panvram_b200 (C++ reader and pooling, no GPU): every check and refusal text as the reference, the
contig table and header fields, the device layout it pools (decode tables, block table) checked against the oracle's
own parse, and the FASTA rebuild / hashes."""
import os
import shutil

import numpy as np
import pytest
import torch
import xxhash

from conftest import DATASETS, NAMES

P = pytest.importorskip("panvram_b200")
from panvram_b200 import _C  # noqa: E402
from panvram_b200.layout import ALPHA, big_index, TAB_BIDX, TAB_BUCKET, TAB_CUM8, TAB_DENSE, TAB_DOFF  # noqa: E402


def paths(golden, ds):
    return [os.path.join(golden["dirs"][ds], f"{nm}.{ds}.rr3") for nm in NAMES]


@pytest.mark.parametrize("ds", DATASETS)
def test_info_and_contigs(golden, ds):
    c = _C.Core(golden["ref"], paths(golden, ds), 2)
    assert c.n == 2 and c.Q == {"q1k": 1024, "q4k": 4096, "q16k": 16384}[ds]
    assert c.ref_sha256 == golden["info"]["reference_sha256"] == _C.sha256_file_bases(golden["ref"])
    for i, nm in enumerate(NAMES):
        g, mine = golden["info"]["archives"][f"{nm}.{ds}"], c.info(i)
        for k in ("Q", "bases", "blocks", "file_bytes", "payload_bytes", "block_hashes", "fasta_xxh3", "contigs",
                  "lower_case_runs", "reference_name"):
            want = len(g["contigs"]) if k == "contigs" else g[k]
            assert mine[k] == want, k
        assert [list(x) for x in c.contigs(i)] == g["contigs"]


def test_refusals(golden, tmp_path):
    from tests.golden.make_golden import mutations
    good = paths(golden, "q4k")[0]
    raw = open(good, "rb").read()
    for k, b in mutations(raw).items():
        p = tmp_path / f"{k}.rr3"
        p.write_bytes(b)
        with pytest.raises(_C.FormatError, match="refused") as e:
            _C.Core(golden["ref"], [str(p)], 1)
        assert str(e.value).replace(str(p), "<path>") == golden["info"]["refusals"][k]
    # wrong reference: one base changed (the reference's test_refusals)
    ref = bytearray(open(golden["ref"], "rb").read())
    i = ref.index(b"\n") + 5
    ref[i] ^= 0x01 if ref[i] != ord("A") else 0x02
    (tmp_path / "bad_ref.fa").write_bytes(bytes(ref))
    with pytest.raises(_C.FormatError, match="wrong reference"):
        _C.Core(str(tmp_path / "bad_ref.fa"), [good], 1)
    # one block size per cohort
    with pytest.raises(_C.FormatError, match="block size 1024 differs from 4096"):
        _C.Core(golden["ref"], [good, paths(golden, "q1k")[1]], 1)
    with pytest.raises(_C.FormatError, match="no archives"):
        _C.Core(golden["ref"], [], 1)
    with pytest.raises(_C.FormatError, match="cannot open"):
        _C.Core(golden["ref"], [str(tmp_path / "missing.rr3")], 1)
    with pytest.raises(_C.FormatError, match="not FASTA"):
        _C.Core(good, [good], 1)


def test_more_refusals_match_oracle(golden, oracle, tmp_path):
    """Truncations and byte flips over the header and meta: the same refusal (or acceptance) as the oracle."""
    raw = open(paths(golden, "q16k")[0], "rb").read()
    ref = oracle.Reference(golden["ref"])
    rng = np.random.default_rng(5)
    cases = [raw[:k] for k in (0, 10, 137, 138, 200, len(raw) - 100)]
    for _ in range(60):
        b = bytearray(raw)
        p = int(rng.integers(0, min(len(raw), 600)))
        b[p] ^= 1 << int(rng.integers(0, 8))
        cases.append(bytes(b))
    for k, b in enumerate(cases):
        p = tmp_path / f"m{k}.rr3"
        p.write_bytes(b)
        try:
            oracle.Archive(str(p), ref)
            want = None
        except oracle.OracleError as e:
            want = str(e)
        try:
            _C.Core(golden["ref"], [str(p)], 1)
            got = None
        except _C.FormatError as e:
            got = str(e)
        assert got == want, k


def lookup_all_slots(tab, c):
    """The device's decode-table lookup (pv_kernels.cu dsym) over every slot of context c -> (sym, freq, cum)."""
    slot = np.arange(4096, dtype=np.int64)
    bi = big_index(c)
    if bi < 0:
        cum8 = np.frombuffer(tab[TAB_CUM8 + 16 * c: TAB_CUM8 + 16 * c + 16].tobytes(), dtype=np.uint16).astype(np.int64)
        s = sum((cum8[k] <= slot).astype(np.int64) for k in range(1, 6))
        cm = cum8[s]
        f = cum8[s + 1] - cm
        return s, f, cm
    nb = 4096 // TAB_BUCKET
    bidx = tab[TAB_BIDX + nb * bi: TAB_BIDX + nb * bi + nb].astype(np.int64)
    doff = np.frombuffer(tab[TAB_DOFF:TAB_DOFF + 32].tobytes(), dtype=np.uint16).astype(np.int64)
    dense = np.frombuffer(tab[TAB_DENSE:].tobytes()[: 4 * int(doff[15])], dtype=np.uint32).astype(np.int64)
    u = doff[bi] + bidx[slot // TAB_BUCKET]
    for _ in range(TAB_BUCKET + 2):
        e = dense[u]
        fr, cu = (e >> 12) & 8191, e & 4095
        step = (fr > 0) & (slot >= cu + fr)
        u = u + step
    e = dense[u]
    return e >> 25, (e >> 12) & 8191, e & 4095


@pytest.mark.parametrize("ds", DATASETS)
def test_decode_tables(golden, oracle_cohorts, ds):
    """Every slot of every context: the compact table gives the reference table's symbol, frequency and start."""
    c = _C.Core(golden["ref"], paths(golden, ds), 2)
    tabs = c.pools()["tabs"]
    _, arcs = oracle_cohorts[ds]
    for i, a in enumerate(arcs):
        rec = c.pools()["asms"].view(np.uint64).reshape(-1, 8)[i]
        tab = tabs[int(rec[5]):int(rec[5]) + int(rec[6])]
        assert int(rec[6]) % 16 == 0 and int(rec[5]) % 16 == 0 and int(rec[6]) <= c.pools()["tab_max"] <= _C.PV_TAB_MAX_BYTES
        freq = a.freq()
        for ctx in range(61):
            A = ALPHA[ctx]
            f = freq[ctx, :A].astype(np.int64)
            cum = np.concatenate([[0], np.cumsum(f)])
            s, fr, cm = lookup_all_slots(tab, ctx)
            if cum[-1] == 0:
                assert (fr == 0).all(), ctx                 # an all-zero context decodes as an error
                continue
            want = np.repeat(np.arange(A), f)
            assert np.array_equal(s, want), ctx
            assert np.array_equal(fr, f[want]) and np.array_equal(cm, cum[want]), ctx


@pytest.mark.parametrize("ds", DATASETS)
def test_block_table(golden, oracle_cohorts, ds):
    c = _C.Core(golden["ref"], paths(golden, ds), 2)
    p = c.pools()
    blocks, asms = p["blocks"], p["asms"].view(np.uint64).reshape(-1, 8)
    _, arcs = oracle_cohorts[ds]
    for i, a in enumerate(arcs):
        base, nb = int(asms[i, 1]), int(asms[i, 2])
        assert nb == a.nblocks and int(asms[i, 0]) == a.nbases
        pb = int(blocks[2 * base]) & ((1 << 40) - 1)
        lens = [a.block_payload(b) for b in range(nb)]
        offs = np.concatenate([[0], np.cumsum(lens)])
        for b in range(nb):
            loc, st = int(blocks[2 * (base + b)]), int(blocks[2 * (base + b) + 1])
            assert (loc >> 40) == lens[b] and (loc & ((1 << 40) - 1)) - pb == offs[b]
            cc, dd = a.block_state(b)
            st_signed = st - (1 << 64) if st >= 1 << 63 else st
            assert (st_signed >> 1) & ((1 << 64) - 1) == cc and (st & 1) == dd


@pytest.mark.parametrize("ds", DATASETS)
def test_fasta_rebuild_and_hashes(golden, oracle_cohorts, ds):
    c = _C.Core(golden["ref"], paths(golden, ds), 2)
    _, arcs = oracle_cohorts[ds]
    for i, a in enumerate(arcs):
        n = a.nbases
        upper = a.window(0, n, apply_case=False)
        assert c.first_bad_block(i, torch.from_numpy(upper.copy())) == -1
        cased = c.apply_case(i, torch.from_numpy(upper.copy()))
        assert np.array_equal(cased.numpy(), a.window(0, n))
        fa = c.fasta_bytes(i, cased)
        assert fa == a.fasta(verify=True)
        assert c.fasta_xxh3(i, cased) == c.info(i)["fasta_xxh3"] == "%016x" % xxhash.xxh3_64_intdigest(fa)
        bad = upper.copy()
        bad[min(n - 1, 3 * c.Q + 7)] ^= 0x04
        assert c.first_bad_block(i, torch.from_numpy(bad)) == min(n - 1, 3 * c.Q + 7) // c.Q


def test_pools_padding(golden):
    c = _C.Core(golden["ref"], paths(golden, "q4k"), 2)
    p = c.pools()
    assert len(p["ref_padded"]) == c.ref_bases + 128
    assert not p["ref_padded"][:64].any() and not p["ref_padded"][-64:].any()
    assert not p["payload"][-64:].any()
    asms = p["asms"].view(np.uint64).reshape(-1, 8)
    # the tables back to back, then 16 zero bytes (a dense-list lookup may read one entry ahead)
    assert len(p["tabs"]) == int(asms[:, 6].sum()) + 16 and p["tab_max"] == int(asms[:, 6].max())
    assert not p["tabs"][-16:].any()


def test_release_uploaded_keeps_the_rest(golden):
    """After the cohort is on the device, the host copies of the reference and the payload are freed; the block table,
    runs, tables, contigs and every archive's metadata stay, and the core still answers contigs / info."""
    c = _C.Core(golden["ref"], paths(golden, "q4k"), 2)
    before = c.pools()
    kept = {k: before[k].copy() for k in ("blocks", "asms", "tabs", "low", "ctg_len")}
    info0, ctg0 = c.info(0), c.contigs(0)
    c.release_uploaded()
    after = c.pools()
    assert after["payload"].size == 0 and after["ref_padded"].size == 0
    for k, v in kept.items():
        assert np.array_equal(after[k], v), k
    assert c.info(0) == info0 and c.contigs(0) == ctg0 and c.ref_bases > 0


def test_cohort_is_gpu_only(golden):
    with pytest.raises(RuntimeError, match="GPU only"):
        P.Cohort.open(golden["dirs"]["q4k"], device="cpu", reference=golden["ref"])
    with pytest.raises(ValueError):
        P.Cohort.open(golden["dirs"]["q4k"], device="cpu", dataset="bad")
    with pytest.raises(FileNotFoundError):
        P.Cohort.open(golden["dirs"]["q4k"], device="cpu", dataset="q1k")
    d = os.path.join(golden["root"], "copy")
    shutil.copytree(golden["dirs"]["q4k"], d, dirs_exist_ok=True)
    with pytest.raises(FileNotFoundError, match="not in"):
        P.Cohort.open(d, device="cuda", reference=golden["ref"], assemblies=["nope"])


def test_xxh3_restatement_equals_the_library():
    """The XXH3 steps the device path splits (block sums from zero accumulators, the scramble chain, the partial block,
    the last stripe, the merge; panvram_b200/csrc/pv_xxh3.h), run on the host, against the xxHash library at every
    length class of the long-input path: block edges, stripe edges, one and many blocks."""
    rng = np.random.default_rng(3)
    lens = list(range(241, 1300)) + [2047, 2048, 2049, 3 * 1024, 3 * 1024 + 1, 16384, 16385, 1 << 20, (1 << 20) + 63]
    for n in lens:
        d = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert _C.xxh3_64_long_host(d) == xxhash.xxh3_64_intdigest(d), n
    with pytest.raises(ValueError):
        _C.xxh3_64_long_host(b"x" * 240)
