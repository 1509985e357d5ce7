"""The oracle (oracle/pv_oracle.c) pinned against the reference: every golden window (the reference's compiled CPU
decoder's output, hashed), every fixture archive's full decode (== the header's source-FASTA XXH3), the refusal text of
host-made corruptions, and - where the reference checkout is present - the reference's own decoder on fresh windows."""
import os

import numpy as np
import pytest
import xxhash

from conftest import DATASETS, NAMES, golden_cases


def test_oracle_golden_windows(golden, oracle_cohorts, oracle):
    win = golden["windows"]
    n = 0
    for (di, W, tok, case), rows in golden_cases(win).items():
        ref, arcs = oracle_cohorts[DATASETS[di]]
        rows = np.array(rows)
        x = oracle.windows(arcs, ref, win["asm"][rows], win["start"][rows], W, rc=win["rc"][rows], tokens=tok, apply_case=case, threads=4)
        got = np.array([xxhash.xxh3_64_intdigest(r.tobytes()) for r in x], dtype=np.uint64)
        assert np.array_equal(got, win["xxh3"][rows]), (DATASETS[di], W, tok, case)
        n += len(rows)
    assert n == len(win["W"])


@pytest.mark.parametrize("ds", DATASETS)
def test_oracle_full_decode_matches_header(golden, oracle_cohorts, ds):
    ref, arcs = oracle_cohorts[ds]
    for nm, a in zip(NAMES, arcs):
        g = golden["info"]["archives"][f"{nm}.{ds}"]
        fa = a.fasta(verify=True)
        assert "%016x" % xxhash.xxh3_64_intdigest(fa) == g["fasta_xxh3"] == g["fasta_decoded_xxh3"]
        assert a.nbases == g["bases"] and a.nblocks == g["blocks"] and a.payload_bytes == g["payload_bytes"]
        assert [list(c) for c in a.contigs()] == g["contigs"]


def test_oracle_refusals(golden, oracle, tmp_path):
    from tests.golden.make_golden import mutations
    raw = open(os.path.join(golden["dirs"]["q4k"], "synthA.q4k.rr3"), "rb").read()
    ref = oracle.Reference(golden["ref"])
    for k, b in mutations(raw).items():
        p = tmp_path / f"{k}.rr3"
        p.write_bytes(b)
        with pytest.raises(oracle.OracleError) as e:
            oracle.Archive(str(p), ref)
        assert str(e.value).replace(str(p), "<path>") == golden["info"]["refusals"][k]


def test_oracle_vs_reference_decoder(golden, oracle_cohorts, oracle):
    """Fresh windows against the reference's compiled decoder (needs oracle/_ref, built where the reference is)."""
    R = oracle.reference_extension()
    if R is None:
        pytest.skip("oracle/_ref not built (python oracle/build_ref.py where the reference checkout is)")
    import torch
    rng = np.random.default_rng(99)
    for ds in DATASETS:
        ref, arcs = oracle_cohorts[ds]
        core = R.Core(golden["ref"], [a.path for a in arcs], 2, False, False)
        for W in (1, 300, 4097, 20000):
            n = 200
            asm = rng.integers(0, 2, n)
            start = np.array([rng.integers(0, arcs[a].nbases - W + 1) for a in asm])
            rc = rng.random(n) < 0.5
            for tok in (False, True):
                x = oracle.windows(arcs, ref, asm, start, W, rc=rc, tokens=tok, threads=4)
                y = core.windows(torch.tensor(asm), torch.tensor(start), W, torch.tensor(rc), tok, True, False, 2).numpy()
                assert np.array_equal(x, y), (ds, W, tok)
