"""The whole-assembly checks on the device (check_full / fasta, panvram/cohort.py:224-234): the FASTA read over a
decoded stream on the GPU, its XXH3 (block sums on the device, scramble chain on the host), per-block XXH3 and
lower-case runs, each against the host implementation of the same step on the same bytes (pv_core.cpp:138-176 as
restated in pv_host.cpp) and the oracle. Edited streams (bytes changed anywhere, the last block included) check that
the hashes follow the bytes, not the archive. Integer work: exact."""
import os

import numpy as np
import pytest
import torch
import xxhash

from conftest import DATASETS

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cohorts(golden, cuda):
    import panvram_b200 as P
    return {ds: P.Cohort.open(golden["dirs"][ds], device=cuda, dataset=ds, reference=golden["ref"]) for ds in DATASETS}


@pytest.fixture(scope="module")
def synth_cohort(tmp_path_factory, cuda):
    import panvram_b200 as P
    from panvram_b200 import synth
    d = str(tmp_path_factory.mktemp("cfg0") / "c")
    synth.make_cohort(d, "cfg0")
    return P.Cohort.open(d, device=cuda, dataset="q4k", reference=os.path.join(d, "reference.fa"))


def _streams(c, a):
    upper = c._decode_device(a, 1 << 28, False)
    cased = c._decode_device(a, 1 << 28, True)
    return upper, cased


@pytest.mark.parametrize("ds", DATASETS)
def test_device_fasta_and_hashes_equal_the_host_steps(cohorts, oracle_cohorts, ds):
    c = cohorts[ds]
    core = c._core
    _, arcs = oracle_cohorts[ds]
    for a in range(len(c)):
        upper, cased = _streams(c, a)
        # lower-case runs on the device = the decode with case applied = the oracle
        u2 = upper.clone()
        from panvram_b200 import _C
        _C.apply_case_device(c._devc, a, c.info(a)["lower_case_runs"], u2)
        assert torch.equal(u2, cased)
        host = cased.cpu()
        assert np.array_equal(host.numpy(), arcs[a].window(0, arcs[a].nbases))
        # the FASTA: device bytes = host rebuild = the oracle's
        fa = core.fasta_device(a, cased).cpu().numpy().tobytes()
        assert fa == core.fasta_bytes(a, host) == arcs[a].fasta(verify=True)
        # its XXH3: device path (several chunk sizes, so the host chain crosses chunk ends) = host = xxhash = header
        want = "%016x" % xxhash.xxh3_64_intdigest(fa)
        assert want == c.info(a)["fasta_xxh3"] == core.fasta_xxh3(a, host)
        for chunk in (0, 1, 3, 64):
            assert core.fasta_xxh3_device(a, cased, chunk_blocks=chunk) == want, chunk
        # block hashes: none bad on the archive's own stream
        assert core.first_bad_block_device(a, upper) == -1 == core.first_bad_block(a, upper.cpu())


@pytest.mark.parametrize("ds", DATASETS)
def test_hashes_follow_edited_bytes(cohorts, ds):
    """A byte changed in block k: the device's first bad block is k, as the host's; the FASTA hash changes and equals the
    host's hash of the same edited stream (edits at the start, in the middle, in the last block and at the last byte)."""
    c = cohorts[ds]
    core = c._core
    rng = np.random.default_rng(11)
    for a in range(len(c)):
        upper, cased = _streams(c, a)
        n, Q = upper.numel(), c.block_size
        for p in sorted({0, int(rng.integers(0, n)), n // 2, (n - 1) // Q * Q, n - 1}):
            bad = upper.clone()
            bad[p] ^= 0x04
            assert core.first_bad_block_device(a, bad) == p // Q == core.first_bad_block(a, bad.cpu()), p
            ed = cased.clone()
            ed[p] ^= 0x04
            h = core.fasta_xxh3_device(a, ed, chunk_blocks=2)
            assert h == core.fasta_xxh3(a, ed.cpu()) != c.info(a)["fasta_xxh3"], p


def test_synthetic_cohort_checks(synth_cohort):
    """config 0 generated (contigs of Mbp, thousands of lower-case runs, reverse-complemented contigs): check_full and
    fasta."""
    c = synth_cohort
    for a in range(len(c)):
        ok, h = c.check_full(a)
        assert ok and h == c.info(a)["fasta_xxh3"]
        fa = c.fasta(a)
        assert "%016x" % xxhash.xxh3_64_intdigest(fa) == h
        _, cased = _streams(c, a)
        assert c._core.fasta_xxh3_device(a, cased, chunk_blocks=5) == h


def test_device_checks_refuse_wrong_streams(cohorts, cuda):
    from panvram_b200 import _C
    c = cohorts["q4k"]
    n = c.info(0)["bases"]
    with pytest.raises(_C.FormatError):
        c._core.fasta_xxh3_device(0, torch.zeros(n - 1, dtype=torch.uint8, device=cuda))
    with pytest.raises(_C.FormatError):
        c._core.first_bad_block_device(0, torch.zeros(n, dtype=torch.uint8))          # a CPU tensor
