"""GPU parity on larger cohorts: config 0 as the reference's encoder wrote it (the config's workload, sample(1024, 8192,
seed 0), byte-compared with the CPU decoder), and synthesizer cohorts at every block size with structural variants,
reverse-complemented contigs, N runs, IUPAC codes and soft-masking - thousands of windows against the oracle on both
kernel paths."""
import glob
import os

import numpy as np
import pytest
import torch
import xxhash

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
synth = pytest.importorskip("panvram_b200.synth")


@pytest.fixture(scope="module")
def cfg0(tmp_path_factory, cuda, oracle):
    import shutil
    import panvram_b200 as P
    d = tmp_path_factory.mktemp("cfg0")
    synth.make_cohort(str(d / "gen"), "cfg0")
    os.makedirs(d / "ref_enc")
    shutil.copyfile(d / "gen" / "reference.fa", d / "ref_enc" / "reference.fa")
    for p in glob.glob(os.path.join(GOLDEN, "cfg0", "*.q4k.rr3")):
        shutil.copyfile(p, d / "ref_enc" / os.path.basename(p))
    c = P.Cohort.open(str(d / "ref_enc"), device=cuda)
    ref = oracle.Reference(str(d / "ref_enc" / "reference.fa"))
    arcs = [oracle.Archive(p, ref) for p in sorted(glob.glob(str(d / "ref_enc" / "*.q4k.rr3")))]
    return c, ref, arcs


def test_cfg0_workload(cfg0, oracle, cuda):
    """config 0: sample(1024, 8192, seed 0) on the GPU == the CPU decoder at the same coordinates."""
    c, ref, arcs = cfg0
    g = torch.Generator(device=cuda).manual_seed(0)
    x, co = c.sample(1024, 8192, generator=g, return_coords=True)
    co = co.cpu().numpy()
    start = np.array([c.contigs(int(a))[int(ci)][3] + int(s) for a, ci, s, _ in co])
    assert np.array_equal(x.cpu().numpy(), oracle.windows(arcs, ref, co[:, 0], start, 8192, threads=8))


def test_cfg0_golden(cfg0):
    c, _, _ = cfg0
    gw = dict(np.load(os.path.join(GOLDEN, "cfg0", "windows.npz")))
    for tag, rc, tok in (("plain", None, False), ("rc_tokens", gw["rc"], True), ("rc", gw["rc"], False)):
        for flags in (0, 1):
            x, st = c._launch(torch.from_numpy(gw["asm"]), torch.from_numpy(gw["start"]), 8192,
                              torch.from_numpy(rc) if rc is not None else None, tok, True, flags=flags)
            assert int(st.item()) == 0
            got = np.array([xxhash.xxh3_64_intdigest(r.tobytes()) for r in x.cpu().numpy()], dtype=np.uint64)
            assert np.array_equal(got, gw["xxh3_" + tag]), (tag, flags)


@pytest.mark.parametrize("Q", [1024, 2048, 4096, 16384])
def test_synth_cohort_parity(tmp_path_factory, oracle, cuda, Q):
    import panvram_b200 as P
    d = str(tmp_path_factory.mktemp(f"syn{Q}"))
    synth.make_cohort(d, "cfg1", Q=Q, nasm=4, scale=0.004)
    c = P.Cohort.open(d, device=cuda, dataset=synth.dataset_of(Q))
    ref = oracle.Reference(os.path.join(d, "reference.fa"))
    arcs = [oracle.Archive(p, ref) for p in sorted(glob.glob(os.path.join(d, f"*.{synth.dataset_of(Q)}.rr3")))]
    g = torch.Generator(device=cuda).manual_seed(Q)
    for W in (1, 77, 1000, 8192, 40000):
        for rcp, tok in ((False, False), (0.5, False), (0.5, True)):
            x, co = c.sample(512, W, generator=g, reverse_complement=rcp, tokens=tok, return_coords=True)
            co = co.cpu().numpy()
            start = np.array([c.contigs(int(a))[int(ci)][3] + int(s) for a, ci, s, _ in co])
            want = oracle.windows(arcs, ref, co[:, 0], start, W, rc=co[:, 3], tokens=tok, threads=8)
            assert np.array_equal(x.cpu().numpy(), want), (Q, W, rcp, tok)
            xb, st = c._launch(torch.from_numpy(co[:, 0]), torch.from_numpy(start), W, torch.from_numpy(co[:, 3]), tok, True, flags=1)
            assert int(st.item()) == 0 and np.array_equal(xb.cpu().numpy(), want), ("block path", Q, W)
    for a in range(len(c)):
        ok, _ = c.check_full(a)
        assert ok
