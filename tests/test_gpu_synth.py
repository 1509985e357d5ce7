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
        for flags in (2, 3, 4, 5):                            # fused / split, each also on the block path
            x, st = c._launch(torch.from_numpy(gw["asm"]), torch.from_numpy(gw["start"]), 8192,
                              torch.from_numpy(rc) if rc is not None else None, tok, True, flags=flags)
            assert int(st.item()) == 0
            got = np.array([xxhash.xxh3_64_intdigest(r.tobytes()) for r in x.cpu().numpy()], dtype=np.uint64)
            assert np.array_equal(got, gw["xxh3_" + tag]), (tag, flags)


@pytest.mark.parametrize("Q", [1024, 16384])
def test_block_cache_same_output(tmp_path_factory, oracle, cuda, Q):
    """Blocks served from the open-time cache give the oracle's bytes, in every window that touches them."""
    import panvram_b200 as P
    d = str(tmp_path_factory.mktemp(f"cache{Q}"))
    synth.make_cohort(d, "cfg1", Q=Q, nasm=3, scale=0.004)
    ds = synth.dataset_of(Q)
    c = P.Cohort.open(d, device=cuda, dataset=ds)
    c0 = P.Cohort.open(d, device=cuda, dataset=ds, block_cache=False)
    assert c.cached_blocks > 0 and c0.cached_blocks == 0 and c.resident_bytes()["cache"] > 0
    ref = oracle.Reference(os.path.join(d, "reference.fa"))
    arcs = [oracle.Archive(p, ref) for p in sorted(glob.glob(os.path.join(d, f"*.{ds}.rr3")))]
    blocks = c._dev["blocks"].cpu().numpy().view(np.uint64)[0::2]
    cached = np.nonzero((blocks >> np.uint64(40)) == np.uint64(0xFFFFFE))[0]
    asms = c._core.pools()["asms"].view(np.uint64).reshape(-1, 8)
    base = asms[:, 1].astype(np.int64)
    rng = np.random.default_rng(Q)
    for W in (1, 300, Q, 3 * Q + 5):
        asm, start = [], []
        for g in rng.choice(cached, min(200, len(cached))):
            a = int(np.searchsorted(base, g, side="right") - 1)
            s = int((g - base[a]) * Q) + int(rng.integers(-W + 1, Q))
            s = max(0, min(s, arcs[a].nbases - W))
            asm.append(a)
            start.append(s)
        rcm = rng.random(len(asm)) < 0.5
        for tok in (False, True):
            want = oracle.windows(arcs, ref, np.array(asm), np.array(start), W, rc=rcm, tokens=tok, threads=8)
            for co in (c, c0):
                x, st = co._launch(torch.tensor(asm), torch.tensor(start), W, torch.from_numpy(rcm), tok, True)
                assert int(st.item()) == 0 and np.array_equal(x.cpu().numpy(), want), (Q, W, tok, co.cached_blocks)


@pytest.mark.parametrize("Q,stride", [(4096, None), (16384, 512)])
def test_costly_blocks_cached(tmp_path_factory, oracle, cuda, monkeypatch, Q, stride):
    """The block cache also takes the blocks whose costliest stride cell decodes longest (the index build's costs):
    with a large fraction asked, blocks beyond the long-stream rule are cached, every checkpoint of a cached block
    points at its cache row, and windows over them - both kernel forms - give the oracle's bytes."""
    import panvram_b200 as P
    from panvram_b200 import _C
    d = str(tmp_path_factory.mktemp(f"costly{Q}"))
    synth.make_cohort(d, "cfg1", Q=Q, nasm=3, scale=0.004)
    ds = synth.dataset_of(Q)
    monkeypatch.setattr(P.Cohort, "CACHE_COSTLY", 0.0)
    c0 = P.Cohort.open(d, device=cuda, dataset=ds, checkpoint_stride=stride)
    monkeypatch.setattr(P.Cohort, "CACHE_COSTLY", 0.3)
    c = P.Cohort.open(d, device=cuda, dataset=ds, checkpoint_stride=stride)
    assert c.cached_blocks > c0.cached_blocks > 0
    blocks = c._dev["blocks"].cpu().numpy().view(np.uint64)
    cached = np.nonzero((blocks[0::2] >> np.uint64(40)) == np.uint64(0xFFFFFE))[0]
    assert len(cached) == c.cached_blocks
    ncell = Q // c.checkpoint_stride
    rec = c._ckpt.view(torch.int32).view(-1, 8).cpu().numpy()
    slots = (blocks[0::2][cached] & np.uint64((1 << 40) - 1)).astype(np.int64)
    for b, slot in zip(cached, slots):
        r = rec[b * ncell:(b + 1) * ncell]
        assert ((r[:, 7] >> 16) & _C.PV_CKPT_CACHED).all() and (r[:, 1] == slot).all()
    ref = oracle.Reference(os.path.join(d, "reference.fa"))
    arcs = [oracle.Archive(p, ref) for p in sorted(glob.glob(os.path.join(d, f"*.{ds}.rr3")))]
    asms = c._core.pools()["asms"].view(np.uint64).reshape(-1, 8)
    base = asms[:, 1].astype(np.int64)
    rng = np.random.default_rng(Q + 1)
    for W in (300, 2 * Q + 7):
        asm, start = [], []
        for g in rng.choice(cached, min(300, len(cached))):
            a = int(np.searchsorted(base, g, side="right") - 1)
            s = int((g - base[a]) * Q) + int(rng.integers(-W + 1, Q))
            asm.append(a)
            start.append(max(0, min(s, arcs[a].nbases - W)))
        rcm = rng.random(len(asm)) < 0.5
        want = oracle.windows(arcs, ref, np.array(asm), np.array(start), W, rc=rcm, threads=8)
        for flags in (_C.PV_WIN_FUSED, _C.PV_WIN_SPLIT):
            x, st = c._launch(torch.tensor(asm), torch.tensor(start), W, torch.from_numpy(rcm), False, True, flags=flags)
            assert int(st.item()) == 0 and np.array_equal(x.cpu().numpy(), want), (Q, W, flags)


@pytest.mark.parametrize("Q,stride", [(1024, None), (2048, None), (4096, None), (16384, None), (4096, 256), (16384, 512), (4096, 0),
                                      (16384, 0)])
def test_synth_cohort_parity(tmp_path_factory, oracle, cuda, Q, stride):
    """Synthesizer cohorts against the oracle with the default checkpoint index, the smallest strides (long copies of
    the structural variants span many cells, so many items own no event and one item a long one) and no index."""
    import panvram_b200 as P
    d = str(tmp_path_factory.mktemp(f"syn{Q}"))
    synth.make_cohort(d, "cfg1", Q=Q, nasm=4, scale=0.004)
    c = P.Cohort.open(d, device=cuda, dataset=synth.dataset_of(Q), checkpoint_stride=stride)
    assert c.checkpoint_stride == (min(2048, Q) if stride is None else stride) and c.bad_blocks == 0
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
            for flags, tag in ((3, "fused block path"), (2, "fused"), (4, "split"), (5, "split block path")):
                xb, st = c._launch(torch.from_numpy(co[:, 0]), torch.from_numpy(start), W, torch.from_numpy(co[:, 3]), tok, True, flags=flags)
                assert int(st.item()) == 0 and np.array_equal(xb.cpu().numpy(), want), (tag, Q, W)
    for a in range(len(c)):
        ok, _ = c.check_full(a)
        assert ok


@pytest.mark.parametrize("native", [True, False], ids=["kernel-draws", "torch-draws"])
def test_sampler_graph_equals_sample(cfg0, cuda, native, monkeypatch):
    """Cohort.sampler (sample() captured as one CUDA graph, its draws made in the coordinate kernel) gives, call after
    call, exactly what eager sample() gives with an identically seeded generator - windows, coordinates and status -
    and leaves the generator where eager calls leave it, also across a reseed between calls. With a torch release the
    in-kernel draws were not checked against, both take torch's own randint / rand (the graph captures them)."""
    from panvram_b200 import cohort as cohort_mod
    if not native:
        monkeypatch.setattr(cohort_mod, "TORCH_DRAWS_CHECKED", ())
    c, _, _ = cfg0
    for rcp, tok, coords in ((False, False, False), (0.5, True, True), (True, False, True)):
        g1 = torch.Generator(device=cuda).manual_seed(11)
        g2 = torch.Generator(device=cuda).manual_seed(11)
        s = c.sampler(256, 3000, g1, reverse_complement=rcp, tokens=tok, return_coords=coords)
        for k in range(6):
            if k == 3:                                   # reseeded, then used elsewhere: the sampler follows
                g1.manual_seed(77); g2.manual_seed(77)
                torch.rand(5, generator=g1, device=cuda); torch.rand(5, generator=g2, device=cuda)
            got = s()
            want = c.sample(256, 3000, generator=g2, reverse_complement=rcp, tokens=tok, return_coords=coords)
            if coords:
                assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
            else:
                assert torch.equal(got, want)
            assert g1.get_offset() == g2.get_offset()   # the generator advanced as the eager call advanced its twin
        assert s.status() == 0


def test_samplers_on_two_streams_after_a_larger_call(cfg0, cuda):
    """Two captured samplers replayed concurrently on two streams, after a larger eager call, give what eager sample()
    gives with identically seeded generators: every call has its own scratch (torch's allocator; a graph keeps the one
    it was captured with), so neither concurrency nor a later, larger call can disturb a captured sampler."""
    c, _, _ = cfg0
    s1 = c.sampler(256, 8192, torch.Generator(device=cuda).manual_seed(11), reverse_complement=0.5, tokens=True)
    s2 = c.sampler(256, 8192, torch.Generator(device=cuda).manual_seed(12), reverse_complement=0.5)
    e1, e2 = torch.Generator(device=cuda).manual_seed(11), torch.Generator(device=cuda).manual_seed(12)
    nb = c.info(0)["bases"]
    big = c.windows(torch.zeros(4096, dtype=torch.int64), torch.arange(4096, dtype=torch.int64) * 100, 20000)
    assert big.shape == (4096, 20000) and nb > 4096 * 100 + 20000
    st1, st2 = torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)
    for _ in range(3):
        st1.wait_stream(torch.cuda.current_stream(cuda))
        st2.wait_stream(torch.cuda.current_stream(cuda))
        with torch.cuda.stream(st1):
            x1 = s1().clone()
        with torch.cuda.stream(st2):
            x2 = s2().clone()
        torch.cuda.synchronize(cuda)
        assert torch.equal(x1, c.sample(256, 8192, generator=e1, reverse_complement=0.5, tokens=True))
        assert torch.equal(x2, c.sample(256, 8192, generator=e2, reverse_complement=0.5))
    assert s1.status() == 0 and s2.status() == 0
