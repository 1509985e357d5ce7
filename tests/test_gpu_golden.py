"""GPU parity on the reference's own fixtures: the CUDA window decode (through the C ABI, via Cohort) against the
golden windows of the reference's compiled CPU decoder and against the oracle, byte for byte; sample / fetch /
decode / check_full / fasta as the reference's tests exercise them; edge cases and corrupt payloads."""
import os
import random

import numpy as np
import pytest
import torch
import xxhash

from conftest import DATASETS, NAMES, golden_cases

pytestmark = pytest.mark.gpu


# the cohorts with the default checkpoint index (stride 2048, capped at the block size), without one (every item
# decodes its whole block), and with the smallest stride (many items per block, most starting mid-block)
STRIDES = {"index": None, "no-index": 0, "stride-256": 256}


@pytest.fixture(scope="module", params=list(STRIDES))
def cohorts(golden, cuda, request):
    import panvram_b200 as P
    cs = {ds: P.Cohort.open(golden["dirs"][ds], device=cuda, dataset=ds, reference=golden["ref"], checkpoint_stride=STRIDES[request.param])
          for ds in DATASETS}
    for c in cs.values():
        want = 0 if STRIDES[request.param] == 0 else min(STRIDES[request.param] or 2048, c.block_size)
        assert c.checkpoint_stride == want and c.bad_blocks == 0
    return cs


def _hashes(x):
    x = x.cpu().numpy()
    return np.array([xxhash.xxh3_64_intdigest(r.tobytes()) for r in x], dtype=np.uint64)


@pytest.mark.parametrize("flags", [2, 3, 4, 5, 4 | (1 << 8), 4 | (5 << 8)],
                         ids=["fused", "fused-block-path", "split", "split-block-path", "split-1-lane", "split-5-lanes"])
def test_golden_windows(golden, cohorts, flags):
    win = golden["windows"]
    for (di, W, tok, case), rows in golden_cases(win).items():
        c = cohorts[DATASETS[di]]
        rows = np.array(rows)
        x, status = c._launch(torch.from_numpy(win["asm"][rows].astype(np.int64)), torch.from_numpy(win["start"][rows]), W,
                              torch.from_numpy(win["rc"][rows]), tok, case, flags=flags)
        assert int(status.item()) == 0
        assert np.array_equal(_hashes(x), win["xxh3"][rows]), (DATASETS[di], W, tok, case)


@pytest.mark.parametrize("ds", DATASETS)
def test_sample_fetch_vs_oracle(golden, cohorts, oracle_cohorts, oracle, ds, cuda):
    """The reference's test_windows_fetch_fasta (tests/test_synth.py:41-76), with the oracle as the comparison side."""
    c = cohorts[ds]
    ref, arcs = oracle_cohorts[ds]
    assert c.names == list(NAMES) and c.block_size == {"q1k": 1024, "q4k": 4096, "q16k": 16384}[ds]
    g = torch.Generator(device=cuda).manual_seed(7)
    for W in (1, 13, 1024, 4096, 5000, 16385):
        x, co = c.sample(300, W, generator=g, return_coords=True)
        assert x.shape == (300, W) and x.dtype == torch.uint8 and x.device.type == "cuda"
        co = co.cpu().numpy()
        assert (co[:, 3] == 0).all()
        start = np.array([c.contigs(int(a))[int(ci)][3] + int(s) for a, ci, s, _ in co])
        want = oracle.windows(arcs, ref, co[:, 0], start, W, threads=4)
        assert np.array_equal(x.cpu().numpy(), want), W
    for W in (100, 8192):
        x, co = c.sample(200, W, generator=g, reverse_complement=0.5, tokens=True, return_coords=True)
        co = co.cpu().numpy()
        assert 0 < co[:, 3].sum() < 200
        start = np.array([c.contigs(int(a))[int(ci)][3] + int(s) for a, ci, s, _ in co])
        want = oracle.windows(arcs, ref, co[:, 0], start, W, rc=co[:, 3], tokens=True, threads=4)
        assert np.array_equal(x.cpu().numpy(), want), W
    rng = random.Random(11)
    for _ in range(200):
        a = rng.randrange(len(c))
        ctgs = c.contigs(a)
        ci = rng.randrange(len(ctgs))
        name, _, n, boff, _ = ctgs[ci]
        L = min(n, int(2 ** (rng.random() * 15)))
        s = rng.randrange(n - L + 1)
        rcf, tok = rng.random() < 0.3, rng.random() < 0.3
        y = c.fetch(c.names[a] if rng.random() < 0.5 else a, name if rng.random() < 0.5 else ci, s, L, reverse_complement=rcf, tokens=tok)
        assert y.shape == (L,)
        assert np.array_equal(y.cpu().numpy(), arcs[a].window(boff + s, L, rc=rcf, tokens=tok))
    for a in range(len(c)):
        for name, _, n, boff, _ in c.contigs(a):
            assert np.array_equal(c.fetch(a, name, 0, n).cpu().numpy(), arcs[a].window(boff, n))


@pytest.mark.parametrize("ds", DATASETS)
def test_decode_check_full_fasta(golden, cohorts, oracle_cohorts, ds):
    c = cohorts[ds]
    _, arcs = oracle_cohorts[ds]
    for a in range(len(c)):
        ok, h = c.check_full(a)
        assert ok and h == c.info(a)["fasta_xxh3"]
        assert np.array_equal(c.decode(a, chunk=7777).numpy(), arcs[a].window(0, arcs[a].nbases))
        assert c.fasta(a) == arcs[a].fasta(verify=True)


def test_edge_cases(golden, cohorts, oracle_cohorts):
    c = cohorts["q1k"]
    _, arcs = oracle_cohorts["q1k"]
    e = torch.zeros(0, dtype=torch.int64)
    assert c.windows(e, e, 100).shape == (0, 100)
    assert c.windows(torch.tensor([0]), torch.tensor([5]), 0).shape == (1, 0)
    nb = arcs[0].nbases
    # the last bases of the assembly (last block partial), windows over many blocks, block-aligned starts
    for s, W in ((nb - 1, 1), (nb - 1500, 1500), (0, nb), (1024, 1024), (1023, 2), (3 * 1024, 50000), (nb - 50001, 50001)):
        for rcf in (False, True):
            x = c.windows(torch.tensor([0]), torch.tensor([s]), W, torch.tensor([rcf]))
            assert np.array_equal(x[0].cpu().numpy(), arcs[0].window(s, W, rc=rcf)), (s, W, rcf)
    # windows outside the assembly: status 8, as the reference's kernel
    for asm, s, W in (([0], [nb - 10], 11), ([0], [-1], 5), ([2], [0], 5), ([-1], [0], 5)):
        with pytest.raises(RuntimeError, match="status 8"):
            c.windows(torch.tensor(asm), torch.tensor(s), W)
    x = c.windows(torch.tensor([0, 0]), torch.tensor([0, nb]), 4, check=False)
    assert np.array_equal(x[0].cpu().numpy(), arcs[0].window(0, 4))
    with pytest.raises(RuntimeError):
        c.windows(torch.tensor([0]), torch.tensor([0]), 1 << 31)
    with pytest.raises(ValueError):
        c.sample(4, 10 ** 9)
    with pytest.raises(IndexError):
        c.fetch(0, c.contigs(0)[0][0], c.contigs(0)[0][2] - 5, 6)
    with pytest.raises(KeyError):
        c.fetch("nope", 0, 0, 1)


@pytest.mark.parametrize("stride", [None, 0, 256], ids=["index", "no-index", "stride-256"])
def test_corrupt_payload_parity(golden, oracle, tmp_path, cuda, stride):
    """A payload byte flipped: per block, the GPU reports status 1 exactly where the reference decoder fails, and
    otherwise returns exactly the reference decoder's bytes (valid-looking corruption included). With a checkpoint
    index the failing blocks are found when it is built at open; windows over any part of them report status 1."""
    import panvram_b200 as P
    raw = bytearray(open(os.path.join(golden["dirs"]["q4k"], "synthA.q4k.rr3"), "rb").read())
    ref = oracle.Reference(golden["ref"])
    caught = 0
    for k in range(24):
        b = bytearray(raw)
        p = len(b) - 1 - (k * 97) % 3000
        b[p] ^= 1 << (k % 8)
        d = tmp_path / f"c{k}"
        d.mkdir()
        (d / "synthA.q4k.rr3").write_bytes(bytes(b))
        arc = oracle.Archive(str(d / "synthA.q4k.rr3"), ref)
        c = P.Cohort.open(str(d), device=cuda, reference=golden["ref"], checkpoint_stride=stride)
        Q, n = c.block_size, arc.nbases
        bad = 0
        for blk in range(arc.nblocks):
            s, W = blk * Q, min(Q, n - blk * Q)
            try:
                want = arc.window(s, W, apply_case=False)
            except oracle.OracleError:
                want = None
            bad += want is None
            # the whole block, and a window inside it that starts and ends mid-block
            for ws, ww in ((s, W), (s + W // 3, max(1, W // 3))):
                for flags in (2, 4):                        # the fused kernel, and the decode + emission pair
                    x, status = c._launch(torch.tensor([0]), torch.tensor([ws]), ww, None, False, False, flags=flags)
                    st = int(status.item())
                    if want is None:
                        assert st == 1, (k, blk, flags, ws, ww)
                        caught += 1
                    else:
                        assert st == 0 and np.array_equal(x[0].cpu().numpy(), want[ws - s:ws - s + ww]), (k, blk, flags, ws, ww)
        assert c.bad_blocks == (bad if c.checkpoint_stride else 0), k
    assert caught > 0


def test_pinned_host_coordinates(golden, cohorts, cuda):
    """Coordinates in pinned host memory (gathered by a kernel through their mapped addresses, pv_coords_from_host)
    give exactly what the same coordinates on the device give, with and without strands, bool or uint8."""
    c = cohorts["q4k"]
    rng = np.random.default_rng(4)
    nb = [c.info(i)["bases"] for i in range(len(NAMES))]
    for n, W in ((1, 50), (777, 3000), (4096, 257)):
        a = rng.integers(0, len(NAMES), n)
        s = np.array([rng.integers(0, nb[k] - W + 1) for k in a])
        rcb = rng.random(n) < 0.5
        ah, sh = torch.from_numpy(a.astype(np.int64)).pin_memory(), torch.from_numpy(s.astype(np.int64)).pin_memory()
        for rc in (None, torch.from_numpy(rcb).pin_memory(), torch.from_numpy(rcb.astype(np.uint8)).pin_memory()):
            want = c.windows(ah.to(cuda), sh.to(cuda), W, None if rc is None else rc.to(cuda), tokens=True)
            got = c.windows(ah, sh, W, rc, tokens=True)
            assert torch.equal(got, want), (n, W, rc is None)
