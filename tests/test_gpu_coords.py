"""sample()'s coordinate step (pv_sample_coords) against the reference's own arithmetic, restated here with the torch
ops of panvram/cohort.py:168-194 on the same draws. Integer work: compared exactly."""
import numpy as np
import pytest
import torch

from conftest import DATASETS

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cohorts(golden, cuda):
    import panvram_b200 as P
    return {ds: P.Cohort.open(golden["dirs"][ds], device=cuda, dataset=ds, reference=golden["ref"]) for ds in DATASETS}


def _reference_coords(ctg, W, n, g, rcarg, device):
    """panvram/cohort.py:168-194, the coordinate half of sample(), as the reference writes it."""
    v = (ctg["ctg_len"] - W + 1).clamp_min(0)
    cum = torch.cumsum(v, 0)
    total = int(cum[-1].item())
    u = torch.randint(0, total, (n,), generator=g, device=device, dtype=torch.int64)
    k = torch.searchsorted(cum, u, right=True)
    pos = u - (cum[k] - v[k])
    if rcarg is True:
        rc = torch.ones(n, dtype=torch.bool, device=device)
    elif rcarg is False:
        rc = None
    else:
        rc = torch.rand(n, generator=g, device=device) < float(rcarg)
    strand = rc.to(torch.int64) if rc is not None else torch.zeros(n, dtype=torch.int64, device=device)
    return torch.stack([ctg["ctg_asm"][k], ctg["ctg_local"][k], pos, strand], 1)


@pytest.mark.parametrize("ds", DATASETS)
def test_sample_coords_equal_reference_arithmetic(cohorts, ds, cuda):
    """Same seed -> the same (assembly, contig, start, strand) as the reference's sample(), for every strand mode and
    for window lengths that leave some contigs without a valid start; the generators end in the same state."""
    c = cohorts[ds]
    for W, rcarg, n in ((1, False, 50), (1000, True, 300), (5000, 0.5, 1000), (16385, 0.3, 257), (8192, 1.0, 4), (64, 0.5, 0)):
        g1 = torch.Generator(device=cuda).manual_seed(W + n)
        g2 = torch.Generator(device=cuda).manual_seed(W + n)
        x, co = c.sample(n, W, generator=g1, reverse_complement=rcarg, return_coords=True)
        want = _reference_coords(c._ctg, W, n, g2, rcarg, cuda)
        assert co.dtype == torch.int64 and co.shape == (n, 4)
        assert torch.equal(co, want), (W, rcarg)
        assert torch.equal(g1.get_state(), g2.get_state())
        assert x.shape == (n, W)


def test_sample_default_generator_and_user_capture(cohorts, cuda):
    """Eager sample() makes its draws in the coordinate kernel from the generator's state: with the default CUDA
    generator too (the same coordinates as the reference's torch calls, the generator left where they leave it). Inside
    a CUDA graph a caller captures, sample() keeps torch's own draw calls, so each replay draws anew as torch's
    graph-safe generator does: replays equal successive eager calls."""
    c = cohorts["q4k"]
    torch.cuda.manual_seed(123)
    _, co = c.sample(300, 1000, reverse_complement=0.5, return_coords=True)
    st = torch.cuda.get_rng_state(cuda)
    torch.cuda.manual_seed(123)
    want = _reference_coords(c._ctg, 1000, 300, None, 0.5, cuda)
    assert torch.equal(co, want) and torch.equal(st, torch.cuda.get_rng_state(cuda))
    g = torch.Generator(device=cuda).manual_seed(9)
    e = torch.Generator(device=cuda).manual_seed(9)
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(side):
        c.sample(64, 3000, generator=torch.Generator(device=cuda).manual_seed(1), check=False)      # warm-up off the graph
    torch.cuda.current_stream(cuda).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    graph.register_generator_state(g)
    with torch.cuda.graph(graph):
        x, co = c.sample(64, 3000, generator=g, reverse_complement=0.5, return_coords=True, check=False)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize(cuda)
        wx, wco = c.sample(64, 3000, generator=e, reverse_complement=0.5, return_coords=True)
        assert torch.equal(co, wco) and torch.equal(x, wx)


def test_coords_kernel_many_contigs(cuda):
    """The 32-way search at several levels: 40,000 contigs (about a fifth shorter than W, so runs of equal prefix
    sums), draws including both ends of the range, against torch.searchsorted(right=True)."""
    from panvram_b200 import _C
    rng = np.random.default_rng(5)
    for nctg, W in ((1, 100), (31, 100), (33, 100), (1025, 1000), (40000, 5000)):
        lens = rng.integers(1, 3 * W, nctg)
        lens[rng.random(nctg) < 0.2] = W - 1
        lens[0] = max(lens[0], W)
        ctg = {"ctg_len": torch.from_numpy(lens.astype(np.int64)).to(cuda),
               "ctg_asm": torch.from_numpy(rng.integers(0, 100, nctg).astype(np.int64)).to(cuda),
               "ctg_boff": torch.from_numpy(rng.integers(0, 1 << 40, nctg).astype(np.int64)).to(cuda),
               "ctg_local": torch.arange(nctg, dtype=torch.int64, device=cuda) * 7}
        v = (ctg["ctg_len"] - W + 1).clamp_min(0)
        cum = torch.cumsum(v, 0)
        total = int(cum[-1].item())
        n = 5000
        u = torch.from_numpy(np.concatenate([[0, total - 1], rng.integers(0, total, n - 2)]).astype(np.int64)).to(cuda)
        r = torch.rand(n, device=cuda)
        asm = torch.empty(n, dtype=torch.int64, device=cuda)
        start = torch.empty(n, dtype=torch.int64, device=cuda)
        rc = torch.empty(n, dtype=torch.uint8, device=cuda)
        coords = torch.empty((n, 4), dtype=torch.int64, device=cuda)
        status = torch.full((1,), 77, dtype=torch.int32, device=cuda)
        _C.sample_coords(cum, v, ctg, u, r, 0.25, 2, asm, start, rc, coords, status)
        k = torch.searchsorted(cum, u, right=True)
        pos = u - (cum[k] - v[k])
        strand = (r < 0.25).to(torch.int64)
        assert int(status.item()) == 0
        assert torch.equal(asm, ctg["ctg_asm"][k]) and torch.equal(start, ctg["ctg_boff"][k] + pos), nctg
        assert torch.equal(rc.to(torch.int64), strand)
        assert torch.equal(coords, torch.stack([ctg["ctg_asm"][k], ctg["ctg_local"][k], pos, strand], 1)), nctg
        assert bool((v[k] > 0).all()) and bool((pos >= 0).all()) and bool((pos < v[k]).all())


@pytest.mark.parametrize("total", [1, 1000, (1 << 28) - 1, 1 << 28, 198_000_000_007])
def test_in_kernel_draws_equal_torch(cohorts, total, cuda):
    """pv_sample_draw_coords makes the draws torch.randint(0, total, (n,)) and torch.rand(n) make on a generator in the
    same state, bit for bit, for both of randint's paths (range below / from 2^28), for n from 1 to beyond one pass of
    torch's grid-stride loop (more than 2 x 303,104 elements on a 148-SM B200), after the generator has been used; and
    it advances its copy of the offset exactly as those calls advance the generator."""
    from panvram_b200 import _C
    c = cohorts["q4k"]
    cum = torch.tensor([total], dtype=torch.int64, device=cuda)            # one contig holding every start
    ctg = {"ctg_asm": torch.zeros(1, dtype=torch.int64, device=cuda), "ctg_boff": torch.zeros(1, dtype=torch.int64, device=cuda),
           "ctg_local": torch.zeros(1, dtype=torch.int64, device=cuda)}
    for n in (1, 3, 256, 1023, 4096, 303_105, 700_001, 1_300_000):
        g = torch.Generator(device=cuda).manual_seed(1000 + n)
        torch.rand(17, generator=g, device=cuda)                              # a used generator: offset > 0
        seed, off = g.initial_seed(), g.get_offset()
        rng = torch.tensor([seed - (1 << 64) if seed >= 1 << 63 else seed, off, 0], dtype=torch.int64, device=cuda)
        want_u = torch.randint(0, total, (n,), generator=g, device=cuda, dtype=torch.int64)
        want_r = torch.rand(n, generator=g, device=cuda)
        asm = torch.empty(n, dtype=torch.int64, device=cuda)
        start = torch.empty(n, dtype=torch.int64, device=cuda)
        rc = torch.empty(n, dtype=torch.uint8, device=cuda)
        u = torch.empty(n, dtype=torch.int64, device=cuda)
        r = torch.empty(n, dtype=torch.float32, device=cuda)
        _C.sample_draw_coords(cum, cum, ctg, total, rng, 0.5, 2, n, asm, start, rc, u_out=u, r_out=r)
        torch.cuda.synchronize(cuda)
        assert torch.equal(u, want_u), (total, n)
        assert torch.equal(r.view(torch.int32), want_r.view(torch.int32)), (total, n)
        assert torch.equal(start, want_u) and torch.equal(rc, (want_r < 0.5).to(torch.uint8)), (total, n)
        assert int(rng[1].item()) == g.get_offset() and int(rng[2].item()) == 0, (total, n)
