"""panvram_b200 against the reference's own GPU kernel: its csrc/pv_cuda.cu built from its sources for sm_100a into
oracle/_ref/panvram_ref_Ccu.so (oracle/build_ref.py --cuda). Same cohort, coordinates and flags -> byte-identical
windows and the same status word; sample() with the same seed -> the same windows and coordinates. Integer work:
compared exactly. Skipped when that build is absent."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import DATASETS, NAMES

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def refext(oracle):
    ext = oracle.reference_extension(cuda=True)
    if ext is None:
        pytest.skip("the reference's CUDA extension is not built (oracle/build_ref.py --cuda)")
    return ext


@pytest.fixture(scope="module")
def pairs(golden, refext, oracle, cuda):
    import panvram_b200 as P
    out = {}
    for ds in DATASETS:
        paths = [os.path.join(golden["dirs"][ds], f"{nm}.{ds}.rr3") for nm in NAMES]
        out[ds] = (P.Cohort.open(golden["dirs"][ds], device=cuda, dataset=ds, reference=golden["ref"]),
                   oracle.ReferenceGPU(refext, golden["ref"], paths, cuda))
    return out


@pytest.mark.parametrize("ds", DATASETS)
def test_windows_equal_reference_kernel(pairs, ds, cuda):
    ours, ref = pairs[ds]
    rng = np.random.default_rng(17)
    nb = [ours.info(i)["bases"] for i in range(len(NAMES))]
    for W in (1, 15, 100, 1024, 4097, 5000, 8192, 16385):
        for tokens in (False, True):
            for rc_mode in ("none", "half", "all"):
                n = 257
                a = rng.integers(0, len(NAMES), n)
                s = np.array([rng.integers(0, max(1, nb[k] - W + 1)) for k in a])
                asm = torch.from_numpy(a.astype(np.int64)).to(cuda)
                start = torch.from_numpy(s.astype(np.int64)).to(cuda)
                rc = None if rc_mode == "none" else (torch.ones(n, dtype=torch.bool, device=cuda) if rc_mode == "all"
                                                     else torch.from_numpy(rng.random(n) < 0.5).to(cuda))
                want, st_want = ref.windows(asm, start, W, rc, tokens)
                got, st_got = ours._launch(asm, start, W, rc, tokens, True)
                torch.cuda.synchronize(cuda)
                assert int(st_got.item()) == int(st_want.item()) == 0, (W, tokens, rc_mode)
                assert torch.equal(got, want), (ds, W, tokens, rc_mode)


@pytest.mark.parametrize("ds", DATASETS)
def test_sample_equal_reference_kernel(pairs, ds, cuda):
    ours, ref = pairs[ds]
    for W, rcarg, tokens in ((8192, 0.5, True), (1000, False, False), (5000, True, True)):
        g1 = torch.Generator(device=cuda).manual_seed(W)
        g2 = torch.Generator(device=cuda).manual_seed(W)
        x, co = ours.sample(300, W, generator=g1, reverse_complement=rcarg, tokens=tokens, return_coords=True)
        y, st, co_ref = ref.sample(300, W, g2, reverse_complement=rcarg, tokens=tokens)
        torch.cuda.synchronize(cuda)
        assert int(st.item()) == 0
        assert torch.equal(co, co_ref), (ds, W)
        assert torch.equal(x, y), (ds, W)


def test_outside_windows_same_status(pairs, cuda):
    """Windows outside their assembly (bad index, negative start, past the end) report status 8, the reference's
    queue kernel's value for them (pv_cuda.cu:47-49). The reference's kernels are not run on these windows: its
    lower-case kernel reads low_cnt[a] before any bounds check (pv_cuda.cu:90), so a window naming no assembly makes it
    read outside its arrays (it faulted the GPU here once)."""
    ours, _ = pairs["q4k"]
    nb = ours.info(0)["bases"]
    for a, s in ((5, 0), (-1, 0), (0, -3), (0, nb)):
        asm = torch.tensor([0, a], dtype=torch.int64, device=cuda)
        start = torch.tensor([0, s], dtype=torch.int64, device=cuda)
        _, st_got = ours._launch(asm, start, 64, None, False, True)
        torch.cuda.synchronize(cuda)
        assert int(st_got.item()) == 8, (a, s)
