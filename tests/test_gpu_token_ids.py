"""The token-id map fused into the decode's store (pv_windows_ids): windows(token_ids=ids) equals the reference
Megatron adapter's two-pass form, lut5[windows(tokens=True).long()] (tools/megatron/panvram_loader.py:96-97), on both
kernel paths, for aligned and unaligned window lengths, with and without reverse complement. Integer work: exact."""
import numpy as np
import pytest
import torch

from conftest import NAMES

pytestmark = pytest.mark.gpu

IDS = (65, 67, 71, 84, 78)           # arbitrary ids, one of them above 64 so a byte-width mistake would show


@pytest.fixture(scope="module")
def cohort(golden, cuda):
    import panvram_b200 as P
    return P.Cohort.open(golden["dirs"]["q1k"], device=cuda, dataset="q1k", reference=golden["ref"])


def test_token_ids_equal_the_two_pass_map(cohort, cuda):
    from panvram_b200 import _C
    rng = np.random.default_rng(8)
    lut = torch.tensor(IDS, dtype=torch.int64, device=cuda)
    nb = [cohort.info(i)["bases"] for i in range(len(NAMES))]
    for W in (1, 77, 1000, 5000, 8192):
        n = 300
        a = rng.integers(0, len(NAMES), n)
        s = np.array([rng.integers(0, nb[k] - W + 1) for k in a])
        asm = torch.from_numpy(a.astype(np.int64)).to(cuda)
        start = torch.from_numpy(s.astype(np.int64)).to(cuda)
        for rc in (None, torch.from_numpy(rng.random(n) < 0.5).to(cuda)):
            want = lut[cohort.windows(asm, start, W, rc, tokens=True).long()]
            got = cohort.windows(asm, start, W, rc, token_ids=IDS)
            assert got.dtype == torch.int64 and got.shape == (n, W)
            assert torch.equal(got, want), (W, rc is None)
            got2, st = cohort._launch(asm, start, W, rc, True, True, flags=_C.PV_WIN_BLOCK_PATH, ids=list(IDS))
            torch.cuda.synchronize(cuda)
            assert int(st.item()) == 0 and torch.equal(got2, want), (W, "block path")


def test_token_ids_refuses_a_wrong_count(cohort, cuda):
    with pytest.raises(ValueError):
        cohort.windows(torch.zeros(1, dtype=torch.int64), torch.zeros(1, dtype=torch.int64), 10, token_ids=(1, 2, 3))

