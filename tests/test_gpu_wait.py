"""Status bit 4, the bounded wait that expired (the reference's semantics: pv_cuda.cu:20,26,78), without a fault: with
PV_WIN_TEST_WAIT every kernel's wait on its shared-memory bulk copies expects 16 bytes no copy brings, so it expires;
each window reports 4, the kernel completes the missing bytes with one more copy and waits until every copy has landed,
and returns. The process stays healthy: the next call on the same stream gives the oracle's windows. Only the one-kernel
form stages copies; the split form's kernels read global memory and wait on nothing, so there the flag changes nothing
(status 0, the oracle's windows)."""
import numpy as np
import pytest
import torch

from conftest import NAMES

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("form", ["fused", "split"])
def test_expired_wait_reports_status_4(golden, cuda, oracle, oracle_cohorts, form):
    import panvram_b200 as P
    from panvram_b200 import _C
    c = P.Cohort.open(golden["dirs"]["q4k"], device=cuda, dataset="q4k", reference=golden["ref"], block_cache=False)
    ref, arcs = oracle_cohorts["q4k"]
    flags = _C.PV_WIN_FUSED if form == "fused" else _C.PV_WIN_SPLIT
    rng = np.random.default_rng(44)
    n, W = 300, 3000
    nb = [c.info(i)["bases"] for i in range(len(NAMES))]
    a = rng.integers(0, len(NAMES), n)
    s = np.array([rng.integers(0, nb[k] - W + 1) for k in a])
    asm, start = torch.from_numpy(a.astype(np.int64)).to(cuda), torch.from_numpy(s.astype(np.int64)).to(cuda)
    ws = torch.zeros((n + 3) // 4 * 4, dtype=torch.uint8, device=cuda)
    with torch.cuda.device(cuda):
        x_t, st = _C.windows_cuda(c._devc, asm, start, W, None, False, True, flags=flags | _C.PV_WIN_TEST_WAIT, wstatus=ws)
        torch.cuda.synchronize(cuda)
    want = oracle.windows(arcs, ref, a, s, W, threads=4)
    got_ws = ws[:n].cpu().numpy()
    if form == "split":
        assert int(st.item()) == 0 and (got_ws == 0).all() and np.array_equal(x_t.cpu().numpy(), want)
    else:
        # every item stages copies without the block cache (but those the general path decodes, after the wait):
        # every window reports 4
        assert int(st.item()) == 4 and (got_ws == 4).all()
    x, st = c._launch(asm, start, W, None, False, True, flags=flags)
    assert int(st.item()) == 0
    assert np.array_equal(x.cpu().numpy(), want)
