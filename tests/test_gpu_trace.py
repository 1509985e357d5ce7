"""The per-item kernel trace (pv_windows_trace): %globaltimer at every phase of every work item, for measuring where a
call's time goes (the reference has no such mode; its logs time its decode ad hoc)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_trace_mode(golden, cuda):
    """pv_windows_trace: the same windows as the plain call, one record per work item, phases in time order, every
    located item decoded and emitted, on both kernel forms."""
    import panvram_b200 as P
    from panvram_b200 import _C
    c = P.Cohort.open(golden["dirs"]["q16k"], device=cuda, dataset="q16k", reference=golden["ref"])
    rng = np.random.default_rng(3)
    nb = [c.info(i)["bases"] for i in range(len(c))]
    n, W = 700, 8192
    a = rng.integers(0, len(c), n)
    s = np.array([rng.integers(0, nb[k] - W + 1) for k in a])
    for flags, form in ((_C.PV_WIN_FUSED, 1), (_C.PV_WIN_SPLIT, 2)):
        want = c.windows(torch.from_numpy(a), torch.from_numpy(s), W, tokens=True)
        x, st, summ, tr = c.trace_windows(a, s, W, tokens=True, flags=flags)
        assert st == 0 and torch.equal(x, want)
        assert tr.shape == (_C._lib.pv_windows_items(ctypes.byref(c._devc), n, W), 8)
        t = tr.astype(np.int64)
        state = (tr[:, 7] >> np.uint64(8)) & np.uint64(15)
        done = state == 1
        assert done.sum() > n and summ["decoded"] == done.sum()
        d = t[done]
        assert ((d[:, 0] <= d[:, 1]) & (d[:, 1] <= d[:, 2]) & (d[:, 2] <= d[:, 3]) & (d[:, 3] <= d[:, 6])).all()
        assert (((tr[done, 7] >> np.uint64(12)) & np.uint64(3)) == form).all()
        if form == 2:
            assert ((d[:, 3] <= d[:, 4]) & (d[:, 4] <= d[:, 5]) & (d[:, 5] <= d[:, 6])).all()
        assert summ["decode_ns"]["max"] > 0 and summ["call_ns"] > 0
