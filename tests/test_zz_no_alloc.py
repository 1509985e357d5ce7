"""pv_windows_noalloc: the window decode for callers that cannot allocate device memory (for example a data-loading
hook inside a training framework whose allocator owns the GPU's memory). It keeps its scratch in a fixed array inside
the library instead of a caller buffer. Here it is called through the C ABI three times in a row on different windows,
and each result (bytes and status) must equal the ordinary entry point's exactly - the path is integer work, so the
tolerance is zero. The third call is large enough for the two-kernel split form, whose plan also lives in the fixed
array. This file sorts last so that a run stopping at its first failure has run every other test."""
import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import NAMES

pytestmark = pytest.mark.gpu


def _cohort(golden, cuda):
    import panvram_b200 as P
    return P.Cohort.open(golden["dirs"]["q1k"], device=cuda, dataset="q1k", reference=golden["ref"])


def _call(fn, c, asm, start, W, rc, tokens, extra):
    n = asm.numel()
    out = torch.empty((n, W), dtype=torch.uint8, device=c.device)
    status = torch.zeros(1, dtype=torch.int32, device=c.device)
    stream = torch.cuda.current_stream(c.device).cuda_stream
    code = fn(ctypes.byref(c._devc), asm.data_ptr(), start.data_ptr(), n, W, rc.data_ptr() if rc is not None else None,
              int(tokens), 1, out.data_ptr(), status.data_ptr(), *extra, stream)
    return code, out, status


def test_noalloc_matches_windows_twice(golden, cuda):
    from panvram_b200 import _C
    lib = _C._lib
    c = _cohort(golden, cuda)
    rng = np.random.default_rng(2026)
    nb = [c.info(i)["bases"] for i in range(len(NAMES))]
    # two small calls (the one-kernel form), then one of 1,500 x 4 items (the split form, whose plan of every item's
    # decode results also lives in the fixed array)
    for call, (n, W, tokens) in enumerate(((600, 3000, False), (600, 777, True), (1500, 3000, False))):
        if call == 2:
            assert _C.windows_form(c.item_cell, n, W)[0] == 3 and lib.pv_windows_work_bytes(ctypes.byref(c._devc), n, W) <= 16 << 20
        a = rng.integers(0, len(NAMES), n)
        s = np.array([rng.integers(0, nb[k] - W + 1) for k in a])
        asm = torch.from_numpy(a.astype(np.int64)).to(cuda)
        start = torch.from_numpy(s.astype(np.int64)).to(cuda)
        rc = torch.from_numpy((rng.random(n) < 0.5).astype(np.uint8)).to(cuda)
        need = lib.pv_windows_work_bytes(ctypes.byref(c._devc), n, W)
        work = torch.empty(max(need, 1), dtype=torch.uint8, device=cuda)
        code, want, st_want = _call(lib.pv_windows, c, asm, start, W, rc, tokens, (work.data_ptr(), need))
        assert code == 0
        code, got, st_got = _call(lib.pv_windows_noalloc, c, asm, start, W, rc, tokens, ())
        assert code == 0, lib.pv_kernels_last_error()
        torch.cuda.synchronize(cuda)
        assert int(st_got.item()) == int(st_want.item()) == 0, call
        assert torch.equal(got, want), call


def test_noalloc_refuses_beyond_its_scratch(golden, cuda):
    from panvram_b200 import _C
    lib = _C._lib
    c = _cohort(golden, cuda)
    W = 1 << 20                                     # a call whose scratch need exceeds the fixed array: refused, no launch
    n = 4096
    need = lib.pv_windows_work_bytes(ctypes.byref(c._devc), n, W)
    assert need > 16 << 20
    asm = torch.zeros(n, dtype=torch.int64, device=cuda)
    start = torch.zeros(n, dtype=torch.int64, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    code = lib.pv_windows_noalloc(ctypes.byref(c._devc), asm.data_ptr(), start.data_ptr(), n, W, None, 0, 1, None,
                                  status.data_ptr(), torch.cuda.current_stream(cuda).cuda_stream)
    assert code == _C.PV_EARG
    assert b"scratch" in lib.pv_kernels_last_error()
