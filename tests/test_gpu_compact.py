"""The opt-in compact resident forms on the GPU: a cohort opened with the packed reference, the compact block table or
both gives the same windows (bytes and status) as the plain form - which the other GPU tests check against the oracle
and the reference's kernel - on both kernel paths, with and without the block cache, and uses less device memory."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import NAMES

pytestmark = pytest.mark.gpu

FORMS = {"packed": dict(packed_reference=True), "compact": dict(compact_blocks=True),
         "both": dict(packed_reference=True, compact_blocks=True)}


@pytest.fixture(scope="module")
def sources(golden, tmp_path_factory):
    from panvram_b200 import synth
    d = str(tmp_path_factory.mktemp("cfg0") / "c")
    synth.make_cohort(d, "cfg0")
    out = {ds: dict(path=golden["dirs"][ds], dataset=ds, reference=golden["ref"]) for ds in ("q1k", "q4k", "q16k")}
    out["cfg0"] = dict(path=d, dataset="q4k", reference=os.path.join(d, "reference.fa"))
    return out


def _coords(c, rng, n, W):
    nb = [c.info(i)["bases"] for i in range(len(c))]
    a = rng.integers(0, len(c), n)
    s = np.array([rng.integers(0, max(1, nb[k] - W + 1)) for k in a])
    s[: n // 8] = 0                                        # assembly starts: copies from the reference's first bases
    return a, s


@pytest.mark.parametrize("src", ["q1k", "q4k", "q16k", "cfg0"])
@pytest.mark.parametrize("form", list(FORMS))
def test_forms_give_the_same_windows(sources, src, form, cuda):
    import panvram_b200 as P
    from panvram_b200 import _C
    kw = sources[src]
    plain = P.Cohort.open(kw["path"], device=cuda, dataset=kw["dataset"], reference=kw["reference"])
    rng = np.random.default_rng(5)
    for cache in (True, False):
        c = P.Cohort.open(kw["path"], device=cuda, dataset=kw["dataset"], reference=kw["reference"], block_cache=cache, **FORMS[form])
        if src == "cfg0" and cache:
            assert c.resident_bytes()["total"] < plain.resident_bytes()["total"]
        for W in (1, 100, 4096, 8192, 20000):
            for tokens, rcp in ((False, 0.0), (True, 0.5), (False, 1.0)):
                a, s = _coords(c, rng, 200, W)
                asm = torch.from_numpy(a.astype(np.int64)).to(cuda)
                start = torch.from_numpy(s.astype(np.int64)).to(cuda)
                rc = torch.from_numpy(rng.random(200) < rcp).to(cuda) if rcp else None
                want, st_w = plain._launch(asm, start, W, rc, tokens, True)
                for flags in (_C.PV_WIN_FUSED, _C.PV_WIN_SPLIT, _C.PV_WIN_BLOCK_PATH | _C.PV_WIN_FUSED, _C.PV_WIN_BLOCK_PATH | _C.PV_WIN_SPLIT):
                    got, st_g = c._launch(asm, start, W, rc, tokens, True, flags=flags)
                    torch.cuda.synchronize(cuda)
                    assert int(st_g.item()) == int(st_w.item()) == 0, (src, form, cache, W, flags)
                    assert torch.equal(got, want), (src, form, cache, W, tokens, rcp, flags)


def test_forms_sample_and_full_decode(sources, cuda):
    """sample() and check_full through both forms at once, on the synthetic cohort."""
    import panvram_b200 as P
    kw = sources["cfg0"]
    plain = P.Cohort.open(kw["path"], device=cuda, dataset="q4k", reference=kw["reference"])
    both = P.Cohort.open(kw["path"], device=cuda, dataset="q4k", reference=kw["reference"], **FORMS["both"])
    g1 = torch.Generator(device=cuda).manual_seed(3)
    g2 = torch.Generator(device=cuda).manual_seed(3)
    x, co = plain.sample(512, 8192, generator=g1, reverse_complement=0.5, tokens=True, return_coords=True)
    y, co2 = both.sample(512, 8192, generator=g2, reverse_complement=0.5, tokens=True, return_coords=True)
    assert torch.equal(co, co2) and torch.equal(x, y)
    for a in range(len(both)):
        ok, h = both.check_full(a)
        assert ok, (a, h)
