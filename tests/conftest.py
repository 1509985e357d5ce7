"""Shared fixtures. GPU tests are marked `gpu` (run: pytest -m gpu on a B200); everything else runs on the CPU.
The golden fixtures (tests/golden/) come from the reference itself: its own test archives, its deterministic
reference FASTA, and windows produced by its compiled CPU decoder (see tests/golden/make_golden.py)."""
import json
import lzma
import os
import shutil
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")
DATASETS = ("q1k", "q4k", "q16k")
NAMES = ("synthA", "synthB")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (the B200 parity and scale tests)")


@pytest.fixture(scope="session")
def golden(tmp_path_factory):
    d = tmp_path_factory.mktemp("golden")
    ref = d / "synth_ref.fa"
    ref.write_bytes(lzma.open(os.path.join(GOLDEN, "synth_ref.fa.xz")).read())
    dirs = {}
    for ds in DATASETS:
        dd = d / ds
        dd.mkdir()
        for nm in NAMES:
            shutil.copyfile(os.path.join(GOLDEN, "data", f"{nm}.{ds}.rr3"), dd / f"{nm}.{ds}.rr3")
        dirs[ds] = str(dd)
    with open(os.path.join(GOLDEN, "info.json")) as f:
        info = json.load(f)
    win = dict(np.load(os.path.join(GOLDEN, "windows.npz")))
    return {"root": str(d), "ref": str(ref), "dirs": dirs, "info": info, "windows": win}


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def oracle_cohorts(golden, oracle):
    """dataset -> (Reference, [Archive per name]) opened by the oracle."""
    ref = oracle.Reference(golden["ref"])
    return {ds: (ref, [oracle.Archive(os.path.join(golden["dirs"][ds], f"{nm}.{ds}.rr3"), ref) for nm in NAMES]) for ds in DATASETS}


def golden_cases(win):
    """Group the golden windows into calls: (ds index, W, tokens, apply_case) -> row indices."""
    keys = {}
    for i in range(len(win["W"])):
        k = (int(win["ds"][i]), int(win["W"][i]), bool(win["tokens"][i]), bool(win["apply_case"][i]))
        keys.setdefault(k, []).append(i)
    return keys


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
