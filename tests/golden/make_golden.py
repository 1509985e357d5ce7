"""Regenerate the golden fixtures of tests/golden/ from the reference checkout (run where the reference is present):

    python tests/golden/make_golden.py [--reference <the reference checkout>]

What it writes, all produced by the reference itself:
  data/{synthA,synthB}.{q1k,q4k,q16k}.rr3  the reference's own test archives (its tests/data), unchanged bytes
  synth_ref.fa.xz                          the reference FASTA those archives pin by SHA-256, written by running the
                                           reference's deterministic tests/synth.py (xz-compressed here)
  windows.npz                              seeded window coordinates and flags with the XXH3-64 of each window as the
                                           reference's compiled CPU decoder (Core.windows, oracle/_ref) returns it
  info.json                                per archive: header fields and contig table as the reference's Core reports
                                           them, the XXH3 of its CPU full decode (fasta), and the FormatError text of
                                           each host-made corruption the reference's tests use
"""
import argparse
import json
import lzma
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
DATASETS = ("q1k", "q4k", "q16k")
NAMES = ("synthA", "synthB")
WS = (1, 13, 100, 777, 1024, 4096, 5000, 8192, 16385)
FLAGS = ((False, False, True), (True, False, True), (True, True, True), (False, False, False))   # rc, tokens, apply_case
PER = 48


def mutations(raw):
    """Host-made corruptions (the reference's tests/test_synth.py:103-110 uses these four)."""
    return {
        "header_byte": raw[:40] + bytes([raw[40] ^ 1]) + raw[41:],
        "header_xxh3": raw[:130] + bytes([raw[130] ^ 1]) + raw[131:],
        "truncated": raw[:-1],
        "version": raw[:8] + b"\x02" + raw[9:],
    }


def main():
    ap = argparse.ArgumentParser()
    # the reference checkout: $PANVRAM_REFERENCE, else a directory named "reference" beside this repository
    ap.add_argument("--reference", default=os.environ.get("PANVRAM_REFERENCE") or
                    os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))), "reference"))
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.reference, "tests"))
    import synth  # the reference's own deterministic generator
    import torch
    from oracle import oracle as O
    R = O.reference_extension()
    if R is None:
        sys.exit("build the reference first: python oracle/build_ref.py")
    tmp = tempfile.mkdtemp()
    files = synth.write(tmp)
    with open(files["synth_ref.fa"], "rb") as f, lzma.open(os.path.join(HERE, "synth_ref.fa.xz"), "wb", preset=9) as g:
        g.write(f.read())
    os.makedirs(os.path.join(HERE, "data"), exist_ok=True)
    for ds in DATASETS:
        for nm in NAMES:
            shutil.copyfile(os.path.join(a.reference, "tests", "data", f"{nm}.{ds}.rr3"), os.path.join(HERE, "data", f"{nm}.{ds}.rr3"))
    import xxhash
    rng = np.random.default_rng(20261201)
    rows = {k: [] for k in ("ds", "W", "rc", "tokens", "apply_case", "asm", "start", "xxh3")}
    info = {"reference_sha256": None, "archives": {}, "refusals": {}}
    for di, ds in enumerate(DATASETS):
        paths = [os.path.join(HERE, "data", f"{nm}.{ds}.rr3") for nm in NAMES]
        core = R.Core(files["synth_ref.fa"], paths, 2, False, False)
        info["reference_sha256"] = core.ref_sha256
        ctgs = [core.contigs(i) for i in range(len(NAMES))]
        for i, nm in enumerate(NAMES):
            d = dict(core.info(i))
            d["contigs"] = [list(c) for c in ctgs[i]]
            d["fasta_decoded_xxh3"] = "%016x" % xxhash.xxh3_64_intdigest(core.fasta(i, True))
            d.pop("path", None)
            info["archives"][f"{nm}.{ds}"] = d
        for W in WS:
            for rc, tok, case in FLAGS:
                asm, start = [], []
                for _ in range(PER):
                    ai = int(rng.integers(0, len(NAMES)))
                    ok = [c for c in ctgs[ai] if c[2] >= W]
                    if ok and rng.random() < 0.85:                    # inside one contig, as sample() draws
                        c = ok[int(rng.integers(0, len(ok)))]
                        s = c[3] + int(rng.integers(0, c[2] - W + 1))
                    else:                                             # anywhere in the stream (windows() allows it)
                        s = int(rng.integers(0, core.info(ai)["bases"] - W + 1))
                    asm.append(ai)
                    start.append(s)
                rcm = rng.random(PER) < 0.5 if rc else np.zeros(PER, bool)
                x = core.windows(torch.tensor(asm), torch.tensor(start), W, torch.tensor(rcm) if rc else None, tok, case, True, 2).numpy()
                for k in range(PER):
                    rows["ds"].append(di); rows["W"].append(W); rows["rc"].append(bool(rcm[k])); rows["tokens"].append(tok)
                    rows["apply_case"].append(case); rows["asm"].append(asm[k]); rows["start"].append(start[k])
                    rows["xxh3"].append(xxhash.xxh3_64_intdigest(x[k].tobytes()))
    np.savez_compressed(os.path.join(HERE, "windows.npz"), ds=np.array(rows["ds"], np.int8), W=np.array(rows["W"], np.int64),
                        rc=np.array(rows["rc"], bool), tokens=np.array(rows["tokens"], bool), apply_case=np.array(rows["apply_case"], bool),
                        asm=np.array(rows["asm"], np.int8), start=np.array(rows["start"], np.int64), xxh3=np.array(rows["xxh3"], np.uint64))
    raw = open(os.path.join(HERE, "data", "synthA.q4k.rr3"), "rb").read()
    for k, b in mutations(raw).items():
        p = os.path.join(tmp, "synthA.q4k.rr3")
        open(p, "wb").write(b)
        try:
            R.Core(files["synth_ref.fa"], [p], 1, False, False)
            info["refusals"][k] = None
        except ValueError as e:
            info["refusals"][k] = str(e).replace(p, "<path>")
    with open(os.path.join(HERE, "info.json"), "w") as f:
        json.dump(info, f, indent=1, sort_keys=True)
    shutil.rmtree(tmp)
    print("golden fixtures written:", len(rows["W"]), "windows")


if __name__ == "__main__":
    main()
