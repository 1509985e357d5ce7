"""Config 0 encoded by the reference's own encoder (run where oracle/_ref/refrel3v1 was built from the reference):

    python tests/golden/make_cfg0.py

The synthetic 8 Mbp reference and the 4 assembly FASTAs come from panvram_b200.synth (config "cfg0", deterministic);
each assembly is encoded as refrel3 v1 q4k by the reference encoder (tools/rr3bench/refrel3v1.cpp) into
tests/golden/cfg0/. Also written: cfg0/windows.npz, the XXH3-64 of windows of sample(1024, 8192)-distributed
coordinates (seed 0), with and without reverse complement / tokens, as the reference's compiled CPU decoder returns
them. The tests regenerate reference.fa with the synthesizer (its SHA-256 is pinned in every archive header)."""
import glob
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
OUT = os.path.join(HERE, "cfg0")


def main():
    import torch
    import xxhash
    from oracle import oracle as O
    from panvram_b200.synth import make_cohort
    R = O.reference_extension()
    if R is None or not os.path.exists(O.REF_ENCODER):
        sys.exit("build the reference first: python oracle/build_ref.py")
    tmp = tempfile.mkdtemp()
    make_cohort(tmp, "cfg0", write_fasta=True)
    os.makedirs(OUT, exist_ok=True)
    fas = sorted(glob.glob(os.path.join(tmp, "asm*.fa")))
    for fa in fas:
        name = os.path.basename(fa)[:-3]
        subprocess.run([O.REF_ENCODER, "encode", os.path.join(tmp, "reference.fa"), "4096", "8", fa, os.path.join(OUT, f"{name}.q4k.rr3")],
                       check=True, stdout=subprocess.DEVNULL)
    paths = sorted(glob.glob(os.path.join(OUT, "*.q4k.rr3")))
    core = R.Core(os.path.join(tmp, "reference.fa"), paths, 4, False, False)
    for i, fa in enumerate(fas):
        assert core.fasta(i, True) == open(fa, "rb").read()
    rng = np.random.default_rng(0)
    lens = [c[2] for i in range(len(paths)) for c in core.contigs(i)]
    boff = [c[3] for i in range(len(paths)) for c in core.contigs(i)]
    casm = [i for i in range(len(paths)) for _ in core.contigs(i)]
    W, n = 8192, 1024
    v = np.clip(np.array(lens) - W + 1, 0, None)
    cum = np.cumsum(v)
    u = rng.integers(0, cum[-1], n)
    k = np.searchsorted(cum, u, side="right")
    start = np.array(boff)[k] + (u - (cum[k] - v[k]))
    asm = np.array(casm)[k]
    rc = rng.random(n) < 0.5
    out = {"asm": asm.astype(np.int64), "start": start.astype(np.int64), "rc": rc}
    for tag, r, tok in (("plain", None, False), ("rc_tokens", rc, True), ("rc", rc, False)):
        x = core.windows(torch.from_numpy(asm), torch.from_numpy(start), W, torch.from_numpy(r) if r is not None else None, tok, True, True, 4)
        out["xxh3_" + tag] = np.array([xxhash.xxh3_64_intdigest(row.tobytes()) for row in x.numpy()], dtype=np.uint64)
    np.savez_compressed(os.path.join(OUT, "windows.npz"), **out)
    print("wrote", OUT, [os.path.getsize(p) for p in paths])


if __name__ == "__main__":
    main()
