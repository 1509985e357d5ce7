"""The Megatron adapter's calls into panvram, run against this package.

The reference's tools/megatron adapter cannot be imported on the GPU box (it needs Megatron-LM, and the reference tree
is not there), so its two calls into panvram are restated here with their surroundings, line for line where they
touch the cohort:
  * PanvramGPTLoader.batch's fast path (tools/megatron/panvram_loader.py:80-122): one Cohort.windows(asm, start, L,
    tokens=True) call for the micro-batch's in-document samples, then `lut5[raw.long()]`, the next-token shift, the
    loss mask and position ids;
  * PanvramIndexedDataset.get (tools/megatron/panvram_dataset.py:105-120): a document's slice as token ids through a
    case-blind byte table, the virtual end-of-document id past the document's bases.
Both run through panvram_b200 as `import panvram_b200 as panvram` would, and are checked against the oracle's bytes
for the same coordinates; the fused id map (windows(token_ids=...)) must equal the adapter's two-step map."""
import numpy as np
import pytest
import torch

from conftest import NAMES

pytestmark = pytest.mark.gpu

EOD_ID = 12
TOKEN_IDS = (8, 5, 6, 7, 9)                      # A, C, G, T, other (tools/megatron/panvram_dataset.py:30-31)


def _lut(token_ids=TOKEN_IDS):
    """byte -> id, both cases mapped (tools/megatron/panvram_dataset.py:38-45)"""
    a, c, g, t, n = token_ids
    lut = np.full(256, n, dtype=np.uint16)
    for ch, v in (("A", a), ("C", c), ("G", g), ("T", t)):
        lut[ord(ch)] = v
        lut[ord(ch.lower())] = v
    return lut


class Docs:
    """The document table PanvramIndexedDataset builds from the cohort (tools/megatron/panvram_dataset.py:64-79): one
    document per contig, assemblies in order; its get() (:105-120)."""

    def __init__(self, cohort):
        self.cohort = cohort
        asm, ln, boff = [], [], []
        for a in range(len(cohort.names)):
            for cname, _, clen, off, _ in cohort._core.contigs(a):
                asm.append(a)
                ln.append(int(clen))
                boff.append(int(off))
        self.doc_asm = np.array(asm, dtype=np.int64)
        self.doc_start = np.array(boff, dtype=np.int64)
        self.doc_bases = np.array(ln, dtype=np.int64)
        self.lengths = (self.doc_bases + 1).astype(np.int32)
        self.lut = _lut()
        self.token_ids = TOKEN_IDS

    def get(self, idx, offset=0, length=None):
        idx, offset = int(idx), int(offset)
        total = int(self.lengths[idx])
        length = total - offset if length is None else int(length)
        if offset < 0 or length < 0 or offset + length > total:
            raise IndexError(f"document {idx}: offset {offset} length {length} outside {total}")
        take = max(0, min(length, int(self.doc_bases[idx]) - offset))
        out = np.empty(length, dtype=np.uint16)
        if take:
            asm = torch.tensor([int(self.doc_asm[idx])], dtype=torch.int64)
            st = torch.tensor([int(self.doc_start[idx]) + offset], dtype=torch.int64)
            raw = self.cohort.windows(asm, st, take)[0]
            out[:take] = self.lut[raw.cpu().numpy()]
        if take < length:
            out[take:] = EOD_ID
        return out


def fast_batch(cohort, docs, samples, S, extra, eod, pad, eod_mask_loss, reset_position_ids, fused_ids):
    """PanvramGPTLoader.batch for a micro-batch whose samples are all on the fast path (panvram_loader.py:88-122):
    samples = [(document, offset)], each sample L = S + extra tokens inside its document. fused_ids: decode through
    windows(token_ids=lut5) instead of lut5[windows(tokens=True).long()] (the same ids, written by the kernel)."""
    dev = cohort.device
    L = S + extra
    lut5 = torch.tensor(docs.token_ids, dtype=torch.int64, device=dev)
    ar = torch.arange(S, dtype=torch.int64, device=dev)
    asm = torch.tensor([int(docs.doc_asm[d]) for d, _ in samples], dtype=torch.int64, device=dev)
    st = torch.tensor([int(docs.doc_start[d]) + int(o) for d, o in samples], dtype=torch.int64, device=dev)
    if fused_ids:
        text = cohort.windows(asm, st, L, token_ids=docs.token_ids)
    else:
        raw = cohort.windows(asm, st, L, tokens=True)
        text = lut5[raw.long()]
    if extra:
        tk, lb = text[:, :-1], text[:, 1:]
    else:
        tk = text
        lb = torch.roll(text, shifts=-1, dims=1)
        lb[:, -1] = pad
    lm = torch.ones(tk.shape, dtype=torch.float32, device=dev)
    if eod_mask_loss:
        lm[tk == eod] = 0.0
    pos = ar.expand(tk.shape[0], S)
    if reset_position_ids:
        mark = torch.zeros(tk.shape, dtype=torch.bool, device=dev)
        mark[:, 1:] = tk[:, :-1] == eod
        seg = torch.where(mark, ar.expand_as(mark), torch.zeros_like(pos)).cummax(dim=1).values
        pos = pos - seg
    lm[lb == pad] = 0.0
    tk = tk.masked_fill(tk == pad, 0)
    lb = lb.masked_fill(lb == pad, 0)
    return {"tokens": tk, "labels": lb, "loss_mask": lm, "position_ids": pos}


@pytest.fixture(scope="module")
def q16k(golden, cuda, oracle_cohorts):
    import panvram_b200 as panvram
    c = panvram.Cohort.open(golden["dirs"]["q16k"], device=cuda, dataset="q16k", reference=golden["ref"])
    return c, Docs(c), oracle_cohorts["q16k"]


@pytest.mark.parametrize("extra", [1, 0])
def test_loader_fast_path(q16k, extra):
    c, docs, (ref, arcs) = q16k
    S = 1000
    L = S + extra
    rng = np.random.default_rng(5 + extra)
    ok = np.nonzero(docs.doc_bases >= L)[0]
    samples = [(int(d), int(rng.integers(0, docs.doc_bases[d] - L + 1))) for d in rng.choice(ok, 64)]
    lutv = np.array(TOKEN_IDS, dtype=np.int64)
    # the oracle's bytes -> tokens 0..4 (A/a 0, C/c 1, G/g 2, T/t 3, else 4) -> ids: what the fast path must give
    want_text = np.stack([lutv[arcs[int(docs.doc_asm[d])].window(int(docs.doc_start[d]) + o, L, tokens=True)] for d, o in samples])
    for fused in (False, True):
        b = fast_batch(c, docs, samples, S, extra, eod=EOD_ID, pad=-1, eod_mask_loss=True, reset_position_ids=True, fused_ids=fused)
        tk = b["tokens"].cpu().numpy()
        lb = b["labels"].cpu().numpy()
        assert np.array_equal(tk, want_text[:, :S]), fused
        if extra:
            assert np.array_equal(lb, want_text[:, 1:])
        else:
            assert np.array_equal(lb[:, :-1], want_text[:, 1:]) and (lb[:, -1] == 0).all()
        lm = b["loss_mask"].cpu().numpy()                       # no end-of-document id inside a document; without the
        assert (lm[:, :S - 1 + extra] == 1).all() and (lm[:, -1] == extra).all()   # extra token the last label is padding
        assert np.array_equal(b["position_ids"].cpu().numpy(), np.broadcast_to(np.arange(S), (len(samples), S)))


def test_dataset_get(q16k):
    c, docs, (ref, arcs) = q16k
    lut = _lut()
    rng = np.random.default_rng(9)
    for _ in range(100):
        d = int(rng.integers(0, len(docs.lengths)))
        total = int(docs.lengths[d])
        off = int(rng.integers(0, total))
        ln = int(rng.integers(0, min(total - off, 20000) + 1))
        got = docs.get(d, off, ln)
        take = max(0, min(ln, int(docs.doc_bases[d]) - off))
        a = int(docs.doc_asm[d])
        want = np.concatenate([lut[arcs[a].window(int(docs.doc_start[d]) + off, take)] if take else np.zeros(0, np.uint16),
                               np.full(ln - take, EOD_ID, np.uint16)])
        assert np.array_equal(got, want), (d, off, ln)
    whole = docs.get(0)
    assert len(whole) == docs.lengths[0] and whole[-1] == EOD_ID
    with pytest.raises(IndexError):
        docs.get(0, 1, int(docs.lengths[0]))
    assert len(NAMES) == len(c.names)
