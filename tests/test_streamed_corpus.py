"""The streamed corpus (chunk-by-chunk generation for corpora larger than a
device) reproduces generate_torch's corpus exactly, and its one-pass ground
truth equals the brute-force MaxSim top-k.  Run on the CPU generator with
small chunks, so that documents straddle chunk boundaries."""
import dataclasses

import numpy as np
import pytest

from chimera_b200 import workloads as W

torch = pytest.importorskip("torch")

CFG = dataclasses.replace(W.CONFIGS["mini"], num_queries=12)
CHUNK = 997  # not a multiple of any doc length: docs straddle chunks


def test_streamed_corpus_matches_generate_torch():
    emb, dl, qs = W.generate_torch(CFG, seed=3, device="cpu", chunk=CHUNK)
    sc = W.StreamedCorpus(CFG, seed=3, device="cpu", chunk=CHUNK)
    assert sc.n == emb.shape[0] and sc.num_chunks == (sc.n + CHUNK - 1) // CHUNK
    assert torch.equal(sc.doclens, dl)
    parts = [x for _, _, x in sc.chunks()]
    assert torch.equal(torch.cat(parts), emb)
    # a sub-range (a document shard) and an arbitrary gather
    lo, hi = 1234, 4321
    assert torch.equal(torch.cat([x for _, _, x in sc.chunks(lo, hi)]), emb[lo:hi])
    ids = torch.tensor([5, sc.n - 1, 0, 998, 997, 5, 2500])
    assert torch.equal(sc.gather(ids), emb[ids])
    assert torch.equal(sc.queries(), qs)


def _brute(emb, dl, queries, k):
    ptr = np.concatenate([[0], np.cumsum(dl.numpy().astype(np.int64))])
    owner = torch.from_numpy(np.repeat(np.arange(len(dl)), dl.numpy()))
    out = []
    for q in queries:
        s = q @ emb.T
        best = torch.full((q.shape[0], len(dl)), -float("inf"))
        best.scatter_reduce_(1, owner.unsqueeze(0).expand(q.shape[0], -1), s, reduce="amax")
        out.append(torch.topk(best.sum(0), k).indices.numpy())
    del ptr
    return out


def test_streamed_ground_truth_matches_brute_force():
    emb, dl, qs = W.generate_torch(CFG, seed=3, device="cpu", chunk=CHUNK)
    sc = W.StreamedCorpus(CFG, seed=3, device="cpu", chunk=CHUNK)
    k = 10
    got = W.ground_truth_streamed(sc, qs, k, group=5)
    want = _brute(emb, dl, qs, k)
    assert len(got) == len(want)
    for g, w in zip(got, want):
        assert set(g.tolist()) == set(w.tolist())
