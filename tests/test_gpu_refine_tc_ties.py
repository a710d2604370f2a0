"""Documents whose tokens all carry one code tie on every estimate, so every
row is a candidate: an item holding one of them overflows the tensor-core
refinement's 512 candidate slots, the query is flagged, and the SIMT kernels
rescore it.  The scores must still equal the plain kernels' bit for bit, for
the 1-bit and the full-bit scores, and the queries without such a document
must keep the tensor-core path's (identical) scores."""
import numpy as np
import pytest

from chimera_b200 import capi
from tests import _corpus
from tests.test_gpu_fullbit_tc import _both
from tests.test_gpu_refine_tc import _run_both

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _tied_index(c, docs):
    """A device index of corpus c in which each doc of `docs` repeats its
    first token's 1-bit code, full code and factors."""
    codes1 = c["index"].codes1.copy()
    factor1 = c["index"].factor1.copy()
    full = c["full"].copy()
    ff = c["ff"].copy()
    ptr, t2p = c["ptr"], c["tok2pos"]
    for d in docs:
        t0, t1 = int(ptr[d]), int(ptr[d + 1])
        for tok in range(t0 + 1, t1):
            codes1[t2p[tok]] = codes1[t2p[t0]]
            factor1[t2p[tok]] = factor1[t2p[t0]]
            full[tok] = full[t0]
            ff[tok] = ff[t0]
    return capi.DeviceIndex.from_host(
        cluster_pos=c["cluster_pos"], codes1=codes1, factor1=factor1, doc_ids=c["index"].doc_ids,
        tok2pos=t2p, doc_ptrs=ptr, full_codes=full, full_factors=ff, centroids_rot=c["centroids_rot"],
        flips=c["flips"], dim=c["dim"], ex_bits=c["cfg"].ex_bits)


def _lists(c, tied, cap):
    """Query 0 starts with the tied docs; query 1 has none of them."""
    cfg = c["cfg"]
    rng = np.random.default_rng(11)
    nq = c["qrot"].shape[0]
    others = np.array([d for d in range(cfg.num_docs) if d not in set(tied)], np.int32)
    lists = np.stack([rng.permutation(others)[:cap] for _ in range(nq)]).astype(np.int32)
    lists[0, :len(tied)] = tied
    counts = np.full(nq, cap, np.int32)
    return lists, counts


def _pick_tied(c, n=3):
    """Docs of 20..120 tokens: one 128-row item each, more than 512 candidates."""
    lens = np.diff(c["ptr"])
    docs = [int(d) for d in np.nonzero((lens >= 20) & (lens <= 120))[0][:n]]
    assert len(docs) == n
    return docs


def test_refine_tc_tied_rows_overflow_to_simt():
    c = _corpus.corpus("small")
    tied = _pick_tied(c)
    d = _tied_index(c, tied)
    lists, counts = _lists(c, tied, 200)
    a = _run_both(c, d, lists, counts, 200)
    assert np.all(np.isfinite(a[0, :len(tied)]))


def test_fullbit_tc_tied_rows_overflow_to_simt():
    c = _corpus.corpus("small")
    tied = _pick_tied(c)
    d = _tied_index(c, tied)
    lists, counts = _lists(c, tied, 120)
    a = _both(c, d, lists, counts, 120)
    assert np.all(np.isfinite(a[0, :len(tied)]))


def test_refine_tc_at_max_k_refine():
    """k_refine = CHM_MAX_K_REFINE (8192): the item planner's doubling tables
    take about 225 KB of shared memory, the largest launch of that kernel."""
    c = _corpus.corpus("small")
    cfg = c["cfg"]
    d = _corpus.device_index(c, torch)
    rng = np.random.default_rng(13)
    nq = c["qrot"].shape[0]
    cap = 8192
    lists = np.full((nq, cap), -1, np.int32)
    counts = np.full(nq, cfg.num_docs, np.int32)
    for q in range(nq):
        lists[q, :cfg.num_docs] = rng.permutation(cfg.num_docs)
    _run_both(c, d, lists, counts, cap)
    _both(c, d, lists, counts, cap)
