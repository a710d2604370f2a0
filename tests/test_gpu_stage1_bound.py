"""Stage 1's dense-bound path (csrc/stage1_bound.cu) against its hash-table
path and the oracle: the refined lists (docs, order, partial-score bits) are
identical whichever path produces them, and on realistic corpora the
dense-bound path, not the fallback, produces most of them.  A boundary that
cannot be proven (forced here by an inflated max_doc_len, which widens the
rounding slack) gets a second, larger candidate round.  Queries with fewer
positive docs than k_refine go to the hash-table path (the zero-score fill)."""
import ctypes as C

import numpy as np
import pytest

from chimera_b200 import capi
from oracle import oracle as O
from tests import _corpus

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def P(t):
    return C.c_void_p(t.data_ptr())


def _stage1(c, d, nprobe=None, k_refine=None, labels=None):
    cfg = c["cfg"]
    nprobe = nprobe or cfg.nprobe
    k_refine = k_refine or cfg.k_refine
    nq = c["qrot"].shape[0]
    labels = c["labels"] if labels is None else labels
    lut = torch.from_numpy(O.build_lut(c["qrot"].reshape(-1, 128))).cuda()
    cb1 = torch.from_numpy(np.ascontiguousarray(c["cb1"].reshape(-1))).cuda()
    lab = torch.from_numpy(np.ascontiguousarray(labels.astype(np.uint32)).view(np.int32)).cuda()
    rd = torch.full((nq, k_refine), -7, dtype=torch.int32, device="cuda")
    rp = torch.zeros(nq, k_refine, device="cuda")
    nr = torch.zeros(nq, dtype=torch.int32, device="cuda")
    L = capi.lib()
    st = capi._stream(torch)
    v = C.byref(d.view)
    nb = L.chm_stage1_workspace_bytes(v, nq, nprobe, k_refine)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    capi.check(L.chm_stage1(v, nq, P(lut), P(cb1), P(lab), nprobe, k_refine, P(rd), P(rp), P(nr), None, P(ws), nb,
                            st), "stage1")
    tq = torch.zeros(nq, dtype=torch.int32, device="cuda")
    capi.check(L.chm_stage1_table_queries(v, nq, nprobe, k_refine, 0, P(ws), nb, P(tq), st), "table queries")
    torch.cuda.synchronize()
    return rd.cpu().numpy(), rp.cpu().numpy().view(np.uint32), nr.cpu().numpy(), tq.cpu().numpy()


def _same(a, b):
    rd_a, rp_a, nr_a, _ = a
    rd_b, rp_b, nr_b, _ = b
    np.testing.assert_array_equal(nr_a, nr_b)
    for q in range(len(nr_a)):
        np.testing.assert_array_equal(rd_a[q, :nr_a[q]], rd_b[q, :nr_b[q]], err_msg=f"query {q}")
        np.testing.assert_array_equal(rp_a[q, :nr_a[q]], rp_b[q, :nr_b[q]], err_msg=f"query {q}")


@pytest.mark.parametrize("name", ["mini", "small", "long", "sparse"])
def test_dense_bound_equals_table_path_and_oracle(name):
    c = _corpus.corpus(name)
    d = _corpus.device_index(c, torch)
    dense = _stage1(c, d)
    table = _stage1(c, d.with_dense_stage1(False))
    assert table[3].all()  # the hash-table path alone
    _same(dense, table)
    rd, rp, nr, _ = dense
    for q in range(c["qrot"].shape[0]):
        o = _corpus.oracle_search(c, q)
        assert nr[q] == o["n_refined"]
        np.testing.assert_array_equal(rd[q, :nr[q]], o["refined_docs"])
        np.testing.assert_array_equal(rp[q, :nr[q]], o["refined_partial"].view(np.uint32))


@pytest.mark.parametrize("name", ["sparse", "small"])
def test_dense_bound_produces_most_lists(name):
    """The dense-bound path, not the fallback, produces most refined lists:
    with sparse probing in its first round (K' = 1.5 k_refine); on the small
    corpus, where every doc has several tokens in each query token's lists
    and the sum of visits overestimates, in its second round (K' = every
    doc)."""
    c = _corpus.corpus(name)
    d = _corpus.device_index(c, torch)
    got = _stage1(c, d)
    assert (got[3] == 0).sum() >= len(got[3]) // 2, got[3]
    _same(got, _stage1(c, d.with_dense_stage1(False)))


def test_unproven_first_round_goes_to_second_round():
    """k_refine 20 keeps 84 first-round candidates, far fewer than any query's
    positive docs, and a rounding slack of 40x proves no boundary; the second
    round takes every doc of this corpus (2,000 <= 12,288) as a candidate,
    which needs no boundary, so the dense-bound path still produces every
    list -- identical to the hash-table path's."""
    c = _corpus.corpus("small")
    d = _corpus.device_index(c, torch)
    wide = d.with_dense_stage1(True)
    wide.view.max_doc_len = 1 << 24
    got = _stage1(c, wide, k_refine=20)
    assert not got[3].any()
    _same(got, _stage1(c, d.with_dense_stage1(False), k_refine=20))


@pytest.mark.parametrize("k_refine", [1999, 2048])
def test_short_lists_fall_back_for_zero_fill(k_refine):
    """Fewer positive docs than k_refine: the zero-score fill comes from the
    hash-table path's visited-doc bitmap.  With one probed list per query
    token nearly every query of this corpus is short at k_refine 1999; above
    the doc count (2048 > 2,000 docs) every query is, and the dense-bound pass
    is skipped altogether."""
    c = _corpus.corpus("small")
    d = _corpus.device_index(c, torch)
    nprobe = 1
    labels = O.probe(c["qrot"].reshape(-1, 128), c["centroids_rot"], c["cnorm"], nprobe).reshape(-1, 32, nprobe)
    got = _stage1(c, d, nprobe=nprobe, k_refine=k_refine, labels=labels)
    if k_refine > 2000:
        assert got[3].all()
    else:
        assert got[3].sum() >= len(got[3]) // 2, got[3]
    _same(got, _stage1(c, d.with_dense_stage1(False), nprobe=nprobe, k_refine=k_refine, labels=labels))


@pytest.mark.parametrize("k_refine", [1, 7, 64, 1999, 2000])
def test_dense_bound_k_refine_edges(k_refine):
    """k_refine from 1 to the whole corpus (every doc a candidate)."""
    c = _corpus.corpus("small")
    d = _corpus.device_index(c, torch)
    _same(_stage1(c, d, k_refine=k_refine), _stage1(c, d.with_dense_stage1(False), k_refine=k_refine))
