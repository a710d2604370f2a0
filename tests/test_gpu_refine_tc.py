"""chm_refine_1bit_tc (int8 tensor-core filter + exact LUT sums of the
candidates) against chm_refine_1bit (exact LUT sums of every token): the
1-bit document scores must be identical bit for bit.  Covers the realistic
refined lists of the oracle, random lists, documents longer than one
128-token tile (tensor-core parts whose maxima merge across parts when the
workspace has room -- chm_refine_tc_workspace_bytes -- else the SIMT
long-document kernel), shard-foreign slots (-1) and short per-query counts."""
import numpy as np
import pytest

from chimera_b200 import capi
from oracle import oracle as O
from tests import _corpus

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _run_both(c, d, lists, counts, k_refine, parts=True):
    L = capi.lib()
    st = capi._stream(torch)
    P = capi._ptr
    nq = lists.shape[0]
    qrot = np.ascontiguousarray(c["qrot"][:nq])
    rot = torch.from_numpy(qrot.reshape(-1, 128)).cuda()
    lut = torch.from_numpy(O.build_lut(qrot.reshape(-1, 128))).cuda()
    cb1 = torch.from_numpy(np.ascontiguousarray(c["cb1"][:nq].reshape(-1), np.float32)).cuda()
    rd = torch.from_numpy(np.ascontiguousarray(lists, np.int32)).cuda()
    nr = torch.from_numpy(np.ascontiguousarray(counts, np.int32)).cuda()
    a = torch.full((nq, k_refine), 7.0, device="cuda")
    b = torch.full((nq, k_refine), 7.0, device="cuda")
    capi.check(L.chm_refine_1bit(C_view(d), nq, P(lut), P(cb1), P(rd), P(nr), k_refine, P(a), st), "simt")
    wb = (L.chm_refine_tc_workspace_bytes(C_view(d), nq, k_refine) if parts else
          L.chm_refine_1bit_tc_workspace_bytes(nq, k_refine))
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    capi.check(L.chm_refine_1bit_tc(C_view(d), nq, P(lut), P(cb1), P(rot), P(rd), P(nr), k_refine, P(b), P(ws), wb,
                                    st), "tc")
    torch.cuda.synchronize()
    a, b = a.cpu().numpy(), b.cpu().numpy()
    for q in range(nq):
        n = int(counts[q])
        np.testing.assert_array_equal(a[q, :n].view(np.uint32), b[q, :n].view(np.uint32), err_msg=f"query {q}")
    return a


def C_view(d):
    import ctypes as C
    return C.byref(d.view)


@pytest.mark.parametrize("parts", [True, False])
@pytest.mark.parametrize("layout", ["token", "cluster"])
@pytest.mark.parametrize("name", ["mini", "small", "long"])
def test_refine_tc_matches_simt_on_oracle_lists(name, layout, parts):
    """Both kernels on both 1-bit layouts: the token-order copies (one span
    per doc) and the cluster-ordered arrays gathered through tok2pos."""
    c = _corpus.corpus(name)
    cfg = c["cfg"]
    d = _corpus.device_index(c, torch).with_token_order(layout == "token")
    nq = c["qrot"].shape[0]
    kr = cfg.k_refine
    lists = np.full((nq, kr), -1, np.int32)
    counts = np.zeros(nq, np.int32)
    for q in range(nq):
        tr = _corpus.oracle_search(c, q)
        n = tr["n_refined"]
        lists[q, :n] = tr["refined_docs"]
        counts[q] = n
        # the oracle's own 1-bit scores are the reference for the first query's list
        if q == 0:
            want0 = tr["onebit_scores"]
    a = _run_both(c, d, lists, counts, kr, parts)
    np.testing.assert_array_equal(a[0, :counts[0]].view(np.uint32), want0.view(np.uint32))


@pytest.mark.parametrize("name", ["small", "long"])
def test_refine_tc_random_lists_foreign_slots_and_counts(name):
    c = _corpus.corpus(name)
    cfg = c["cfg"]
    d = _corpus.device_index(c, torch)
    rng = np.random.default_rng(5)
    nq = c["qrot"].shape[0]
    kr = min(cfg.num_docs, 257)
    lists = np.stack([rng.permutation(cfg.num_docs)[:kr] for _ in range(nq)]).astype(np.int32)
    lists[rng.random(lists.shape) < 0.3] = -1          # slots other shards own
    counts = rng.integers(0, kr + 1, nq).astype(np.int32)
    counts[0] = kr
    if nq > 1:
        counts[1] = 0
    a = _run_both(c, d, lists, counts, kr)
    neg = lists[0, :kr] < 0
    assert np.all(np.isneginf(a[0, :kr][neg]))


def test_refine_tc_long_docs_present():
    """The long corpus exercises the multi-tile items."""
    c = _corpus.corpus("long")
    assert int(c["doclens"].max()) > 256
