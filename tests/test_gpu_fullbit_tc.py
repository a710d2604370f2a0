"""chm_fullbit_score_tc (int8 tensor-core filter + exact sums in the AVX-512
lane order for the candidates) against chm_fullbit_score (exact sums of every
token): identical scores bit for bit, at every code width the filter handles
(w = 1 + ex_bits = 2..7; w = 8 takes the plain kernel), on the oracle's
selected docs, on random doc lists with shard-foreign slots (-1) and short
counts, and on documents longer than one 128-token tile (tensor-core parts
with chm_refine_tc_workspace_bytes' room, else the SIMT long-document
kernel)."""
import ctypes as C

import numpy as np
import pytest

from chimera_b200 import capi
from tests import _corpus

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _both(c, d, lists, counts, cap, parts=True):
    L = capi.lib()
    st = capi._stream(torch)
    P = capi._ptr
    nq = lists.shape[0]
    rot = torch.from_numpy(np.ascontiguousarray(c["qrot"][:nq].reshape(-1, 128))).cuda()
    cbex = torch.from_numpy(np.ascontiguousarray(c["cbex"][:nq].reshape(-1), np.float32)).cuda()
    fd = torch.from_numpy(np.ascontiguousarray(lists, np.int32)).cuda()
    nf = torch.from_numpy(np.ascontiguousarray(counts, np.int32)).cuda()
    a = torch.full((nq, cap), 7.0, device="cuda")
    b = torch.full((nq, cap), 7.0, device="cuda")
    v = C.byref(d.view)
    capi.check(L.chm_fullbit_score(v, nq, P(rot), P(cbex), P(fd), P(nf), cap, P(a), st), "simt")
    wb = L.chm_refine_tc_workspace_bytes(v, nq, cap) if parts else L.chm_fullbit_score_tc_workspace_bytes(nq, cap)
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    capi.check(L.chm_fullbit_score_tc(v, nq, P(rot), P(cbex), P(fd), P(nf), cap, P(b), P(ws), wb, st), "tc")
    torch.cuda.synchronize()
    a, b = a.cpu().numpy(), b.cpu().numpy()
    for q in range(nq):
        n = int(counts[q])
        np.testing.assert_array_equal(a[q, :n].view(np.uint32), b[q, :n].view(np.uint32), err_msg=f"query {q}")
    return a


@pytest.mark.parametrize("name,ex_bits", [("mini", None), ("small", None), ("long", None), ("mini", 1),
                                          ("mini", 2), ("mini", 5), ("mini", 6), ("mini", 7)])
def test_fullbit_tc_matches_simt_on_oracle_lists(name, ex_bits):
    c = _corpus.corpus(name, ex_bits=ex_bits)
    cfg = c["cfg"]
    d = _corpus.device_index(c, torch)
    nq = c["qrot"].shape[0]
    cap = cfg.k_refine
    lists = np.full((nq, cap), -1, np.int32)
    counts = np.zeros(nq, np.int32)
    want = None
    for q in range(nq):
        tr = _corpus.oracle_search(c, q)
        n = len(tr["fullbit_docs"])
        lists[q, :n] = tr["fullbit_docs"]
        counts[q] = n
        if q == 0:
            want = tr["fullbit_scores"]
    a = _both(c, d, lists, counts, cap)
    np.testing.assert_array_equal(a[0, :counts[0]].view(np.uint32), np.asarray(want, np.float32).view(np.uint32))


@pytest.mark.parametrize("parts", [True, False])
@pytest.mark.parametrize("name", ["small", "long"])
def test_fullbit_tc_random_lists(name, parts):
    c = _corpus.corpus(name)
    cfg = c["cfg"]
    d = _corpus.device_index(c, torch)
    rng = np.random.default_rng(9)
    nq = c["qrot"].shape[0]
    cap = min(cfg.num_docs, 200)
    lists = np.stack([rng.permutation(cfg.num_docs)[:cap] for _ in range(nq)]).astype(np.int32)
    lists[rng.random(lists.shape) < 0.25] = -1
    counts = rng.integers(0, cap + 1, nq).astype(np.int32)
    counts[0] = cap
    _both(c, d, lists, counts, cap, parts)
