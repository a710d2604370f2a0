"""chm_build_cluster_order (the IVF lists and cluster-ordered 1-bit arrays
built on the GPU) against the oracle's stable counting sort
(IVF_PG::build_from_assignments, ivf_pg.cpp:110-126) and reorder_by_cluster
(build_index.cu:328-363): bit-identical cluster_pos, inverted list, codes,
factors, owning docs and token positions.  Covers empty lists, a list longer
than one CTA's shared-memory sort (the big-list kernel) and the out-of-range
assignment status."""
import numpy as np
import pytest

from chimera_b200 import capi
from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
P = capi._ptr


def _run(assign, nc, doclens, codes, f1):
    n = assign.shape[0]
    dev = "cuda"
    a = torch.from_numpy(assign.astype(np.uint32).view(np.int32)).to(dev)
    dp = torch.from_numpy(np.concatenate([[0], np.cumsum(doclens)]).astype(np.int64)).to(dev)
    c = torch.from_numpy(codes).to(dev)
    f = torch.from_numpy(f1).to(dev)
    pos = torch.empty(nc + 1, dtype=torch.int64, device=dev)
    inv = torch.empty(n, dtype=torch.int32, device=dev)
    c1 = torch.empty(n, 16, dtype=torch.uint8, device=dev)
    ff = torch.empty(n, dtype=torch.float32, device=dev)
    docs = torch.empty(n, dtype=torch.int32, device=dev)
    t2p = torch.empty(n, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L = capi.lib()
    wb = L.chm_build_cluster_order_workspace_bytes(n, nc)
    ws = torch.empty(wb, dtype=torch.uint8, device=dev)
    capi.check(L.chm_build_cluster_order(P(a), n, nc, P(dp), len(doclens), P(c), P(f), P(pos), P(inv), P(c1), P(ff),
                                         P(docs), P(t2p), P(status), P(ws), wb, capi._stream(torch)), "order")
    torch.cuda.synchronize()
    g = lambda t: t.cpu().numpy()
    return g(pos), g(inv).view(np.uint32), g(c1), g(ff), g(docs), g(t2p).view(np.uint32), int(status.item())


@pytest.mark.parametrize("n,nc,skew", [(5000, 64, False), (70000, 4096, False), (20000, 50, True)])
def test_cluster_order_matches_oracle(n, nc, skew):
    rng = np.random.default_rng(n + nc)
    if skew:  # one list far longer than a CTA's shared-memory sort, several empty lists
        assign = np.where(rng.random(n) < 0.4, 7, rng.integers(10, nc, n)).astype(np.uint32)
    else:
        assign = rng.integers(0, nc, n).astype(np.uint32)
    doclens = []
    left = n
    while left > 0:
        d = int(min(left, rng.integers(8, 180)))
        doclens.append(d)
        left -= d
    doclens = np.array(doclens, np.int64)
    codes = rng.integers(0, 256, (n, 16), dtype=np.uint8)
    f1 = rng.standard_normal(n).astype(np.float32)
    pos, inv, c1, ff, docs, t2p, status = _run(assign, nc, doclens, codes, f1)
    assert status == 0
    opos, oinv = O.cluster_order(assign, nc)
    np.testing.assert_array_equal(pos, opos)
    np.testing.assert_array_equal(inv, oinv)
    owner = np.repeat(np.arange(len(doclens)), doclens).astype(np.int32)
    np.testing.assert_array_equal(c1, codes[oinv])
    np.testing.assert_array_equal(ff.view(np.uint32), f1[oinv].view(np.uint32))
    np.testing.assert_array_equal(docs, owner[oinv])
    want_t2p = np.empty(n, np.uint32)
    want_t2p[oinv] = np.arange(n, dtype=np.uint32)
    np.testing.assert_array_equal(t2p, want_t2p)
    if skew:
        assert (opos[1:] - opos[:-1]).max() > 4096 and ((opos[1:] - opos[:-1]) == 0).any()


def test_cluster_order_flags_out_of_range_assignment():
    n, nc = 1000, 16
    assign = np.arange(n, dtype=np.uint32) % nc
    assign[17] = nc + 3
    *_, status = _run(assign, nc, np.array([n], np.int64), np.zeros((n, 16), np.uint8), np.zeros(n, np.float32))
    assert status & 1
