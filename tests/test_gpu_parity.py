"""GPU parity: every stage of the CUDA search path, called through the C ABI,
against the CPU oracle on the same seeded inputs.

Integer / index outputs (probe labels, candidate counts, refined doc ids and
their order, full-bit selections, final top-k) must match exactly.  The
floating-point scores are reproduced in the reference's operation order, so
they are also compared bit-for-bit (the north-star tolerance for MaxSim
scores is 1e-3 relative; these tests hold the stricter bar)."""
import ctypes as C

import numpy as np
import pytest

from chimera_b200 import capi
from oracle import oracle as O
from tests import _corpus

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def T(a, dtype=None):
    """Device copy of a host array.  Bind the result to a name before taking
    its pointer: a temporary can be recycled by torch's allocator before an
    asynchronous kernel reads it."""
    return torch.from_numpy(np.ascontiguousarray(a if dtype is None else a.astype(dtype))).cuda()


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def S():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def small():
    return _corpus.corpus("small")


@pytest.fixture(scope="module")
def dsmall(small):
    return _corpus.device_index(small, torch)


def test_prepare_queries_bit_exact(small):
    c = small
    q = T(c["queries"], np.float32)
    ntok = q.shape[0] * 32
    rot = torch.empty(ntok, 128, device="cuda")
    cb1 = torch.empty(ntok, device="cuda")
    cbex = torch.empty(ntok, device="cuda")
    lut = torch.empty(ntok, 512, device="cuda")
    flips = T(c["flips"])
    capi.check(capi.lib().chm_prepare_queries(P(flips), c["dim"], c["cfg"].ex_bits, P(q), ntok, P(rot),
                                              P(cb1), P(cbex), P(lut), S()), "prepare")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(rot.cpu().numpy()), bits(c["qrot"].reshape(-1, 128)))
    np.testing.assert_array_equal(bits(cb1.cpu().numpy()), bits(c["cb1"].reshape(-1)))
    np.testing.assert_array_equal(bits(cbex.cpu().numpy()), bits(c["cbex"].reshape(-1)))
    ref_lut = O.build_lut(c["qrot"].reshape(-1, 128))
    np.testing.assert_array_equal(bits(lut.cpu().numpy()), bits(ref_lut))


def test_probe_labels_exact(small, dsmall):
    c = small
    rows = c["qrot"].reshape(-1, 128)
    nprobe = c["cfg"].nprobe
    labels = torch.empty(rows.shape[0], nprobe, dtype=torch.int32, device="cuda")
    L = capi.lib()
    nb = L.chm_probe_workspace_bytes(rows.shape[0], dsmall.n_clusters, nprobe)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    rows_d = T(rows)
    capi.check(L.chm_probe(P(rows_d), rows.shape[0], P(dsmall.centroids), P(dsmall.centroid_norms),
                           dsmall.n_clusters, nprobe, P(labels), P(ws), nb, S()), "probe")
    got = labels.cpu().numpy().view(np.uint32)
    np.testing.assert_array_equal(got, c["labels"].reshape(rows.shape[0], nprobe))


def _stage1(c, d, nprobe=None, k_refine=None, labels=None):
    cfg = c["cfg"]
    nprobe = nprobe or cfg.nprobe
    k_refine = k_refine or cfg.k_refine
    nq = c["qrot"].shape[0]
    if labels is None:
        labels = c["labels"]
    lut = T(O.build_lut(c["qrot"].reshape(-1, 128)))
    cb1 = T(c["cb1"].reshape(-1))
    lab = T(labels.astype(np.uint32).view(np.int32))
    rd = torch.empty(nq, k_refine, dtype=torch.int32, device="cuda")
    rp = torch.empty(nq, k_refine, dtype=torch.float32, device="cuda")
    nr = torch.empty(nq, dtype=torch.int32, device="cuda")
    ncand = torch.empty(nq, dtype=torch.int64, device="cuda")
    L = capi.lib()
    nb = L.chm_stage1_workspace_bytes(C.byref(d.view), nq, nprobe, k_refine)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    capi.check(L.chm_stage1(C.byref(d.view), nq, P(lut), P(cb1), P(lab), nprobe, k_refine, P(rd), P(rp),
                            P(nr), P(ncand), P(ws), nb, S()), "stage1")
    torch.cuda.synchronize()
    return lut, cb1, rd, rp, nr, ncand


def test_stage1_candidates_and_refined_order(small, dsmall):
    c = small
    _, _, rd, rp, nr, ncand = _stage1(c, dsmall)
    rd, rp, nr, ncand = rd.cpu().numpy(), rp.cpu().numpy(), nr.cpu().numpy(), ncand.cpu().numpy()
    for q in range(c["qrot"].shape[0]):
        o = _corpus.oracle_search(c, q)
        assert ncand[q] == o["n_candidates"], q
        assert nr[q] == o["n_refined"], q
        np.testing.assert_array_equal(rd[q, :nr[q]], o["refined_docs"], err_msg=f"query {q}")
        np.testing.assert_array_equal(bits(rp[q, :nr[q]]), bits(o["refined_partial"]), err_msg=f"query {q}")


def test_stage1_zero_score_fill(small, dsmall):
    """Fewer positive candidates than k_refine: zero-score candidates fill the
    refined list in ascending doc order (the reference's bitmap order)."""
    c = small
    nprobe, k_refine = 1, 2048
    labels = O.probe(c["qrot"].reshape(-1, 128), c["centroids_rot"], c["cnorm"], nprobe)
    labels = labels.reshape(-1, 32, nprobe)
    _, _, rd, rp, nr, ncand = _stage1(c, dsmall, nprobe=nprobe, k_refine=k_refine, labels=labels)
    rd, rp, nr, ncand = rd.cpu().numpy(), rp.cpu().numpy(), nr.cpu().numpy(), ncand.cpu().numpy()
    saw_zero = False
    for q in range(c["qrot"].shape[0]):
        o = c["index"].search_one(c["qrot"][q], c["cb1"][q], c["cbex"][q], labels[q], nprobe, k_refine, 100, 5, 10)
        assert ncand[q] == o["n_candidates"]
        assert nr[q] == o["n_refined"]
        np.testing.assert_array_equal(rd[q, :nr[q]], o["refined_docs"])
        np.testing.assert_array_equal(bits(rp[q, :nr[q]]), bits(o["refined_partial"]))
        saw_zero |= bool((o["refined_partial"] == 0).any())
    assert saw_zero, "fixture should exercise zero-score candidates"


def test_refine_select_fullbit_final(small, dsmall):
    c = small
    cfg = c["cfg"]
    lut, cb1, rd, rp, nr, _ = _stage1(c, dsmall)
    nq = c["qrot"].shape[0]
    L = capi.lib()
    ob = torch.empty(nq, cfg.k_refine, device="cuda")
    capi.check(L.chm_refine_1bit(C.byref(dsmall.view), nq, P(lut), P(cb1), P(rd), P(nr), cfg.k_refine, P(ob), S()),
               "refine")
    fb_cap = cfg.k_refine
    fd = torch.empty(nq, fb_cap, dtype=torch.int32, device="cuda")
    nf = torch.empty(nq, dtype=torch.int32, device="cuda")
    capi.check(L.chm_select_fullbit(nq, P(rd), P(ob), P(nr), cfg.k_refine, cfg.k_full_bit, cfg.num_chunks, P(fd),
                                    P(nf), fb_cap, S()), "select")
    fs = torch.empty(nq, fb_cap, device="cuda")
    rot = T(c["qrot"].reshape(-1, 128))
    cbex = T(c["cbex"].reshape(-1))
    capi.check(L.chm_fullbit_score(C.byref(dsmall.view), nq, P(rot), P(cbex), P(fd), P(nf), fb_cap, P(fs), S()),
               "fullbit")
    res = torch.empty(nq, cfg.k, dtype=torch.int64, device="cuda")
    nres = torch.empty(nq, dtype=torch.int32, device="cuda")
    capi.check(L.chm_final_topk(nq, P(fd), P(fs), P(nf), fb_cap, cfg.k, P(res), P(nres), S()), "final")
    torch.cuda.synchronize()
    ob, fd, nf, fs = ob.cpu().numpy(), fd.cpu().numpy(), nf.cpu().numpy(), fs.cpu().numpy()
    res, nres, nr = res.cpu().numpy(), nres.cpu().numpy(), nr.cpu().numpy()
    for q in range(nq):
        o = _corpus.oracle_search(c, q)
        np.testing.assert_array_equal(bits(ob[q, :nr[q]]), bits(o["onebit_scores"]), err_msg=f"1-bit q{q}")
        assert nf[q] == len(o["fullbit_docs"])
        np.testing.assert_array_equal(fd[q, :nf[q]], o["fullbit_docs"], err_msg=f"selection q{q}")
        np.testing.assert_array_equal(bits(fs[q, :nf[q]]), bits(o["fullbit_scores"]), err_msg=f"full-bit q{q}")
        assert nres[q] == len(o["result"])
        np.testing.assert_array_equal(res[q, :nres[q]], o["result"], err_msg=f"top-k q{q}")


def test_search_end_to_end(small, dsmall):
    c = small
    cfg = c["cfg"]
    s = capi.Searcher(dsmall, k=cfg.k, batch=5, **cfg.search_kwargs())
    res, nres = s.search(T(c["queries"], np.float32))
    res, nres = res.cpu().numpy(), nres.cpu().numpy()
    for q in range(c["queries"].shape[0]):
        o = _corpus.oracle_search(c, q)
        assert nres[q] == len(o["result"])
        np.testing.assert_array_equal(res[q, :nres[q]], o["result"], err_msg=f"query {q}")


@pytest.mark.parametrize("ex_bits,dim", [(1, 128), (2, 128), (4, 96), (7, 128), (3, 64), (5, 128), (6, 128)])
def test_build_encode_bit_exact(ex_bits, dim):
    rng = np.random.default_rng(ex_bits * 100 + dim)
    x = rng.standard_normal((3000, dim)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    flips = capi.fhtkac_flips(42)
    n = x.shape[0]
    fb = 128 * (1 + ex_bits) // 8
    c1 = torch.empty(n, 16, dtype=torch.uint8, device="cuda")
    f1 = torch.empty(n, device="cuda")
    full = torch.empty(n, fb, dtype=torch.uint8, device="cuda")
    ff = torch.empty(n, device="cuda")
    rot = torch.empty(n, 128, device="cuda")
    flips_d, x_d = T(flips), T(x)
    capi.check(capi.lib().chm_build_encode(P(flips_d), P(x_d), n, dim, ex_bits, P(c1), P(f1), P(full), P(ff),
                                           P(rot), S()), "encode")
    torch.cuda.synchronize()
    ref_rot = O.rotate(flips, x)
    np.testing.assert_array_equal(bits(rot.cpu().numpy()), bits(ref_rot))
    oc1, of1, ofull, off = O.encode(ref_rot, ex_bits)
    np.testing.assert_array_equal(c1.cpu().numpy(), oc1)
    np.testing.assert_array_equal(bits(f1.cpu().numpy()), bits(of1))
    np.testing.assert_array_equal(full.cpu().numpy(), ofull)
    np.testing.assert_array_equal(bits(ff.cpu().numpy()), bits(off))


def test_build_index_matches_oracle(small):
    c = small
    emb = T(c["emb"])
    d, extra = capi.build_index(emb, c["doclens"], c["cfg"].n_clusters, c["cfg"].ex_bits)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(extra["assign"].cpu().numpy().view(np.uint32), c["assign"])
    h = d.to_host()
    np.testing.assert_array_equal(h["cluster_pos"], c["cluster_pos"])
    np.testing.assert_array_equal(h["codes1"], c["index"].codes1)
    np.testing.assert_array_equal(bits(h["factor1"]), bits(c["index"].factor1))
    np.testing.assert_array_equal(h["doc_ids"], c["index"].doc_ids)
    np.testing.assert_array_equal(h["tok2pos"], c["tok2pos"])
    np.testing.assert_array_equal(h["full_codes"], c["full"])
    np.testing.assert_array_equal(bits(h["full_factors"]), bits(c["ff"]))
    np.testing.assert_array_equal(bits(d.centroids.cpu().numpy()), bits(c["centroids_rot"]))


def test_merge_topk():
    rng = np.random.default_rng(3)
    nq, shards, k = 4, 3, 10
    scores = rng.standard_normal((shards, nq, k)).astype(np.float32)
    scores[0, 0, 3] = scores[1, 0, 5]  # a tie across shards
    docs = rng.choice(100000, size=(shards, nq, k), replace=False).astype(np.int64)
    counts = np.full((shards, nq), k, np.int32)
    counts[2, 1] = 4
    res = torch.empty(nq, k, dtype=torch.int64, device="cuda")
    rs = torch.empty(nq, k, device="cuda")
    nr = torch.empty(nq, dtype=torch.int32, device="cuda")
    sd, dd, cd = T(scores), T(docs), T(counts)
    capi.check(capi.lib().chm_merge_topk(nq, shards, k, P(sd), P(dd), P(cd), P(res), P(rs), P(nr), S()), "merge")
    torch.cuda.synchronize()
    for q in range(nq):
        pairs = [(scores[s, q, j], docs[s, q, j]) for s in range(shards) for j in range(counts[s, q])]
        pairs.sort(key=lambda p: (-p[0], -p[1]))
        np.testing.assert_array_equal(res[q].cpu().numpy(), [p[1] for p in pairs[:k]])


def test_invalid_arguments_rejected(small, dsmall):
    L = capi.lib()
    bad = capi.SearchParams(dsmall.n_clusters + 1, 100, 10, 5, 10, 4, 0)
    assert L.chm_search_workspace_bytes(C.byref(dsmall.view), C.byref(bad)) == 0
    bad = capi.SearchParams(8, 10, 20, 5, 10, 4, 0)  # k_full_bit > k_refine
    assert L.chm_search_workspace_bytes(C.byref(dsmall.view), C.byref(bad)) == 0
    st = L.chm_probe(None, 1, None, None, 10, 2000, None, None, 0, S())
    assert st == capi.CHM_ERR_INVALID


# ---- tensor-core probe: same labels as the exact contract -------------------
def _probe_pair(rows, cents, nprobe):
    """(tensor-core labels, SIMT labels) for rows/centroids as host arrays."""
    L = capi.lib()
    r = T(rows)
    c = T(cents)
    nc = cents.shape[0]
    cn = torch.empty(nc, device="cuda")
    capi.check(L.chm_row_norms(P(c), nc, P(cn), S()), "norms")
    cb = torch.empty(nc, 128, dtype=torch.bfloat16, device="cuda")
    capi.check(L.chm_to_bf16(P(c), nc * 128, P(cb), S()), "bf16")
    cmax = torch.empty(1, device="cuda")
    capi.check(L.chm_max_value(P(cn), nc, P(cmax), S()), "max")
    out = []
    for tc in (True, False):
        lab = torch.full((rows.shape[0], nprobe), -1, dtype=torch.int32, device="cuda")
        if tc:
            nb = L.chm_probe_tc_workspace_bytes(rows.shape[0], nc, nprobe)
            ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
            capi.check(L.chm_probe_tc(P(r), rows.shape[0], P(c), P(cb), P(cn), P(cmax), nc, nprobe, P(lab), P(ws), nb,
                                      S()), "probe_tc")
        else:
            nb = L.chm_probe_workspace_bytes(rows.shape[0], nc, nprobe)
            ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
            capi.check(L.chm_probe(P(r), rows.shape[0], P(c), P(cn), nc, nprobe, P(lab), P(ws), nb, S()), "probe")
        torch.cuda.synchronize()
        out.append(lab.cpu().numpy().view(np.uint32))
    return out


def test_probe_tensor_core_matches_oracle(small):
    c = small
    rows = c["qrot"].reshape(-1, 128)
    tc, simt = _probe_pair(rows, c["centroids_rot"], c["cfg"].nprobe)
    np.testing.assert_array_equal(tc, c["labels"].reshape(rows.shape[0], -1))
    np.testing.assert_array_equal(simt, tc)


@pytest.mark.parametrize("nc,nprobe", [(65536, 128), (20000, 64), (4096, 300)])
def test_probe_tensor_core_random(nc, nprobe):
    rng = np.random.default_rng(nc + nprobe)
    rows = rng.standard_normal((1000, 128)).astype(np.float32)
    rows /= np.linalg.norm(rows, axis=1, keepdims=True)
    cents = rng.standard_normal((nc, 128)).astype(np.float32)
    cents /= np.linalg.norm(cents, axis=1, keepdims=True)
    tc, simt = _probe_pair(rows, cents, nprobe)
    np.testing.assert_array_equal(tc, simt)


def test_probe_tensor_core_fallback_on_ties():
    """Duplicated centroids make exact ties at the boundary, so the
    certificate cannot hold and rows take the exact fallback."""
    rng = np.random.default_rng(7)
    base = rng.standard_normal((300, 128)).astype(np.float32)
    base /= np.linalg.norm(base, axis=1, keepdims=True)
    cents = np.concatenate([base] * 8)            # every centroid 8 times
    rows = base[:200] + 0.01 * rng.standard_normal((200, 128)).astype(np.float32)
    tc, simt = _probe_pair(rows.astype(np.float32), cents, 20)
    np.testing.assert_array_equal(tc, simt)
    # ties resolve to the lower id: the first copy of the nearest centroid leads
    assert (tc[:, 0] < 300).all()


def test_probe_tensor_core_fallback_every_row():
    """One centroid repeated: every dist ties, no row can be certified, and
    all 300 rows take the exact fallback -- the first 64 in the batched GEMM
    pass, the rest row by row."""
    rng = np.random.default_rng(9)
    one = rng.standard_normal((1, 128)).astype(np.float32)
    one /= np.linalg.norm(one)
    cents = np.repeat(one, 2048, axis=0)
    rows = rng.standard_normal((300, 128)).astype(np.float32)
    tc, simt = _probe_pair(rows, cents, 24)
    np.testing.assert_array_equal(tc, simt)
    np.testing.assert_array_equal(tc, np.tile(np.arange(24, dtype=np.uint32), (300, 1)))


def test_build_assign_tensor_core_fallback_every_row():
    rng = np.random.default_rng(12)
    x = rng.standard_normal((700, 128)).astype(np.float32)
    cents = np.repeat(x[:1], 500, axis=0)          # every row ties on all centroids
    L = capi.lib()
    xd, cd = T(x), T(cents)
    cn = torch.empty(cents.shape[0], device="cuda")
    capi.check(L.chm_row_norms(P(cd), cents.shape[0], P(cn), S()), "norms")
    nb = L.chm_build_assign_workspace_bytes(x.shape[0], cents.shape[0])
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    out = torch.full((x.shape[0],), -1, dtype=torch.int32, device="cuda")
    capi.check(L.chm_build_assign(P(xd), x.shape[0], 128, P(cd), P(cn), cents.shape[0], P(out), P(ws), nb, S()),
               "assign")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), np.zeros(x.shape[0], np.int32))
    np.testing.assert_array_equal(O.assign(x[:50], cents), np.zeros(50, np.uint32))


def test_build_assign_tensor_core_with_duplicate_centroids():
    rng = np.random.default_rng(11)
    x = rng.standard_normal((5000, 128)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    cents = np.concatenate([x[:100]] * 3)          # ties everywhere
    want = O.assign(x, cents)
    L = capi.lib()
    xd, cd = T(x), T(cents)
    cn = torch.empty(cents.shape[0], device="cuda")
    capi.check(L.chm_row_norms(P(cd), cents.shape[0], P(cn), S()), "norms")
    nb = L.chm_build_assign_workspace_bytes(x.shape[0], cents.shape[0])
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    out = torch.empty(x.shape[0], dtype=torch.int32, device="cuda")
    capi.check(L.chm_build_assign(P(xd), x.shape[0], 128, P(cd), P(cn), cents.shape[0], P(out), P(ws), nb, S()),
               "assign")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want)


def test_search_end_to_end_simt_probe(small, dsmall):
    c = small
    cfg = c["cfg"]
    s = capi.Searcher(dsmall.with_probe(False), k=cfg.k, batch=7, **cfg.search_kwargs())
    q = T(c["queries"], np.float32)
    res, nres = s.search(q)
    res, nres = res.cpu().numpy(), nres.cpu().numpy()
    for i in range(c["queries"].shape[0]):
        o = _corpus.oracle_search(c, i)
        np.testing.assert_array_equal(res[i, :nres[i]], o["result"], err_msg=f"query {i}")
