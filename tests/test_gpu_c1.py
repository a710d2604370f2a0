"""GPU parity on BASELINE configs[0] (C1: 10,000 documents, about 640k tokens,
4,096 clusters, ex_bits 4, nprobe 32, k_refine 1000, k_full_bit 100, k 100,
seed 0, all 64 queries).

The index is built on the GPU (capi.build_index); a sample of its tokens is
checked against the oracle's encoder and exact assignment.  Then every query
goes through every stage of the CUDA path, called through the C ABI with the
choices chm_search makes (tensor-core probe, tensor-core 1-bit and full-bit
refinement for a batch of 16 or more), and through chm_search itself; each
stage's output is compared bit for bit with the CPU oracle's search of the
same index (oracle/chimera_oracle.c, which restates search_impl.cu:72-574 and
kernels.cu:117-617).  Recall@100 against brute-force fp32 MaxSim is checked
to be the same for both."""
import ctypes as C

import numpy as np
import pytest

from chimera_b200 import capi, workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def S():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def c1():
    cfg = W.CONFIGS["c1"]
    emb, dl, qs = W.generate_numpy(cfg, 0)
    demb = torch.from_numpy(emb).cuda()
    index, aux = capi.build_index(demb, dl, cfg.n_clusters, cfg.ex_bits)
    torch.cuda.synchronize()
    host = O.Index(**index.to_host())
    flips = index.flips.cpu().numpy()
    qrot = O.rotate(flips, qs.reshape(-1, cfg.dim)).reshape(qs.shape[0], 32, 128)
    cb1, cbex = O.query_state(qrot, cfg.ex_bits)
    labels = O.probe(qrot.reshape(-1, 128), index.centroids.cpu().numpy(), index.centroid_norms.cpu().numpy(),
                     cfg.nprobe).reshape(qs.shape[0], 32, cfg.nprobe)
    oracle = [host.search_one(qrot[q], cb1[q], cbex[q], labels[q], cfg.nprobe, cfg.k_refine, cfg.k_full_bit,
                              cfg.num_chunks, cfg.k) for q in range(qs.shape[0])]
    return dict(cfg=cfg, emb=emb, dl=dl, qs=qs, index=index, aux=aux, host=host, qrot=qrot, cb1=cb1, cbex=cbex,
                labels=labels, oracle=oracle)


def test_c1_build_sample_matches_oracle(c1):
    """Encoder output for the first 20,000 tokens and the exact nearest
    centroid of 4,000 sampled tokens equal the oracle's."""
    cfg, index, aux = c1["cfg"], c1["index"], c1["aux"]
    n = 20000
    rot = O.rotate(index.flips.cpu().numpy(), c1["emb"][:n])
    ocodes1, of1, ofull, off = O.encode(rot, cfg.ex_bits)
    np.testing.assert_array_equal(aux["token_codes1"][:n].cpu().numpy(), ocodes1)
    np.testing.assert_array_equal(bits(aux["token_f1"][:n].cpu().numpy()), bits(of1))
    np.testing.assert_array_equal(index.full_codes[:n].cpu().numpy(), ofull)
    np.testing.assert_array_equal(bits(index.full_factors[:n].cpu().numpy()), bits(off))
    rng = np.random.default_rng(1)
    sel = np.sort(rng.choice(c1["emb"].shape[0], 4000, replace=False))
    ids = capi.sample_centroids(c1["emb"].shape[0], cfg.n_clusters, 42)
    oa = O.assign(np.ascontiguousarray(c1["emb"][sel]), np.ascontiguousarray(c1["emb"][ids]))
    np.testing.assert_array_equal(aux["assign"].cpu().numpy()[sel].astype(np.uint32), oa)


def _stages(c1):
    """Every stage through the C ABI, as chm_search runs them for one batch."""
    cfg, d = c1["cfg"], c1["index"]
    L = capi.lib()
    v = C.byref(d.view)
    q = torch.from_numpy(np.ascontiguousarray(c1["qs"])).cuda()
    B = q.shape[0]
    ntok = B * 32
    rot = torch.empty(ntok, 128, device="cuda")
    cb1 = torch.empty(ntok, device="cuda")
    cbex = torch.empty(ntok, device="cuda")
    lut = torch.empty(ntok, 512, device="cuda")
    capi.check(L.chm_prepare_queries(P(d.flips), d.dim, d.ex_bits, P(q), ntok, P(rot), P(cb1), P(cbex), P(lut),
                                     S()), "prepare")
    labels = torch.empty(ntok, cfg.nprobe, dtype=torch.int32, device="cuda")
    pb = L.chm_probe_tc_workspace_bytes(ntok, d.n_clusters, cfg.nprobe)
    pws = torch.empty(pb, dtype=torch.uint8, device="cuda")
    capi.check(L.chm_probe_tc(P(rot), ntok, P(d.centroids), P(d.centroids_bf16), P(d.centroid_norms),
                              P(d.centroid_norm_max), d.n_clusters, cfg.nprobe, P(labels), P(pws), pb, S()), "probe")
    kr = cfg.k_refine
    rd = torch.empty(B, kr, dtype=torch.int32, device="cuda")
    rp = torch.empty(B, kr, device="cuda")
    nr = torch.empty(B, dtype=torch.int32, device="cuda")
    ncand = torch.empty(B, dtype=torch.int64, device="cuda")
    sb = L.chm_stage1_workspace_bytes(v, B, cfg.nprobe, kr)
    sws = torch.empty(sb, dtype=torch.uint8, device="cuda")
    capi.check(L.chm_stage1(v, B, P(lut), P(cb1), P(labels), cfg.nprobe, kr, P(rd), P(rp), P(nr), P(ncand), P(sws),
                            sb, S()), "stage1")
    tb = L.chm_fullbit_score_tc_workspace_bytes(B, kr)
    tws = torch.empty(tb, dtype=torch.uint8, device="cuda")
    ob = torch.empty(B, kr, device="cuda")
    capi.check(L.chm_refine_1bit_tc(v, B, P(lut), P(cb1), P(rot), P(rd), P(nr), kr, P(ob), P(tws), tb, S()),
               "refine")
    fd = torch.empty(B, kr, dtype=torch.int32, device="cuda")
    nf = torch.empty(B, dtype=torch.int32, device="cuda")
    capi.check(L.chm_select_fullbit(B, P(rd), P(ob), P(nr), kr, cfg.k_full_bit, cfg.num_chunks, P(fd), P(nf), kr,
                                    S()), "select")
    fs = torch.empty(B, kr, device="cuda")
    capi.check(L.chm_fullbit_score_tc(v, B, P(rot), P(cbex), P(fd), P(nf), kr, P(fs), P(tws), tb, S()), "fullbit")
    res = torch.empty(B, cfg.k, dtype=torch.int64, device="cuda")
    nres = torch.empty(B, dtype=torch.int32, device="cuda")
    capi.check(L.chm_final_topk(B, P(fd), P(fs), P(nf), kr, cfg.k, P(res), P(nres), S()), "final")
    torch.cuda.synchronize()
    g = lambda t: t.cpu().numpy()
    return dict(rot=g(rot), cb1=g(cb1), cbex=g(cbex), labels=g(labels).view(np.uint32), rd=g(rd), rp=g(rp),
                nr=g(nr), ncand=g(ncand), ob=g(ob), fd=g(fd), nf=g(nf), fs=g(fs), res=g(res), nres=g(nres))


def test_c1_every_stage_bit_exact(c1):
    cfg = c1["cfg"]
    g = _stages(c1)
    np.testing.assert_array_equal(bits(g["rot"]), bits(c1["qrot"].reshape(-1, 128)))
    np.testing.assert_array_equal(bits(g["cb1"]), bits(c1["cb1"].reshape(-1)))
    np.testing.assert_array_equal(bits(g["cbex"]), bits(c1["cbex"].reshape(-1)))
    np.testing.assert_array_equal(g["labels"], c1["labels"].reshape(-1, cfg.nprobe))
    for q, o in enumerate(c1["oracle"]):
        assert g["ncand"][q] == o["n_candidates"], f"candidates q{q}"
        n = g["nr"][q]
        assert n == o["n_refined"], f"refined count q{q}"
        np.testing.assert_array_equal(g["rd"][q, :n], o["refined_docs"], err_msg=f"refined docs q{q}")
        np.testing.assert_array_equal(bits(g["rp"][q, :n]), bits(o["refined_partial"]), err_msg=f"partial q{q}")
        np.testing.assert_array_equal(bits(g["ob"][q, :n]), bits(o["onebit_scores"]), err_msg=f"1-bit q{q}")
        m = g["nf"][q]
        assert m == len(o["fullbit_docs"]), f"full-bit count q{q}"
        np.testing.assert_array_equal(g["fd"][q, :m], o["fullbit_docs"], err_msg=f"full-bit docs q{q}")
        np.testing.assert_array_equal(bits(g["fs"][q, :m]), bits(o["fullbit_scores"]), err_msg=f"full-bit q{q}")
        assert g["nres"][q] == len(o["result"])
        np.testing.assert_array_equal(g["res"][q, :g["nres"][q]], o["result"], err_msg=f"top-k q{q}")


def test_c1_search_and_recall(c1):
    """chm_search (batches of 16 and of 5 queries: both refinement paths)
    returns the oracle's top-100 for every query; recall@100 is identical."""
    cfg = c1["cfg"]
    q = torch.from_numpy(np.ascontiguousarray(c1["qs"])).cuda()
    for batch in (16, 5):
        s = capi.Searcher(c1["index"], k=cfg.k, batch=batch, **cfg.search_kwargs())
        res, nres = s.search(q)
        res, nres = res.cpu().numpy(), nres.cpu().numpy()
        for i, o in enumerate(c1["oracle"]):
            assert nres[i] == len(o["result"])
            np.testing.assert_array_equal(res[i, :nres[i]], o["result"], err_msg=f"batch {batch} query {i}")
    gt = _ground_truth(c1, cfg.k)
    r_gpu = W.recall_at_k(gt, res, cfg.k)
    r_orc = W.recall_at_k(gt, np.stack([o["result"] for o in c1["oracle"]]), cfg.k)
    assert r_gpu == r_orc
    assert r_gpu > 0.5


def _ground_truth(c1, k):
    """Exact fp32 MaxSim top-k of every query (brute force on the GPU)."""
    emb = torch.from_numpy(c1["emb"]).cuda()
    dl = torch.from_numpy(c1["dl"].astype(np.int64)).cuda()
    owner = torch.repeat_interleave(torch.arange(dl.shape[0], device="cuda"), dl)
    out = []
    for q in c1["qs"]:
        sc = torch.from_numpy(q).cuda() @ emb.T                      # [32, N]
        best = torch.full((sc.shape[0], dl.shape[0]), -float("inf"), device="cuda")
        best.scatter_reduce_(1, owner.unsqueeze(0).expand(sc.shape[0], -1), sc, reduce="amax")
        out.append(torch.topk(best.sum(0), k).indices.cpu().numpy())
    return np.stack(out)
