"""The chunked index build (capi.build_index_streamed, for corpora whose raw
embeddings do not fit on the device) gives the same index, array for array,
as the one-shot build over the concatenated rows -- with chunks that split
documents, and for a document shard built with the whole corpus's
centroids."""
import numpy as np
import pytest

from chimera_b200 import capi, workloads as W

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ARRAYS = ("cluster_pos", "codes1", "factor1", "doc_ids", "tok2pos", "doc_ptrs", "full_codes", "full_factors",
          "centroids", "centroid_norms", "codes1_tok", "factor1_tok", "tok_cluster")


def _same(a, b):
    for name in ARRAYS:
        x, y = getattr(a, name), getattr(b, name)
        assert x.dtype == y.dtype and x.shape == y.shape, name
        assert torch.equal(x.view(torch.uint8) if x.dtype.is_floating_point else x,
                           y.view(torch.uint8) if y.dtype.is_floating_point else y), name


@pytest.mark.parametrize("chunk", [997, 4096])
def test_streamed_build_equals_one_shot(chunk):
    cfg = W.CONFIGS["small"]
    sc = W.StreamedCorpus(cfg, seed=1, chunk=chunk)
    emb, dl, _ = W.generate_torch(cfg, seed=1, chunk=chunk)
    dl = dl.cpu().numpy()
    one, _ = capi.build_index(emb, dl, cfg.n_clusters, cfg.ex_bits)
    ids = torch.from_numpy(capi.sample_centroids(sc.n, cfg.n_clusters, 42)).cuda()
    got, _ = capi.build_index_streamed(lambda: sc.chunks(), sc.n, cfg.dim, dl, cfg.n_clusters, cfg.ex_bits,
                                       sc.gather(ids))
    torch.cuda.synchronize()
    _same(got, one)


def test_streamed_shard_build_equals_one_shot():
    cfg = W.CONFIGS["small"]
    chunk = 1500
    sc = W.StreamedCorpus(cfg, seed=2, chunk=chunk)
    emb, dl, _ = W.generate_torch(cfg, seed=2, chunk=chunk)
    dl = dl.cpu().numpy()
    ptr = np.concatenate([[0], np.cumsum(dl)])
    lo, hi = 700, 1400
    t_lo, t_hi = int(ptr[lo]), int(ptr[hi])
    ids = torch.from_numpy(capi.sample_centroids(sc.n, cfg.n_clusters, 42)).cuda()
    cents = sc.gather(ids)
    assert torch.equal(cents, emb[ids])
    one, _ = capi.build_index(emb[t_lo:t_hi].contiguous(), dl[lo:hi], cfg.n_clusters, cfg.ex_bits, centroids=cents)
    got, _ = capi.build_index_streamed(lambda: ((s - t_lo, e - t_lo, x) for s, e, x in sc.chunks(t_lo, t_hi)),
                                       t_hi - t_lo, cfg.dim, dl[lo:hi], cfg.n_clusters, cfg.ex_bits, cents)
    torch.cuda.synchronize()
    _same(got, one)
