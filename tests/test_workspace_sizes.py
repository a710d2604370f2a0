"""Workspace sizing on a machine without a GPU: the *_workspace_bytes calls
only read an index's sizes, so a chm_index with placeholder pointers is
enough.  The k_refine-free size of chm_stage1_ex must cover the size that
chm_stage1 needs at every k_refine, on shards smaller than CHM_MAX_K_REFINE
documents too (the dense-bound pass runs only for k_refine <= num_docs)."""
import ctypes as C

import pytest

from chimera_b200 import capi

POINTERS = ["cluster_pos", "codes1", "factor1", "doc_ids", "tok2pos", "doc_ptrs", "full_codes", "full_factors",
            "centroids", "centroid_norms", "flips", "centroids_bf16", "centroid_norm_max", "codes1_tok",
            "factor1_tok", "tok_cluster"]


def fake_index(n_tokens, num_docs, n_clusters, max_list_len, max_doc_len, ex_bits=4):
    ix = capi.ChmIndex()
    ix.n_tokens, ix.num_docs, ix.n_clusters = n_tokens, num_docs, n_clusters
    ix.ex_bits, ix.dim, ix.max_list_len, ix.max_doc_len = ex_bits, 128, max_list_len, max_doc_len
    for f in POINTERS:
        setattr(ix, f, 4096)
    return ix


@pytest.mark.parametrize("num_docs", [300, 1000, 2000, 20000])
def test_stage1_ex_size_covers_every_k_refine(num_docs):
    L = capi.lib()
    ix = fake_index(num_docs * 64, num_docs, 512, 400, 180)
    nq, nprobe = 24, 16
    ex = L.chm_stage1_ex_workspace_bytes(C.byref(ix), nq, nprobe, 0)
    assert ex > 0
    for k_refine in (1, 64, 299, 300, 999, 1000, 1999, 2000, 2048, 8192):
        need = L.chm_stage1_workspace_bytes(C.byref(ix), nq, nprobe, k_refine)
        assert need <= ex, (k_refine, need, ex)


def test_search_workspace_grows_with_batch():
    L = capi.lib()
    ix = fake_index(64_000_000, 1_000_000, 262_144, 2000, 180)
    sizes = []
    for b in (1, 128, 1024):
        p = capi.SearchParams(128, 3000, 300, 5, 100, b, 0)
        sizes.append(L.chm_search_workspace_bytes(C.byref(ix), C.byref(p)))
    assert 0 < sizes[0] < sizes[1] < sizes[2]
