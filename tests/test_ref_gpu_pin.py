"""Pins the oracle's restatement of the GPU stages to the reference itself:
the reference's own kernels (kernels.cu, built into oracle/_ref by
oracle/Makefile and launched as search_impl.cu:72-420 launches them) and the
plain-C oracle run on the same index, rotated queries and probe lists.

Checked bit for bit: the one-bit LUT (kernels.cu:402-428), the candidate
count (mark/count/scan, kernels.cu:117-278), the stably sorted refined list
with its partial scores (partial_score + sum_partial_scores + radix sort,
kernels.cu:175-400, search_impl.cu:245-261) and the chunked 1-bit document
scores (kernels.cu:430-575).  The GPU parity tests then compare the CUDA path
with the same oracle.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests._corpus import corpus

pytestmark = pytest.mark.gpu


def _need_ref_gpu():
    if not O.ref_gpu_available():
        pytest.skip("oracle/_ref/libchimera_ref_gpu.so not built (needs the reference tree at build time)")


def _compare(c, q, nprobe, k_refine, num_chunks):
    labels = c["labels"][q]
    if nprobe != c["cfg"].nprobe:
        labels = O.probe(c["qrot"][q], c["centroids_rot"], c["cnorm"], nprobe)
    ref = O.ref_gpu_query_stages(c["index"], c["qrot"][q], c["cb1"][q], labels, nprobe, k_refine, num_chunks)
    orc = c["index"].search_one(c["qrot"][q], c["cb1"][q], c["cbex"][q], labels, nprobe, k_refine,
                                min(k_refine, c["cfg"].k_full_bit), num_chunks, c["cfg"].k)
    lut = O.build_lut(c["qrot"][q])  # [32, 512]
    np.testing.assert_array_equal(ref["lut"].view(np.uint32), lut.view(np.uint32))
    assert ref["n_candidates"] == orc["n_candidates"]
    assert ref["n_refined"] == orc["n_refined"]
    np.testing.assert_array_equal(ref["refined_docs"], orc["refined_docs"])
    np.testing.assert_array_equal(ref["refined_partial"].view(np.uint32), orc["refined_partial"].view(np.uint32))
    np.testing.assert_array_equal(ref["onebit_scores"].view(np.uint32), orc["onebit_scores"].view(np.uint32))
    return ref


@pytest.mark.parametrize("name,queries", [("mini", range(0, 6)), ("small", range(0, 8))])
def test_reference_kernels_match_oracle(name, queries):
    _need_ref_gpu()
    c = corpus(name)
    cfg = c["cfg"]
    for q in queries:
        _compare(c, q, cfg.nprobe, cfg.k_refine, cfg.num_chunks)


@pytest.mark.parametrize("nprobe,k_refine,num_chunks", [(2, 1000, 5), (1, 7, 3), (8, 50, 1), (16, 4096, 7)])
def test_reference_kernels_match_oracle_edges(nprobe, k_refine, num_chunks):
    """Few probed lists (zero-score candidates fill the refined list in
    ascending doc order), k_refine above the candidate count, one chunk and
    more chunks than refined docs."""
    _need_ref_gpu()
    c = corpus("mini")
    for q in range(4):
        r = _compare(c, q, nprobe, k_refine, num_chunks)
        assert r["n_refined"] == min(k_refine, r["n_candidates"])
