"""CPU checks: the oracle restatement against the reference's own code
(oracle/_ref), the product's host-side seeded draws against the reference,
and the shape of the synthetic workloads."""
import ctypes as C

import numpy as np
import pytest

from chimera_b200 import capi, workloads as W
from oracle import oracle as O

need_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@need_ref
@pytest.mark.parametrize("dim", [128, 96, 64, 100])
def test_rotation_matches_reference(dim):
    rng = np.random.default_rng(dim)
    R = O.RefRotator(dim, 42)
    x = rng.standard_normal((500, dim)).astype(np.float32)
    np.testing.assert_array_equal(O.rotate(R.flips(), x).view(np.uint32), R.rotate(x).view(np.uint32))


@need_ref
@pytest.mark.parametrize("ex_bits", [1, 2, 3, 4, 5, 6, 7])
def test_encoder_matches_reference(ex_bits):
    rng = np.random.default_rng(ex_bits)
    x = rng.standard_normal((600, 128)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    rot = O.RefRotator(128, 42).rotate(x)
    a, b = O.ref_encode(rot, ex_bits), O.encode(rot, ex_bits)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    np.testing.assert_array_equal(a[2], b[2])
    np.testing.assert_array_equal(a[3].view(np.uint32), b[3].view(np.uint32))


@need_ref
@pytest.mark.parametrize("bits", range(1, 9))
def test_pack_unpack_matches_reference(bits):
    rng = np.random.default_rng(bits)
    for _ in range(50):
        raw = rng.integers(0, 1 << bits, 128).astype(np.uint8)
        p_ref = np.zeros(128 * bits // 8, np.uint8)
        O.ref().cref_pack(raw, p_ref, 128, bits)
        np.testing.assert_array_equal(O.pack(raw, bits), p_ref)
        u = np.zeros(128, np.float32)
        O.ref().cref_unpack(p_ref, u, 128, bits)
        np.testing.assert_array_equal(u.astype(np.uint8), raw)
        np.testing.assert_array_equal(O.unpack(p_ref, bits), raw)


@need_ref
def test_query_state_matches_reference():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((200, 128)).astype(np.float32)
    for ex in (1, 4, 7):
        cb1, cbex = O.query_state(x, ex)
        for i in range(len(x)):
            r1, r2 = O.ref_query_state(x[i], ex)
            assert np.float32(r1) == cb1[i] and np.float32(r2) == cbex[i]


@need_ref
@pytest.mark.parametrize("ex_bits", [2, 4])
def test_fullbit_scores_match_reference_scorer(ex_bits):
    from tests import _corpus
    c = _corpus.corpus("mini", ex_bits=ex_bits)
    for q in range(c["qrot"].shape[0]):
        o = _corpus.oracle_search(c, q)
        docs = o["fullbit_docs"].astype(np.int32)
        out = np.zeros(len(docs), np.float32)
        O.ref().cref_fullbit_doc_scores(np.ascontiguousarray(c["qrot"][q]), np.ascontiguousarray(c["cbex"][q]),
                                        c["full"], c["ff"], c["ptr"], docs, len(docs), ex_bits, out, 1)
        np.testing.assert_array_equal(out.view(np.uint32), o["fullbit_scores"].view(np.uint32))


@need_ref
def test_host_rng_matches_reference():
    np.testing.assert_array_equal(capi.fhtkac_flips(42), O.RefRotator(128, 42).flips())
    ids = np.zeros(257, np.uint64)
    O.ref().cref_sample_centroid_ids.argtypes = [C.c_size_t, C.c_size_t, np.ctypeslib.ndpointer(np.uint64)]
    O.ref().cref_sample_centroid_ids(100003, 257, ids)
    np.testing.assert_array_equal(capi.sample_centroids(100003, 257), ids.astype(np.int64))


def test_workload_shapes_and_determinism():
    cfg = W.CONFIGS["mini"]
    a = W.generate_numpy(cfg, 0)
    b = W.generate_numpy(cfg, 0)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
    emb, dl, qs = a
    assert emb.shape == (int(dl.sum()), 128) and qs.shape == (cfg.num_queries, 32, 128)
    assert dl.min() >= 8 and dl.max() <= 180
    np.testing.assert_allclose(np.linalg.norm(emb, axis=1), 1.0, rtol=1e-5)


def test_oracle_pipeline_recall_and_invariants():
    from tests import _corpus
    c = _corpus.corpus("mini")
    cfg = c["cfg"]
    results = []
    for q in range(c["qrot"].shape[0]):
        o = _corpus.oracle_search(c, q)
        assert o["n_refined"] == min(cfg.k_refine, o["n_candidates"])
        p = o["refined_partial"]
        assert np.all(p[:-1] >= p[1:])                       # descending partial scores
        assert len(set(o["refined_docs"])) == len(o["refined_docs"])
        assert set(o["result"]) <= set(o["fullbit_docs"])
        results.append(o["result"])
    gt = W.maxsim_ground_truth_numpy(c["emb"], c["doclens"], c["queries"], cfg.k)
    assert W.recall_at_k(gt, results, cfg.k) > 0.8
