"""The reference-facing surfaces: pybind11 module ``chimera`` (build / search
/ save / load), the gpu_build / gpu_search CLIs and their flag handling."""
import os
import struct
import subprocess
import sys

import numpy as np
import pytest

from chimera_b200 import build as B
from tests import _corpus

BIN = B.BIN


def _chimera():
    sys.path.insert(0, B.HERE)
    import chimera  # noqa: E402
    return chimera


def run(args, **kw):
    return subprocess.run(args, capture_output=True, text=True, timeout=600, **kw)


def test_cli_help_and_bad_args():
    for tool in ("gpu_build", "gpu_search"):
        exe = os.path.join(BIN, tool)
        r = run([exe])
        assert r.returncode == 0 and "Usage:" in r.stdout
        r = run([exe, "--help"])
        assert r.returncode == 0 and "Usage:" in r.stdout
        r = run([exe, "--bogus"])
        assert r.returncode == 1 and "Argument error: Unknown argument: --bogus" in r.stderr
    r = run([os.path.join(BIN, "gpu_search"), "--query", "q", "--gt", "g", "--index", "/nonexistent"])
    assert r.returncode == 1 and "--index must point to a Chimera index directory" in r.stderr


def test_module_imports_and_signature():
    chimera = _chimera()
    doc = chimera.ChimeraIndex.build.__doc__
    for kw in ("nprobe", "k_refine", "k_full_bit", "cagra_itopk_size", "num_chunks"):
        assert kw in doc


@pytest.mark.gpu
def test_pybind_build_search_save_load(tmp_path):
    chimera = _chimera()
    c = _corpus.corpus("small")
    cfg = c["cfg"]
    kw = dict(nprobe=cfg.nprobe, k_refine=cfg.k_refine, k_full_bit=cfg.k_full_bit, num_chunks=cfg.num_chunks)
    idx = chimera.ChimeraIndex.build(np.ascontiguousarray(c["emb"]), [int(x) for x in c["doclens"]],
                                     cfg.n_clusters, cfg.ex_bits, **kw)
    one = idx.search(np.ascontiguousarray(c["queries"][0]), k=cfg.k)
    many = idx.search(np.ascontiguousarray(c["queries"]), k=cfg.k)
    for q in range(c["queries"].shape[0]):
        want = list(_corpus.oracle_search(c, q)["result"])
        assert many[q] == want, q
    assert one == many[0]
    idx.save(str(tmp_path / "ix"))
    names = sorted(os.listdir(tmp_path / "ix"))
    assert names == sorted(["doclens.bin", "doc_1bit.bin", "doc_full.bin", "cluster_1bit.bin", "ivf.bin",
                            "centroids.f32"])
    # on-disk payloads equal the oracle-built index arrays
    raw = open(tmp_path / "ix" / "cluster_1bit.bin", "rb").read()
    n = c["emb"].shape[0]
    assert len(raw) == n * 28
    np.testing.assert_array_equal(np.frombuffer(raw[:n * 16], np.uint8).reshape(n, 16), c["index"].codes1)
    np.testing.assert_array_equal(np.frombuffer(raw[n * 20:n * 24], np.int32), c["index"].doc_ids)
    idx2 = chimera.ChimeraIndex.load(str(tmp_path / "ix"), **kw)
    assert idx2.search(np.ascontiguousarray(c["queries"]), k=cfg.k) == many
    with pytest.raises(ValueError):
        idx2.search(np.zeros((31, 128), np.float32), k=10)
    with pytest.raises(ValueError):
        idx2.search(np.ascontiguousarray(c["queries"][0]), k=0)
    with pytest.raises(ValueError):
        chimera.ChimeraIndex.load(str(tmp_path / "ix"), nprobe=cfg.n_clusters + 1)
    with pytest.raises(ValueError):
        chimera.ChimeraIndex.load(str(tmp_path / "ix"), k_refine=10, k_full_bit=20)
    with pytest.raises(RuntimeError):
        chimera.ChimeraIndex.load(str(tmp_path / "missing"))


@pytest.mark.gpu
def test_cli_build_and_search(tmp_path):
    c = _corpus.corpus("mini")
    cfg = c["cfg"]
    emb, dl, qs = c["emb"], c["doclens"], c["queries"]
    with open(tmp_path / "emb.bin", "wb") as f:
        f.write(struct.pack("ii", emb.shape[0], emb.shape[1]))
        f.write(np.ascontiguousarray(emb, np.float32).tobytes())
    with open(tmp_path / "doclens.bin", "wb") as f:
        f.write(struct.pack("i", len(dl)))
        f.write(np.asarray(dl, np.int32).tobytes())
    with open(tmp_path / "q.bin", "wb") as f:
        f.write(struct.pack("iii", qs.shape[0], qs.shape[1], qs.shape[2]))
        f.write(np.ascontiguousarray(qs, np.float32).tobytes())
    res = [list(_corpus.oracle_search(c, q)["result"]) for q in range(qs.shape[0])]
    with open(tmp_path / "gt.tsv", "w") as f:
        for q, r in enumerate(res):
            for rank, doc in enumerate(r):
                f.write(f"{q}\t{doc}\t{rank + 1}\n")
    r = run([os.path.join(BIN, "gpu_build"), "--index", str(tmp_path / "ix"), "--doclens", str(tmp_path / "doclens.bin"),
             "--data", str(tmp_path / "emb.bin"), "--n-clusters", str(cfg.n_clusters), "--ex-bits", str(cfg.ex_bits)])
    assert r.returncode == 0, r.stderr
    r = run([os.path.join(BIN, "gpu_search"), "--query", str(tmp_path / "q.bin"), "--gt", str(tmp_path / "gt.tsv"),
             "--index", str(tmp_path / "ix"), "--k", str(cfg.k), "--nprobe", str(cfg.nprobe), "--k-refine",
             str(cfg.k_refine), "--k-full-bit", str(cfg.k_full_bit), "--num-chunks", str(cfg.num_chunks),
             "--cagra-itopk-size", "64", "--warmup", "2", "--batch", "4"])
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert lines[0].startswith("[SEARCH] latency_ms mean=") and " p99=" in lines[0]
    # results equal the oracle's, so recall against them is exactly 1; the
    # latency line leaves std::cout in fixed 3-digit mode (search.cpp:33)
    assert lines[1] == f"[SEARCH] recall@{cfg.k}=1.000"
    assert any(l.startswith("[SEARCH] batched qps=") for l in lines)


def _reference_layout_files(c):
    """The five index files in the reference's layout (chimera_index::save,
    build_index.cu:503-557; IndexHeader, chimera_index.cuh:75-81), written
    here from the oracle-built arrays of the corpus."""
    cfg = c["cfg"]
    n = c["emb"].shape[0]
    dl = np.asarray(c["doclens"], np.int32)
    ix = c["index"]
    files = {}
    files["doclens.bin"] = struct.pack("<i", len(dl)) + dl.tobytes()
    files["doc_1bit.bin"] = (struct.pack("<5Q", n, c["dim"], cfg.n_clusters, cfg.ex_bits, 128) +
                             np.asarray(c["flips"], np.uint8).tobytes() +
                             np.ascontiguousarray(c["codes1_tok"], np.uint8).tobytes() +
                             np.asarray(c["f1_tok"], np.float32).tobytes() + np.asarray(c["ff"], np.float32).tobytes())
    files["doc_full.bin"] = np.ascontiguousarray(c["full"], np.uint8).tobytes()
    files["cluster_1bit.bin"] = (np.ascontiguousarray(ix.codes1, np.uint8).tobytes() +
                                 np.asarray(ix.factor1, np.float32).tobytes() +
                                 np.asarray(ix.doc_ids, np.int32).tobytes() +
                                 np.asarray(c["tok2pos"], np.uint32).tobytes())
    files["ivf.bin"] = (struct.pack("<Q", n) + np.asarray(c["inv"], np.uint32).tobytes() +
                        np.asarray(c["cluster_pos"], np.uint64).tobytes())
    return files


@pytest.mark.gpu
def test_saved_files_are_the_reference_layout_byte_for_byte(tmp_path):
    """ChimeraIndex.build (assignment, encoding and the IVF reorder on the GPU,
    the index kept on the device) then save(): each of the five
    reference-format files equals, byte for byte, the file the reference's
    layout gives for the oracle-built index of the same corpus."""
    chimera = _chimera()
    c = _corpus.corpus("small")
    cfg = c["cfg"]
    idx = chimera.ChimeraIndex.build(np.ascontiguousarray(c["emb"]), [int(x) for x in c["doclens"]],
                                     cfg.n_clusters, cfg.ex_bits)
    idx.save(str(tmp_path / "ix"))
    for name, want in _reference_layout_files(c).items():
        got = open(tmp_path / "ix" / name, "rb").read()
        assert len(got) == len(want), name
        assert got == want, name


def _write_carga_like(path, centroids, degree=8, seed=0):
    """A file laid out as cuVS serialises a CAGRA index with its dataset: a
    few scalars, the graph as a .npy block (uint32, (n, degree)), a bool,
    then the dataset as a .npy block (fp32, (n, dim))."""
    rng = np.random.default_rng(seed)
    n = centroids.shape[0]
    with open(path, "wb") as f:
        f.write(b"<f4\x00")                                   # dtype string
        f.write(struct.pack("<iqqqi", 4, n, centroids.shape[1], degree, 0))
        np.lib.format.write_array(f, rng.integers(0, n, (n, degree), dtype=np.uint32))
        f.write(b"\x01")                                      # dataset included
        np.lib.format.write_array(f, np.ascontiguousarray(centroids, np.float32))


@pytest.mark.gpu
def test_load_reference_index_with_carga_centroids(tmp_path):
    """An index directory as the reference writes it (centroids.carga, no
    centroids.f32) loads: the rotated centroids come from the CAGRA file's
    dataset block, and the searches equal those of the original index."""
    chimera = _chimera()
    c = _corpus.corpus("mini")
    cfg = c["cfg"]
    kw = dict(nprobe=cfg.nprobe, k_refine=cfg.k_refine, k_full_bit=cfg.k_full_bit, num_chunks=cfg.num_chunks)
    idx = chimera.ChimeraIndex.build(np.ascontiguousarray(c["emb"]), [int(x) for x in c["doclens"]],
                                     cfg.n_clusters, cfg.ex_bits, **kw)
    want = idx.search(np.ascontiguousarray(c["queries"]), k=cfg.k)
    ix = tmp_path / "ix"
    idx.save(str(ix))
    raw = open(ix / "centroids.f32", "rb").read()
    nc, d = struct.unpack("<qq", raw[:16])
    cents = np.frombuffer(raw[16:], np.float32).reshape(nc, d)
    os.remove(ix / "centroids.f32")
    _write_carga_like(ix / "centroids.carga", cents)
    got = chimera.ChimeraIndex.load(str(ix), **kw).search(np.ascontiguousarray(c["queries"]), k=cfg.k)
    assert got == want
    # no dataset block of the right shape: a clear error
    _write_carga_like(ix / "centroids.carga", cents[:, :64][: nc - 1])
    with pytest.raises(RuntimeError):
        chimera.ChimeraIndex.load(str(ix), **kw)
