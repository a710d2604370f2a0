"""Test infrastructure only: ctypes bindings to the CPU checkers.

* ``liboracle.so``  -- plain-C restatement of the Chimera search path
  (oracle/chimera_oracle.c), the parity checker for the CUDA kernels.
* ``_ref/libchimera_ref.so`` -- the reference's own CPU code (rotator, RaBitQ
  encoder, packer, AVX-512 full-bit scorer) compiled from the reference
  sources by oracle/Makefile.  Used to pin the restatement and to generate
  golden fixtures; absent on machines without the reference tree unless a
  prebuilt copy travelled with the repository.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module.  The product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libchimera_ref.so")
REF_GPU_SO = os.path.join(HERE, "_ref", "libchimera_ref_gpu.so")
DIM = 128
QLEN = 32

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")


def reference_tree():
    """The reference source tree used to build ``_ref``: the directory named by
    $CHIMERA_REFERENCE, else a ``reference`` directory beside the repository
    root; None when neither holds the reference's ``cpp/`` sources."""
    cands = [os.environ.get("CHIMERA_REFERENCE", ""),
             os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "cpp")):
            return os.path.abspath(c)
    return None


def build(ref: bool = True) -> None:
    """Compile liboracle.so, and ``_ref`` from the reference tree when one is
    found (``reference_tree``); without it a prebuilt ``_ref`` is kept."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    tree = reference_tree() if ref else None
    if tree:
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF=" + tree], check=True)


class _Index(C.Structure):
    _fields_ = [
        ("n_tokens", C.c_int64), ("num_docs", C.c_int64), ("n_clusters", C.c_int64),
        ("ex_bits", C.c_int32),
        ("cluster_pos", C.c_void_p), ("codes1", C.c_void_p), ("factor1", C.c_void_p),
        ("doc_ids", C.c_void_p), ("tok2pos", C.c_void_p), ("doc_ptrs", C.c_void_p),
        ("full_codes", C.c_void_p), ("full_factors", C.c_void_p),
    ]


class _Params(C.Structure):
    _fields_ = [("nprobe", C.c_int32), ("k_refine", C.c_int32), ("k_full_bit", C.c_int32),
                ("num_chunks", C.c_int32), ("k", C.c_int32)]


class _Trace(C.Structure):
    _fields_ = [
        ("n_candidates", C.c_int64), ("n_refined", C.c_int32),
        ("refined_docs", C.c_void_p), ("refined_partial", C.c_void_p),
        ("onebit_scores", C.c_void_p), ("fullbit_cap", C.c_int32), ("n_fullbit", C.c_int32),
        ("fullbit_docs", C.c_void_p), ("fullbit_scores", C.c_void_p),
        ("n_result", C.c_int32), ("result", C.c_void_p),
    ]


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        L = C.CDLL(ORACLE_SO)
        L.orc_rotate.argtypes = [_u8p, _f32p, C.c_int, _f32p]
        L.orc_query_state.argtypes = [_f32p, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float)]
        L.orc_build_lut.argtypes = [_f32p, _f32p]
        L.orc_probe.argtypes = [_f32p, C.c_int64, _f32p, _f32p, C.c_int64, C.c_int, _u32p, C.c_int]
        L.orc_dot128.argtypes = [_f32p, _f32p]
        L.orc_dot128.restype = C.c_float
        L.orc_search_one.argtypes = [C.POINTER(_Index), _f32p, _f32p, _f32p, _u32p,
                                     C.POINTER(_Params), C.POINTER(_Trace)]
        L.orc_search_batch.argtypes = [C.POINTER(_Index), _f32p, _f32p, _f32p, _u32p, C.c_int64,
                                       C.POINTER(_Params), _i64p, _i32p, C.c_int]
        L.orc_fullbit_doc_score.argtypes = [C.POINTER(_Index), _f32p, _f32p, C.c_int64]
        L.orc_fullbit_doc_score.restype = C.c_float
        L.orc_onebit_doc_score.argtypes = [C.POINTER(_Index), _f32p, _f32p, C.c_int64]
        L.orc_onebit_doc_score.restype = C.c_float
        L.orc_pack.argtypes = [_u8p, _u8p, C.c_int, C.c_int]
        L.orc_unpack.argtypes = [_u8p, _u8p, C.c_int, C.c_int]
        L.orc_best_rescale_factor.argtypes = [_f32p, C.c_int, C.c_int]
        L.orc_best_rescale_factor.restype = C.c_double
        L.orc_encode.argtypes = [_f32p, C.c_int, C.c_int, _u8p, C.POINTER(C.c_float), _u8p,
                                 C.POINTER(C.c_float)]
        L.orc_assign.argtypes = [_f32p, C.c_int64, C.c_int, _f32p, _f32p, C.c_int64, _u32p, C.c_int]
        L.orc_cluster_order.argtypes = [_u32p, C.c_int64, C.c_int64, _i64p, _u32p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own CPU code (oracle/_ref)."""
    global _ref
    if _ref is None:
        R = C.CDLL(REF_SO)
        R.cref_rotator_create.argtypes = [C.c_size_t, C.c_size_t, C.c_uint64]
        R.cref_rotator_create.restype = C.c_void_p
        R.cref_rotator_destroy.argtypes = [C.c_void_p]
        R.cref_rotator_flips.argtypes = [C.c_void_p, _u8p, C.c_size_t]
        R.cref_rotate.argtypes = [C.c_void_p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t]
        R.cref_encode.argtypes = [_f32p, C.c_size_t, C.c_size_t, C.c_size_t, _u64p, _f32p, _u8p, _f32p]
        R.cref_best_rescale_factor.argtypes = [_f32p, C.c_size_t, C.c_size_t]
        R.cref_best_rescale_factor.restype = C.c_double
        R.cref_quantize_ex.argtypes = [_f32p, _u8p, C.c_size_t, C.c_size_t]
        R.cref_pack.argtypes = [_u8p, _u8p, C.c_size_t, C.c_size_t]
        R.cref_unpack.argtypes = [_u8p, _f32p, C.c_size_t, C.c_size_t]
        R.cref_gemv_batch8.argtypes = [_f32p, _f32p, _f32p, C.c_size_t, C.c_size_t]
        R.cref_fullbit_doc_scores.argtypes = [_f32p, _f32p, _u8p, _f32p, _i64p, _i32p, C.c_int,
                                              C.c_size_t, _f32p, C.c_int]
        R.cref_query_state.argtypes = [_f32p, C.c_size_t, C.c_size_t, C.POINTER(C.c_float),
                                       C.POINTER(C.c_float)]
        _ref = R
    return _ref


_ref_gpu = None


def ref_gpu_available() -> bool:
    return os.path.exists(REF_GPU_SO)


def ref_gpu():
    """The reference's own CUDA kernels (oracle/_ref), driven as search_impl.cu
    drives them; needs a GPU."""
    global _ref_gpu
    if _ref_gpu is None:
        R = C.CDLL(REF_GPU_SO)
        R.cref_gpu_query_stages.argtypes = [
            _f32p, _f32p, _u32p, C.c_int, _u8p, _f32p, _i32p, C.c_int64, _u64p, C.c_int64, _i32p, _u32p,
            C.c_int64, C.c_int, C.c_int, _f32p, C.POINTER(C.c_int64), _i32p, _f32p, C.POINTER(C.c_int32),
            _f32p, C.c_char_p, C.c_int]
        R.cref_gpu_query_stages.restype = C.c_int
        _ref_gpu = R
    return _ref_gpu


def ref_gpu_query_stages(index, rot_q, cb1, labels, nprobe, k_refine, num_chunks):
    """Runs the reference kernels for one query: LUT, candidate set, sorted
    partial scores (refined prefix) and 1-bit document scores."""
    lut = np.zeros((32, 512), np.float32)
    ncand = C.c_int64(0)
    nref = C.c_int32(0)
    rd = np.zeros(k_refine, np.int32)
    rp = np.zeros(k_refine, np.float32)
    ob = np.zeros(k_refine, np.float32)
    err = C.create_string_buffer(512)
    n_tokens = index.factor1.shape[0]
    rc = ref_gpu().cref_gpu_query_stages(
        np.ascontiguousarray(rot_q, np.float32), np.ascontiguousarray(cb1, np.float32),
        np.ascontiguousarray(labels, np.uint32), nprobe, index.codes1.reshape(-1), index.factor1,
        index.doc_ids, n_tokens, index.cluster_pos.astype(np.uint64), index.cluster_pos.shape[0] - 1,
        index.doc_ptrs.astype(np.int32), index.tok2pos, index.doc_ptrs.shape[0] - 1, k_refine, num_chunks,
        lut, C.byref(ncand), rd, rp, C.byref(nref), ob, err, 512)
    if rc != 0:
        raise RuntimeError(f"reference kernels failed ({rc}): {err.value.decode()}")
    R = nref.value
    return dict(lut=lut, n_candidates=ncand.value, n_refined=R, refined_docs=rd[:R].copy(),
                refined_partial=rp[:R].copy(), onebit_scores=ob[:R].copy())


REF_SEARCH_SO = os.path.join(HERE, "_ref", "libchimera_ref_search.so")
_ref_search = None


def ref_search_available() -> bool:
    return os.path.exists(REF_SEARCH_SO)


def ref_search_lib():
    global _ref_search
    if _ref_search is None:
        ref()  # libchimera_ref.so first (the session links against it)
        R = C.CDLL(REF_SEARCH_SO)
        R.cref_session_create.argtypes = [
            _u8p, _f32p, _i32p, C.c_int64, _u64p, C.c_int64, _i64p, C.c_int64, _u32p, _u8p, _f32p, C.c_int,
            C.c_int, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int]
        R.cref_session_create.restype = C.c_void_p
        R.cref_session_destroy.argtypes = [C.c_void_p]
        R.cref_session_search.argtypes = [
            C.c_void_p, _f32p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _i64p,
            C.POINTER(C.c_int), C.POINTER(C.c_int64), C.POINTER(C.c_int), C.c_char_p, C.c_int]
        R.cref_session_search.restype = C.c_int
        _ref_search = R
    return _ref_search


class RefSearchSession:
    """The reference's own search_one (its CUDA kernels, host flow and AVX-512
    full-bit scorer, oracle/ref_search.cu) over a persistent index: one query
    per call, exact-probe shim in place of cuVS CAGRA.  Needs a GPU."""

    def __init__(self, index, centroids_rot, centroid_norms, dim, nprobe_max, k_refine_max, threads=None):
        err = C.create_string_buffer(512)
        self.index = index
        self.dim = dim
        n_tokens = index.factor1.shape[0]
        self.h = ref_search_lib().cref_session_create(
            np.ascontiguousarray(index.codes1.reshape(-1)), index.factor1, index.doc_ids, n_tokens,
            np.ascontiguousarray(index.cluster_pos.astype(np.uint64)), index.cluster_pos.shape[0] - 1,
            np.ascontiguousarray(index.doc_ptrs, dtype=np.int64), index.doc_ptrs.shape[0] - 1,
            np.ascontiguousarray(index.tok2pos.view(np.uint32)), np.ascontiguousarray(index.full_codes.reshape(-1)),
            index.full_factors, int(index.ex_bits), int(dim), np.ascontiguousarray(centroids_rot, np.float32),
            np.ascontiguousarray(centroid_norms, np.float32), int(nprobe_max), int(k_refine_max),
            int(threads or os.cpu_count()), err, 512)
        if not self.h:
            raise RuntimeError(f"reference session: {err.value.decode()}")
        self._err = err

    def search(self, query, nprobe, k_refine, k_full_bit, num_chunks, k, labels=None):
        """query [32, dim] fp32 (host) -> (doc ids best first, n_candidates,
        n_refined).  labels ([32, nprobe] host) replaces the probe shim."""
        out = np.zeros(k, np.int64)
        n = C.c_int(0)
        ncand = C.c_int64(0)
        nref = C.c_int(0)
        lab = None if labels is None else np.ascontiguousarray(labels, np.uint32)
        rc = ref_search_lib().cref_session_search(
            self.h, np.ascontiguousarray(query, np.float32), None if lab is None else lab.ctypes.data, nprobe,
            k_refine, k_full_bit, num_chunks, k, out, C.byref(n), C.byref(ncand), C.byref(nref), self._err, 512)
        if rc != 0:
            raise RuntimeError(f"reference search failed ({rc}): {self._err.value.decode()}")
        return out[:n.value].copy(), ncand.value, nref.value

    def close(self):
        if self.h:
            ref_search_lib().cref_session_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# reference-code helpers
# ---------------------------------------------------------------------------
class RefRotator:
    def __init__(self, dim: int, seed: int = 42):
        self.dim = dim
        self.h = ref().cref_rotator_create(dim, DIM, seed)

    def flips(self) -> np.ndarray:
        out = np.zeros(64, np.uint8)
        n = ref().cref_rotator_flips(self.h, out, 64)
        assert n == 64, n
        return out

    def rotate(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.dim)
        out = np.zeros((x.shape[0], DIM), np.float32)
        ref().cref_rotate(self.h, x, out, x.shape[0], self.dim, DIM)
        return out

    def __del__(self):
        try:
            ref().cref_rotator_destroy(self.h)
        except Exception:
            pass


def ref_encode(rot: np.ndarray, ex_bits: int):
    rot = np.ascontiguousarray(rot, np.float32).reshape(-1, DIM)
    n = rot.shape[0]
    c1 = np.zeros((n, 2), np.uint64)
    f1 = np.zeros(n, np.float32)
    full = np.zeros((n, DIM * (1 + ex_bits) // 8), np.uint8)
    ff = np.zeros(n, np.float32)
    ref().cref_encode(rot, n, DIM, ex_bits, c1, f1, full, ff)
    return c1.view(np.uint8).reshape(n, 16), f1, full, ff


def ref_query_state(rot: np.ndarray, ex_bits: int):
    cb1, cbex = C.c_float(), C.c_float()
    ref().cref_query_state(np.ascontiguousarray(rot, np.float32), DIM, ex_bits, C.byref(cb1),
                           C.byref(cbex))
    return cb1.value, cbex.value


# ---------------------------------------------------------------------------
# oracle helpers
# ---------------------------------------------------------------------------
def rotate(flips: np.ndarray, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    dim = x.shape[-1]
    flat = x.reshape(-1, dim)
    out = np.zeros((flat.shape[0], DIM), np.float32)
    L = lib()
    fl = np.ascontiguousarray(flips, np.uint8)
    for i in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[i])
        o = np.zeros(DIM, np.float32)
        L.orc_rotate(fl, row, dim, o)
        out[i] = o
    return out.reshape(x.shape[:-1] + (DIM,))


def query_state(rot: np.ndarray, ex_bits: int):
    """(cb1, cbex) per rotated query token; rot is [..., 128]."""
    flat = np.ascontiguousarray(rot, np.float32).reshape(-1, DIM)
    cb1 = np.zeros(flat.shape[0], np.float32)
    cbex = np.zeros(flat.shape[0], np.float32)
    L = lib()
    a, b = C.c_float(), C.c_float()
    for i in range(flat.shape[0]):
        L.orc_query_state(np.ascontiguousarray(flat[i]), ex_bits, C.byref(a), C.byref(b))
        cb1[i], cbex[i] = a.value, b.value
    return cb1.reshape(rot.shape[:-1]), cbex.reshape(rot.shape[:-1])


def build_lut(rot: np.ndarray) -> np.ndarray:
    flat = np.ascontiguousarray(rot, np.float32).reshape(-1, DIM)
    out = np.zeros((flat.shape[0], 512), np.float32)
    for i in range(flat.shape[0]):
        o = np.zeros(512, np.float32)
        lib().orc_build_lut(np.ascontiguousarray(flat[i]), o)
        out[i] = o
    return out.reshape(rot.shape[:-1] + (512,))


def dot_norms(c: np.ndarray) -> np.ndarray:
    c = np.ascontiguousarray(c, np.float32).reshape(-1, DIM)
    return np.array([lib().orc_dot128(np.ascontiguousarray(r), np.ascontiguousarray(r)) for r in c],
                    np.float32)


def probe(queries_rot: np.ndarray, centroids_rot: np.ndarray, cnorm: np.ndarray, nprobe: int,
          threads: int = 0) -> np.ndarray:
    q = np.ascontiguousarray(queries_rot, np.float32).reshape(-1, DIM)
    labels = np.zeros((q.shape[0], nprobe), np.uint32)
    lib().orc_probe(q, q.shape[0], np.ascontiguousarray(centroids_rot, np.float32),
                    np.ascontiguousarray(cnorm, np.float32), centroids_rot.shape[0], nprobe,
                    labels, threads or os.cpu_count())
    return labels.reshape(queries_rot.shape[:-1] + (nprobe,))


def pack(raw: np.ndarray, bits: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    out = np.zeros(raw.shape[-1] * bits // 8, np.uint8)
    lib().orc_pack(raw, out, raw.shape[-1], bits)
    return out


def unpack(packed: np.ndarray, bits: int, dim: int = DIM) -> np.ndarray:
    out = np.zeros(dim, np.uint8)
    lib().orc_unpack(np.ascontiguousarray(packed, np.uint8), out, dim, bits)
    return out


def encode(rot: np.ndarray, ex_bits: int):
    rot = np.ascontiguousarray(rot, np.float32).reshape(-1, DIM)
    n = rot.shape[0]
    c1 = np.zeros((n, 16), np.uint8)
    f1 = np.zeros(n, np.float32)
    full = np.zeros((n, DIM * (1 + ex_bits) // 8), np.uint8)
    ff = np.zeros(n, np.float32)
    a, b = C.c_float(), C.c_float()
    L = lib()
    for i in range(n):
        o1 = np.zeros(16, np.uint8)
        of = np.zeros(full.shape[1], np.uint8)
        L.orc_encode(np.ascontiguousarray(rot[i]), DIM, ex_bits, o1, C.byref(a), of, C.byref(b))
        c1[i], f1[i], full[i], ff[i] = o1, a.value, of, b.value
    return c1, f1, full, ff


class Index:
    """Host-side index arrays in the reference layout (see chimera_oracle.h)."""

    def __init__(self, *, cluster_pos, codes1, factor1, doc_ids, tok2pos, doc_ptrs, full_codes,
                 full_factors, ex_bits):
        self.cluster_pos = np.ascontiguousarray(cluster_pos, np.int64)
        self.codes1 = np.ascontiguousarray(codes1, np.uint8)
        self.factor1 = np.ascontiguousarray(factor1, np.float32)
        self.doc_ids = np.ascontiguousarray(doc_ids, np.int32)
        self.tok2pos = np.ascontiguousarray(tok2pos, np.uint32)
        self.doc_ptrs = np.ascontiguousarray(doc_ptrs, np.int64)
        self.full_codes = np.ascontiguousarray(full_codes, np.uint8)
        self.full_factors = np.ascontiguousarray(full_factors, np.float32)
        self.ex_bits = int(ex_bits)
        self._c = _Index(
            self.factor1.shape[0], self.doc_ptrs.shape[0] - 1, self.cluster_pos.shape[0] - 1,
            self.ex_bits,
            self.cluster_pos.ctypes.data, self.codes1.ctypes.data, self.factor1.ctypes.data,
            self.doc_ids.ctypes.data, self.tok2pos.ctypes.data, self.doc_ptrs.ctypes.data,
            self.full_codes.ctypes.data, self.full_factors.ctypes.data)

    def search_one(self, rot_q, cb1, cbex, labels, nprobe, k_refine, k_full_bit, num_chunks, k):
        p = _Params(nprobe, k_refine, k_full_bit, num_chunks, k)
        cap = k_refine
        out = dict(
            refined_docs=np.zeros(k_refine, np.int32), refined_partial=np.zeros(k_refine, np.float32),
            onebit_scores=np.zeros(k_refine, np.float32), fullbit_docs=np.zeros(cap, np.int32),
            fullbit_scores=np.zeros(cap, np.float32), result=np.zeros(k, np.int64))
        tr = _Trace(0, 0, out["refined_docs"].ctypes.data, out["refined_partial"].ctypes.data,
                    out["onebit_scores"].ctypes.data, cap, 0, out["fullbit_docs"].ctypes.data,
                    out["fullbit_scores"].ctypes.data, 0, out["result"].ctypes.data)
        rc = lib().orc_search_one(C.byref(self._c), np.ascontiguousarray(rot_q, np.float32),
                                  np.ascontiguousarray(cb1, np.float32),
                                  np.ascontiguousarray(cbex, np.float32),
                                  np.ascontiguousarray(labels, np.uint32), C.byref(p), C.byref(tr))
        if rc != 0:
            raise RuntimeError(f"oracle search failed: {rc}")
        R, F = tr.n_refined, tr.n_fullbit
        return dict(
            n_candidates=tr.n_candidates, n_refined=R,
            refined_docs=out["refined_docs"][:R].copy(), refined_partial=out["refined_partial"][:R].copy(),
            onebit_scores=out["onebit_scores"][:R].copy(), fullbit_docs=out["fullbit_docs"][:F].copy(),
            fullbit_scores=out["fullbit_scores"][:F].copy(), result=out["result"][:tr.n_result].copy())

    def search_batch(self, rot_q, cb1, cbex, labels, nprobe, k_refine, k_full_bit, num_chunks, k,
                     threads=0):
        nq = rot_q.shape[0]
        p = _Params(nprobe, k_refine, k_full_bit, num_chunks, k)
        res = np.full((nq, k), -1, np.int64)
        nres = np.zeros(nq, np.int32)
        rc = lib().orc_search_batch(C.byref(self._c), np.ascontiguousarray(rot_q, np.float32),
                                    np.ascontiguousarray(cb1, np.float32),
                                    np.ascontiguousarray(cbex, np.float32),
                                    np.ascontiguousarray(labels, np.uint32), nq, C.byref(p), res,
                                    nres, threads or os.cpu_count())
        if rc != 0:
            raise RuntimeError("oracle batch search failed")
        return res, nres

    def onebit_doc_score(self, luts, cb1, doc):
        return lib().orc_onebit_doc_score(C.byref(self._c), np.ascontiguousarray(luts, np.float32).reshape(-1),
                                          np.ascontiguousarray(cb1, np.float32), int(doc))

    def fullbit_doc_score(self, rot_q, cbex, doc):
        return lib().orc_fullbit_doc_score(C.byref(self._c), np.ascontiguousarray(rot_q, np.float32),
                                           np.ascontiguousarray(cbex, np.float32), int(doc))


def assign(x: np.ndarray, centroids: np.ndarray, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    c = np.ascontiguousarray(centroids, np.float32)
    d = x.shape[1]
    cn = _norms_fmaf(c)  # ||c||^2 with the distance dots' sequential fmaf order
    out = np.zeros(x.shape[0], np.uint32)
    lib().orc_assign(x, x.shape[0], d, c, cn, c.shape[0], out, threads or os.cpu_count())
    return out


def _norms_fmaf(c: np.ndarray) -> np.ndarray:
    """Sequential fmaf dot of each row with itself (any width)."""
    d = c.shape[1]
    pad = np.zeros((c.shape[0], DIM), np.float32)
    pad[:, :d] = c
    return dot_norms(pad)


def cluster_order(assign_: np.ndarray, nc: int):
    pos = np.zeros(nc + 1, np.int64)
    inv = np.zeros(assign_.shape[0], np.uint32)
    lib().orc_cluster_order(np.ascontiguousarray(assign_, np.uint32), assign_.shape[0], nc, pos, inv)
    return pos, inv
