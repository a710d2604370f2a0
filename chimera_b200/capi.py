"""ctypes binding of the C ABI (include/chimera_b200.h) plus the device-side
index container and the GPU index build used by the Python entry points.

Torch is used only as device-memory / stream plumbing: every computation on
the search path runs in the sm_100a kernels of ``lib/libchimera_b200.so``.
There is no CPU fallback; importing this module without the built library
raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libchimera_b200.so")
CORE_PATH = os.path.join(HERE, "lib", "libchimera_core.so")
HOST_RNG_PATH = os.path.join(HERE, "lib", "libchimera_hostrng.so")

DIM = 128
QLEN = 32

CHM_OK, CHM_ERR_INVALID, CHM_ERR_CAPACITY, CHM_ERR_CUDA, CHM_ERR_TIMEOUT, CHM_ERR_UNSUPPORTED = range(6)
# include/chimera_b200.h: CHM_PROBE_NOALLOC_MAX_ELEMENTS (static scratch of chm_probe_noalloc)
PROBE_NOALLOC_MAX_ELEMENTS = 1 << 22
_STATUS = {1: "invalid argument", 2: "capacity", 3: "CUDA error", 4: "timeout", 5: "unsupported"}


class ChmError(RuntimeError):
    def __init__(self, status, where):
        msg = f"{where}: {_STATUS.get(status, status)}"
        err = _lib_handle.chm_last_error().decode() if _lib_handle is not None else ""
        if status == CHM_ERR_CUDA and err:
            msg += f" ({err})"
        super().__init__(msg)
        self.status = status


class ChmIndex(C.Structure):
    _fields_ = [
        ("n_tokens", C.c_int64), ("num_docs", C.c_int64), ("n_clusters", C.c_int64),
        ("ex_bits", C.c_int32), ("dim", C.c_int32), ("max_list_len", C.c_int32), ("max_doc_len", C.c_int32),
        ("cluster_pos", C.c_void_p), ("codes1", C.c_void_p), ("factor1", C.c_void_p),
        ("doc_ids", C.c_void_p), ("tok2pos", C.c_void_p), ("doc_ptrs", C.c_void_p),
        ("full_codes", C.c_void_p), ("full_factors", C.c_void_p), ("centroids", C.c_void_p),
        ("centroid_norms", C.c_void_p), ("flips", C.c_void_p), ("centroids_bf16", C.c_void_p),
        ("centroid_norm_max", C.c_void_p), ("codes1_tok", C.c_void_p), ("factor1_tok", C.c_void_p),
        ("tok_cluster", C.c_void_p),
    ]


class SearchParams(C.Structure):
    _fields_ = [("nprobe", C.c_int32), ("k_refine", C.c_int32), ("k_full_bit", C.c_int32),
                ("num_chunks", C.c_int32), ("k", C.c_int32), ("batch", C.c_int32),
                ("table_log2_extra", C.c_int32)]


_lib_handle = None
_rng_handle = None
V = C.c_void_p
I64 = C.c_int64
I32 = C.c_int32
SZ = C.c_size_t

EXPORTS = {
    "chm_version": ([], C.c_char_p),
    "chm_last_error": ([], C.c_char_p),
    "chm_search_workspace_bytes": ([V, V], SZ),
    "chm_search": ([V, V, V, I64, V, V, V, SZ, V], C.c_int),
    "chm_prepare_queries": ([V, I32, I32, V, I64, V, V, V, V, V], C.c_int),
    "chm_probe_workspace_bytes": ([I64, I64, I32], SZ),
    "chm_probe": ([V, I64, V, V, I64, I32, V, V, SZ, V], C.c_int),
    "chm_probe_noalloc": ([V, I64, V, V, I64, I32, V, V], C.c_int),
    "chm_stage1_ex_workspace_bytes": ([V, I32, I32, I32], SZ),
    "chm_stage1_ex": ([V, I32, V, V, V, I32, I32, V, V, V, V, I32, V, SZ, V], C.c_int),
    "chm_merge_refined": ([I32, I32, I32, V, V, V, V, V, V, V, V], C.c_int),
    "chm_shard_localize": ([I32, I32, V, V, I64, I64, V, V], C.c_int),
    "chm_stage1_workspace_bytes": ([V, I32, I32, I32], SZ),
    "chm_stage1": ([V, I32, V, V, V, I32, I32, V, V, V, V, V, SZ, V], C.c_int),
    "chm_refine_1bit": ([V, I32, V, V, V, V, I32, V, V], C.c_int),
    "chm_fullbit_score_tc_workspace_bytes": ([I32, I32], SZ),
    "chm_fullbit_score_tc": ([V, I32, V, V, V, V, I32, V, V, SZ, V], C.c_int),
    "chm_refine_1bit_tc_workspace_bytes": ([I32, I32], SZ),
    "chm_refine_tc_workspace_bytes": ([V, I32, I32], SZ),
    "chm_refine_1bit_tc": ([V, I32, V, V, V, V, V, I32, V, V, SZ, V], C.c_int),
    "chm_select_fullbit": ([I32, V, V, V, I32, I32, I32, V, V, I32, V], C.c_int),
    "chm_fullbit_score": ([V, I32, V, V, V, V, I32, V, V], C.c_int),
    "chm_final_topk": ([I32, V, V, V, I32, I32, V, V, V], C.c_int),
    "chm_merge_topk": ([I32, I32, I32, V, V, V, V, V, V, V], C.c_int),
    "chm_build_assign_workspace_bytes": ([I64, I64], SZ),
    "chm_probe_tc_workspace_bytes": ([I64, I64, I32], SZ),
    "chm_probe_tc": ([V, I64, V, V, V, V, I64, I32, V, V, SZ, V], C.c_int),
    "chm_to_bf16": ([V, I64, V, V], C.c_int),
    "chm_max_value": ([V, I64, V, V], C.c_int),
    "chm_build_assign": ([V, I64, I32, V, V, I64, V, V, SZ, V], C.c_int),
    "chm_build_encode": ([V, V, I64, I32, I32, V, V, V, V, V, V], C.c_int),
    "chm_row_norms": ([V, I64, V, V], C.c_int),
    "chm_token_order_1bit": ([V, V, V, I64, V, V, V], C.c_int),
    "chm_token_clusters": ([V, I64, V, I64, V, V], C.c_int),
    "chm_stage1_table_queries": ([V, I32, I32, I32, I32, V, SZ, V, V], C.c_int),
    "chm_build_cluster_order_workspace_bytes": ([I64, I64], SZ),
    "chm_build_cluster_order": ([V, I64, I64, V, I64, V, V, V, V, V, V, V, V, V, V, SZ, V], C.c_int),
}


def lib():
    """The CUDA library; raises if it has not been built."""
    global _lib_handle
    if _lib_handle is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"chimera_b200 CUDA library missing: {LIB_PATH} "
                               "(run `python -m chimera_b200.build`)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in EXPORTS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib_handle = L
    return _lib_handle


NCCL_PATH = os.path.join(HERE, "lib", "libchimera_nccl.so")
_nccl_handle = None
SH_STEPS = ("prepare", "probe", "gather_labels", "stage1", "gather_lists", "merge", "refine_1bit",
            "reduce_onebit", "select_fullbit", "fullbit", "reduce_fullbit", "final_topk")


class ShardInfo(C.Structure):
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("doc_base", C.c_void_p)]


def nccl_lib():
    """The document-sharded search over NCCL (include/chimera_b200_sharded.h)."""
    global _nccl_handle
    if _nccl_handle is None:
        lib()
        if not os.path.exists(NCCL_PATH):
            raise RuntimeError(f"chimera_b200 NCCL library missing: {NCCL_PATH} (run `python -m chimera_b200.build`)")
        L = C.CDLL(NCCL_PATH)
        L.chm_comm_unique_id.argtypes = [V]
        L.chm_comm_unique_id.restype = C.c_int
        L.chm_comm_init.argtypes = [V, I32, I32, I32, C.POINTER(V)]
        L.chm_comm_init.restype = C.c_int
        L.chm_comm_init_all.argtypes = [I32, V, V]
        L.chm_comm_init_all.restype = C.c_int
        L.chm_comm_destroy.argtypes = [V]
        L.chm_comm_destroy.restype = C.c_int
        L.chm_search_sharded_workspace_bytes.argtypes = [V, V, I32]
        L.chm_search_sharded_workspace_bytes.restype = SZ
        L.chm_search_sharded.argtypes = [V, V, V, V, V, I64, V, V, V, SZ, V, V]
        L.chm_search_sharded.restype = C.c_int
        _nccl_handle = L
    return _nccl_handle


def host_rng():
    global _rng_handle
    if _rng_handle is None:
        R = C.CDLL(HOST_RNG_PATH)
        R.chm_host_fhtkac_flips.argtypes = [C.c_uint64, V, SZ]
        R.chm_host_sample_centroids.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, V]
        _rng_handle = R
    return _rng_handle


def check(status, where):
    if status != CHM_OK:
        raise ChmError(status, where)


def fhtkac_flips(seed: int = 42) -> np.ndarray:
    out = np.zeros(64, np.uint8)
    host_rng().chm_host_fhtkac_flips(seed, out.ctypes.data, 64)
    return out


def sample_centroids(num_embeddings: int, n_clusters: int, seed: int = 42) -> np.ndarray:
    ids = np.zeros(n_clusters, np.uint64)
    host_rng().chm_host_sample_centroids(num_embeddings, n_clusters, seed, ids.ctypes.data)
    return ids.astype(np.int64)


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def _stream(torch, stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class DeviceIndex:
    """Device-resident index arrays (torch tensors) + the chm_index view."""

    FIELDS = ("cluster_pos", "codes1", "factor1", "doc_ids", "tok2pos", "doc_ptrs", "full_codes",
              "full_factors", "centroids", "centroid_norms", "flips", "centroids_bf16", "centroid_norm_max",
              "codes1_tok", "factor1_tok", "tok_cluster")

    def __init__(self, *, dim, ex_bits, tensor_core_probe=True, token_order=True, codes1_tok=None,
                 factor1_tok=None, tok_cluster=None, **arrays):
        """`token_order`: keep a token-order copy of the 1-bit codes and
        factors (20 B per token) and every token's cluster (4 B per token),
        given as codes1_tok / factor1_tok / tok_cluster or derived here from
        the cluster-ordered arrays.  Refinement then reads each doc as one
        span, and stage 1 can take its dense-bound path."""
        import torch
        self.torch = torch
        self.dim = int(dim)
        self.ex_bits = int(ex_bits)
        for k in self.FIELDS[:11]:
            setattr(self, k, arrays[k])
        dev = self.centroids.device
        st = _stream(torch)
        self.centroids_bf16 = torch.empty(self.centroids.shape, dtype=torch.bfloat16, device=dev)
        check(lib().chm_to_bf16(_ptr(self.centroids), self.centroids.numel(), _ptr(self.centroids_bf16), st),
              "to_bf16")
        self.centroid_norm_max = torch.empty(1, dtype=torch.float32, device=dev)
        check(lib().chm_max_value(_ptr(self.centroid_norms), self.centroid_norms.numel(),
                                  _ptr(self.centroid_norm_max), st), "max")
        self.n_tokens = int(self.factor1.shape[0])
        self.num_docs = int(self.doc_ptrs.shape[0] - 1)
        self.n_clusters = int(self.cluster_pos.shape[0] - 1)
        lens = self.cluster_pos[1:] - self.cluster_pos[:-1]
        self.max_list_len = int(lens.max().item()) if self.n_clusters else 0
        self.codes1_tok = self.factor1_tok = self.tok_cluster = None
        dl = self.doc_ptrs[1:] - self.doc_ptrs[:-1]
        self.max_doc_len = int(dl.max().item()) if self.num_docs else 0
        if token_order:
            if codes1_tok is None or factor1_tok is None:
                codes1_tok = torch.empty(self.n_tokens, 16, dtype=torch.uint8, device=dev)
                factor1_tok = torch.empty(self.n_tokens, dtype=torch.float32, device=dev)
                check(lib().chm_token_order_1bit(_ptr(self.codes1), _ptr(self.factor1), _ptr(self.tok2pos),
                                                 self.n_tokens, _ptr(codes1_tok), _ptr(factor1_tok), st),
                      "token_order_1bit")
            if tok_cluster is None:
                tok_cluster = torch.empty(self.n_tokens, dtype=torch.int32, device=dev)
                check(lib().chm_token_clusters(_ptr(self.cluster_pos), self.n_clusters, _ptr(self.tok2pos),
                                               self.n_tokens, _ptr(tok_cluster), st), "token_clusters")
            self.codes1_tok, self.factor1_tok, self.tok_cluster = codes1_tok, factor1_tok, tok_cluster
        ptrs = [self._p(getattr(self, k)) if getattr(self, k) is not None else 0 for k in self.FIELDS]
        if not tensor_core_probe:
            ptrs[11] = ptrs[12] = 0
        self.view = ChmIndex(self.n_tokens, self.num_docs, self.n_clusters, self.ex_bits, self.dim,
                             self.max_list_len, self.max_doc_len, *ptrs)

    def with_probe(self, tensor_core: bool):
        """The same arrays with the tensor-core (True) or SIMT (False) probe."""
        v = ChmIndex.from_buffer_copy(self.view)
        v.centroids_bf16 = self._p(self.centroids_bf16) if tensor_core else 0
        v.centroid_norm_max = self._p(self.centroid_norm_max) if tensor_core else 0
        clone = object.__new__(DeviceIndex)
        clone.__dict__.update(self.__dict__)
        clone.view = v
        return clone

    def with_token_order(self, on: bool):
        """The same arrays with refinement reading the token-order 1-bit
        copies (True) or gathering the cluster-ordered ones (False).  Without
        them stage 1 also keeps to its hash-table path."""
        if on and self.codes1_tok is None:
            raise ValueError("this index has no token-order 1-bit copies")
        v = ChmIndex.from_buffer_copy(self.view)
        v.codes1_tok = self._p(self.codes1_tok) if on else 0
        v.factor1_tok = self._p(self.factor1_tok) if on else 0
        clone = object.__new__(DeviceIndex)
        clone.__dict__.update(self.__dict__)
        clone.view = v
        return clone

    def with_dense_stage1(self, on: bool):
        """The same arrays with stage 1's dense-bound path enabled (True) or
        its hash-table path only (False)."""
        if on and self.tok_cluster is None:
            raise ValueError("this index has no token clusters")
        v = ChmIndex.from_buffer_copy(self.view)
        v.tok_cluster = self._p(self.tok_cluster) if on else 0
        clone = object.__new__(DeviceIndex)
        clone.__dict__.update(self.__dict__)
        clone.view = v
        return clone

    @staticmethod
    def _p(t):
        return t.data_ptr()

    @classmethod
    def from_host(cls, *, cluster_pos, codes1, factor1, doc_ids, tok2pos, doc_ptrs, full_codes,
                  full_factors, centroids_rot, flips, dim, ex_bits, device="cuda", tensor_core_probe=True,
                  token_order=True):
        """Upload host arrays in the reference layout (oracle.Index fields)."""
        import torch
        dev = torch.device(device)
        t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a).astype(dt, copy=False)).to(dev)
        cents = t(centroids_rot, np.float32)
        norms = torch.empty(cents.shape[0], dtype=torch.float32, device=dev)
        check(lib().chm_row_norms(_ptr(cents), cents.shape[0], _ptr(norms), _stream(torch)), "row_norms")
        return cls(dim=dim, ex_bits=ex_bits, tensor_core_probe=tensor_core_probe, token_order=token_order,
                   cluster_pos=t(cluster_pos, np.int64),
                   codes1=t(codes1, np.uint8), factor1=t(factor1, np.float32),
                   doc_ids=t(doc_ids, np.int32), tok2pos=t(tok2pos, np.int32),
                   doc_ptrs=t(doc_ptrs, np.int64), full_codes=t(full_codes, np.uint8),
                   full_factors=t(full_factors, np.float32), centroids=cents, centroid_norms=norms,
                   flips=t(flips, np.uint8))

    def to_host(self):
        """Host copies in the reference layout (for the oracle)."""
        g = lambda x: x.cpu().numpy()
        return dict(cluster_pos=g(self.cluster_pos), codes1=g(self.codes1), factor1=g(self.factor1),
                    doc_ids=g(self.doc_ids), tok2pos=g(self.tok2pos).view(np.uint32),
                    doc_ptrs=g(self.doc_ptrs), full_codes=g(self.full_codes),
                    full_factors=g(self.full_factors), ex_bits=self.ex_bits)


def build_index(emb, doclens, n_clusters: int, ex_bits: int, seed: int = 42, stream=None, centroids=None):
    """GPU index build (chimera_index::build, build_index.cu:394-501) from a
    device tensor of raw embeddings [N, dim] and host doc lengths.

    Reservoir-sampled centroids (host, std::mt19937_64) -> exact nearest
    centroid on the GPU -> stable cluster order -> GPU rotation + RaBitQ
    encoding -> cluster-ordered 1-bit arrays.

    `centroids` ([n_clusters, dim] raw device tensor) replaces the sampling:
    a document shard is built with the centroids sampled from the whole
    corpus, so every shard shares the global cluster ids."""
    n, dim = int(emb.shape[0]), int(emb.shape[1])
    if centroids is None:
        ids = __import__("torch").from_numpy(sample_centroids(n, n_clusters, 42)).to(emb.device)
        centroids = emb[ids].contiguous()
    return build_index_streamed(lambda: iter([(0, n, emb)]), n, dim, doclens, n_clusters, ex_bits, centroids,
                                seed=seed, stream=stream)


def build_index_streamed(chunks, n: int, dim: int, doclens, n_clusters: int, ex_bits: int, centroids,
                         seed: int = 42, stream=None):
    """build_index over embeddings that arrive in chunks, for corpora whose
    raw embeddings do not fit on the device at once.  `chunks()` yields
    (s, e, x): x the [e - s, dim] f32 device rows of tokens s..e-1, in order,
    covering 0..n-1; `centroids` the [n_clusters, dim] raw centroids (for the
    whole corpus: sample_centroids' token ids).  Every token is assigned and
    encoded on its own, so the result equals build_index's on the
    concatenated rows."""
    import time

    import torch
    dev = centroids.device
    st = _stream(torch, stream)
    verbose = bool(os.environ.get("CHM_VERBOSE"))
    t0 = [time.time()]

    def phase(name):
        if verbose:
            torch.cuda.synchronize()
            now = time.time()
            print(f"[build] {name}: {now - t0[0]:.2f}s", flush=True)
            t0[0] = now
    doclens = np.asarray(doclens, np.int64)
    if doclens.sum() != n:
        raise ValueError("Document lengths do not sum to the number of embeddings")
    if tuple(centroids.shape) != (n_clusters, dim):
        raise ValueError("centroids must be [n_clusters, dim]")
    flips_np = fhtkac_flips(seed)
    flips = torch.from_numpy(flips_np).to(dev)
    cent_in = centroids.to(device=dev, dtype=torch.float32).contiguous()
    if dim < DIM:
        cent_raw = torch.zeros(n_clusters, DIM, dtype=torch.float32, device=dev)
        cent_raw[:, :dim] = cent_in
    else:
        cent_raw = cent_in
    cn_raw = torch.empty(n_clusters, dtype=torch.float32, device=dev)
    L = lib()
    check(L.chm_row_norms(_ptr(cent_raw), n_clusters, _ptr(cn_raw), st), "row_norms")
    # rotated centroids (padded dim) for the probe
    rot_c = torch.empty(n_clusters, DIM, dtype=torch.float32, device=dev)
    cb1_c = torch.empty(n_clusters, dtype=torch.float32, device=dev)
    cbex_c = torch.empty(n_clusters, dtype=torch.float32, device=dev)
    check(L.chm_prepare_queries(_ptr(flips), dim, ex_bits, _ptr(cent_in), n_clusters,
                                _ptr(rot_c), _ptr(cb1_c), _ptr(cbex_c), None, st), "rotate centroids")
    del cb1_c, cbex_c
    cnorm = torch.empty(n_clusters, dtype=torch.float32, device=dev)
    check(L.chm_row_norms(_ptr(rot_c), n_clusters, _ptr(cnorm), st), "row_norms")
    # per chunk: exact nearest centroid, rotation + RaBitQ encoding
    fb = DIM * (1 + ex_bits) // 8
    assign = torch.empty(n, dtype=torch.int32, device=dev)
    codes1 = torch.empty(n, 16, dtype=torch.uint8, device=dev)
    f1 = torch.empty(n, dtype=torch.float32, device=dev)
    full = torch.empty(n, fb, dtype=torch.uint8, device=dev)
    ff = torch.empty(n, dtype=torch.float32, device=dev)
    ws, wsb, done = None, 0, 0
    for s, e, x in chunks():
        m = e - s
        if s != done or m <= 0 or tuple(x.shape) != (m, dim):
            raise ValueError("chunks must cover the tokens in order with [e - s, dim] rows")
        done = e
        x = x.contiguous()
        if dim < DIM:
            x128 = torch.zeros(m, DIM, dtype=torch.float32, device=dev)
            x128[:, :dim] = x
        else:
            x128 = x
        need = L.chm_build_assign_workspace_bytes(m, n_clusters)
        if need > wsb:
            ws, wsb = None, 0
            ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
            wsb = need
        check(L.chm_build_assign(_ptr(x128), m, dim, _ptr(cent_raw), _ptr(cn_raw), n_clusters, _ptr(assign[s:e]),
                                 _ptr(ws), wsb, st), "build_assign")
        check(L.chm_build_encode(_ptr(flips), _ptr(x), m, dim, ex_bits, _ptr(codes1[s:e]), _ptr(f1[s:e]),
                                 _ptr(full[s:e]), _ptr(ff[s:e]), None, st), "build_encode")
        del x, x128
    if done != n:
        raise ValueError("chunks must cover every token")
    del ws, cent_raw, cn_raw
    phase("assign + encode")
    doc_ptrs = torch.from_numpy(np.concatenate([[0], np.cumsum(doclens)]).astype(np.int64)).to(dev)
    # IVF_PG::build_from_assignments + reorder_by_cluster (ivf_pg.cpp:110-126,
    # build_index.cu:328-363) on the GPU
    cluster_pos = torch.empty(n_clusters + 1, dtype=torch.int64, device=dev)
    inv = torch.empty(n, dtype=torch.int32, device=dev)
    codes1_cl = torch.empty(n, 16, dtype=torch.uint8, device=dev)
    f1_cl = torch.empty(n, dtype=torch.float32, device=dev)
    doc_ids = torch.empty(n, dtype=torch.int32, device=dev)
    tok2pos = torch.empty(n, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    wsb = L.chm_build_cluster_order_workspace_bytes(n, n_clusters)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
    check(L.chm_build_cluster_order(_ptr(assign), n, n_clusters, _ptr(doc_ptrs), len(doclens), _ptr(codes1),
                                    _ptr(f1), _ptr(cluster_pos), _ptr(inv), _ptr(codes1_cl), _ptr(f1_cl),
                                    _ptr(doc_ids), _ptr(tok2pos), _ptr(status), _ptr(ws), wsb, st), "cluster order")
    del ws
    bad = int(status.item())
    if bad:
        raise ChmError(CHM_ERR_CAPACITY if bad & 2 else CHM_ERR_INVALID, "cluster order")
    phase("cluster order")
    return DeviceIndex(dim=dim, ex_bits=ex_bits, cluster_pos=cluster_pos, codes1=codes1_cl, factor1=f1_cl,
                       doc_ids=doc_ids, tok2pos=tok2pos, doc_ptrs=doc_ptrs, full_codes=full, full_factors=ff,
                       centroids=rot_c, centroid_norms=cnorm, flips=flips, codes1_tok=codes1, factor1_tok=f1,
                       tok_cluster=assign), \
        dict(assign=assign, inv=inv, token_codes1=codes1, token_f1=f1)


class Searcher:
    """Batched GPU search over a DeviceIndex through chm_search."""

    def __init__(self, index: DeviceIndex, *, nprobe=128, k_refine=3000, k_full_bit=300, num_chunks=5,
                 k=100, batch=16):
        import torch
        self.torch = torch
        self.index = index
        self.params = SearchParams(nprobe, k_refine, k_full_bit, num_chunks, k, batch, 0)
        self._ws = None
        self._alloc()

    def _alloc(self):
        L = lib()
        nb = L.chm_search_workspace_bytes(C.byref(self.index.view), C.byref(self.params))
        if nb == 0:
            raise ValueError("invalid search parameters")
        self._ws = self.torch.empty(nb, dtype=self.torch.uint8, device=self.index.factor1.device)
        self.ws_bytes = nb

    def search_device(self, queries, results=None, num_results=None, stream=None):
        """queries: [Q, 32, dim] float32 device tensor."""
        torch = self.torch
        q = queries.contiguous()
        nq = int(q.shape[0])
        k = self.params.k
        if results is None:
            results = torch.empty(nq, k, dtype=torch.int64, device=q.device)
        if num_results is None:
            num_results = torch.empty(nq, dtype=torch.int32, device=q.device)
        check(lib().chm_search(C.byref(self.index.view), C.byref(self.params), _ptr(q), nq, _ptr(results),
                               _ptr(num_results), _ptr(self._ws), self.ws_bytes, _stream(torch, stream)),
              "search")
        return results, num_results

    def search(self, queries, stream=None):
        """Search with automatic retry of queries whose stage-1 table overflowed."""
        torch = self.torch
        res, nres = self.search_device(queries, stream=stream)
        bad = (nres < 0).nonzero().flatten()
        extra = 0
        while bad.numel() > 0 and extra < 6:
            extra += 1
            saved = self.params.table_log2_extra
            self.params.table_log2_extra = extra
            self._alloc()
            r2, n2 = self.search_device(queries[bad], stream=stream)
            res[bad], nres[bad] = r2, n2
            self.params.table_log2_extra = saved
            self._alloc()
            bad = (nres < 0).nonzero().flatten()
        if bad.numel() > 0:
            raise ChmError(CHM_ERR_CAPACITY, "search")
        return res, nres
