"""Document-sharded search: one process per GPU, NCCL exchange steps.

The corpus's documents are split into contiguous ranges, one per rank.
Rank r holds docs [doc_base[r], doc_base[r+1]) with local ids: their tokens'
cluster-ordered 1-bit data, their full codes, and a cluster_pos over the
global clusters.  The centroids are global and held by every rank.  Each step
of one batched search, with the exchange that follows it:

  prepare     every rank, whole batch (rotation, query state, LUT)
  probe       rank r: rows [r*P, (r+1)*P) of the 32*B query tokens -> all_gather
  stage 1     every rank on its docs: local top k_refine by (partial desc,
              doc asc) + overflow flags -> all_gather lists, all_reduce flags
  merge       every rank: the global refined list (chm_merge_refined); it is
              the list one GPU holding the whole corpus produces
  1-bit       every rank scores the refined docs it owns, -inf elsewhere
              -> all_reduce(max): every rank has every score
  selection   every rank, identical (progressive chunked selection)
  full-bit    every rank scores the selected docs it owns -> all_reduce(max)
  final top-k every rank, identical

so the results equal the single-GPU results bit for bit.  The reference has
no multi-GPU path; the stages' own reference citations are in the kernels.

`ShardedPipeline` is the protocol over two interfaces: a stage backend
(`CudaShardBackend`: the C-ABI kernels on this rank's GPU) and a
communicator (`TorchComm`: torch.distributed, NCCL on GPUs).
"""
import ctypes as C

import numpy as np

from . import capi


def shard_bounds(num_docs: int, world: int):
    """Doc ranges of the ranks: rank r holds [b[r], b[r+1])."""
    return [num_docs * r // world for r in range(world + 1)]


def shard_index_arrays(a: dict, lo: int, hi: int) -> dict:
    """The index arrays of docs [lo, hi) with local doc ids, from the arrays
    of the whole corpus (keys as capi.DeviceIndex / the reference layout;
    torch tensors on any device).  Cluster order within a list stays token
    order, as a build over the shard's tokens alone produces it."""
    import torch
    dev = a["doc_ids"].device
    doc_ids = a["doc_ids"].to(torch.int64)
    keep = (doc_ids >= lo) & (doc_ids < hi)
    pos = keep.nonzero().flatten()
    cp = a["cluster_pos"].to(torch.int64)
    nc = cp.numel() - 1
    cl = torch.repeat_interleave(torch.arange(nc, device=dev), cp[1:] - cp[:-1])
    counts = torch.bincount(cl[pos], minlength=nc)
    cluster_pos = torch.zeros(nc + 1, dtype=torch.int64, device=dev)
    cluster_pos[1:] = torch.cumsum(counts, 0)
    dp = a["doc_ptrs"].to(torch.int64)
    t0, t1 = int(dp[lo]), int(dp[hi])
    new_of_old = torch.full((doc_ids.numel(),), -1, dtype=torch.int64, device=dev)
    new_of_old[pos] = torch.arange(pos.numel(), device=dev)
    tok2pos = new_of_old[a["tok2pos"][t0:t1].to(torch.int64)]
    return dict(cluster_pos=cluster_pos, codes1=a["codes1"][pos].contiguous(),
                factor1=a["factor1"][pos].contiguous(), doc_ids=(doc_ids[pos] - lo).to(torch.int32),
                tok2pos=tok2pos.to(a["tok2pos"].dtype), doc_ptrs=(dp[lo:hi + 1] - t0).contiguous(),
                full_codes=a["full_codes"][t0:t1].contiguous(), full_factors=a["full_factors"][t0:t1].contiguous())


class TorchComm:
    """The exchange steps over a torch.distributed process group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._flat = dist.get_backend(group) == "nccl"

    def all_gather(self, t):
        """[world, *t.shape], rank order."""
        t = t.contiguous()
        if self._flat:
            out = t.new_empty((self.world,) + tuple(t.shape))
            self.dist.all_gather_into_tensor(out, t, group=self.group)
            return out
        parts = [t.new_empty(t.shape) for _ in range(self.world)]
        self.dist.all_gather(parts, t, group=self.group)
        import torch
        return torch.stack(parts)

    def all_reduce_max(self, t):
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)
        return t


class ShardedPipeline:
    """One batched search of a document-sharded corpus (module docstring).

    Every rank calls `search_device` with the same queries; every rank gets
    the same results (global doc ids, -1 padded).  A query whose stage-1
    table overflowed on any rank comes back with a negative count on every
    rank; `search` reruns those queries with a larger table."""

    def __init__(self, backend, comm, params):
        self.b = backend
        self.comm = comm
        self.p = params  # nprobe, k_refine, k_full_bit, num_chunks, k

    def search_device(self, queries, table_log2_extra=0):
        b, comm = self.b, self.comm
        B = int(queries.shape[0])
        G, r = comm.world, comm.rank
        st = b.prepare(queries)
        rows = 32 * B
        per = (rows + G - 1) // G
        lo = min(r * per, rows)
        hi = min(lo + per, rows)
        part = b.probe(st, lo, hi, per)
        labels = comm.all_gather(part).reshape(G * per, -1)[:rows]
        docs, partial, counts, flags = b.stage1(st, labels, table_log2_extra)
        flags = comm.all_reduce_max(flags)
        g_docs = comm.all_gather(docs)
        g_partial = comm.all_gather(partial)
        g_counts = comm.all_gather(counts)
        rdocs, rpartial, rcount = b.merge_refined(g_docs, g_partial, g_counts)
        onebit = b.refine_1bit(st, b.localize(rdocs, rcount), rcount)
        onebit = comm.all_reduce_max(onebit)
        fb_docs, nf = b.select_fullbit(rdocs, onebit, rcount)
        fbs = b.fullbit(st, b.localize(fb_docs, nf), nf)
        fbs = comm.all_reduce_max(fbs)
        res, nres = b.final(fb_docs, fbs, nf)
        return res, b.fold_flags(nres, flags)

    def search(self, queries):
        """search_device plus the overflow retry (the same decision on every
        rank: the flags were all-reduced)."""
        res, nres = self.search_device(queries)
        # the backend's result buffers are reused by the retry below
        res, nres = res.clone(), nres.clone()
        extra = 0
        bad = (nres < 0).nonzero().flatten()
        while bad.numel() > 0:
            extra += 1
            if extra > 8:
                raise capi.ChmError(capi.CHM_ERR_CAPACITY, "sharded search")
            r2, n2 = self.search_device(queries[bad].contiguous(), table_log2_extra=extra)
            res[bad], nres[bad] = r2, n2
            bad = (nres < 0).nonzero().flatten()
        return res, nres


class NativeShardSearcher:
    """The sharded search in native code (chm_search_sharded, lib/
    libchimera_nccl.so): the same protocol as ShardedPipeline with the NCCL
    collectives enqueued on the search stream between the stage kernels, one
    call per batch from the host.  Every rank creates one with the same
    parameters; the NCCL unique id travels over `group` (torch.distributed)."""

    def __init__(self, index, doc_bases, rank, world, *, nprobe, k_refine, k_full_bit, num_chunks, k, batch,
                 group=None):
        import torch
        import torch.distributed as dist
        self.torch = torch
        self.ix = index
        self.L = capi.nccl_lib()
        self.rank, self.world = rank, world
        self.params = capi.SearchParams(nprobe, k_refine, k_full_bit, num_chunks, k, batch, 0)
        self._bases = (C.c_int64 * (world + 1))(*[int(b) for b in doc_bases])
        self.shard = capi.ShardInfo(rank, world, C.cast(self._bases, C.c_void_p))
        uid = (C.c_uint8 * 128)()
        if rank == 0:
            capi.check(self.L.chm_comm_unique_id(C.cast(uid, C.c_void_p)), "chm_comm_unique_id")
        if world > 1:
            dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
            t = torch.tensor(list(uid), dtype=torch.uint8, device=dev)
            dist.broadcast(t, src=0, group=group)
            uid = (C.c_uint8 * 128)(*t.cpu().tolist())
        self.comm = C.c_void_p()
        capi.check(self.L.chm_comm_init(C.cast(uid, C.c_void_p), world, rank, torch.cuda.current_device(),
                                         C.byref(self.comm)),
                   "chm_comm_init")
        self._ws = None
        self._alloc()
        self.timing = (C.c_float * len(capi.SH_STEPS))()

    def _alloc(self):
        nb = self.L.chm_search_sharded_workspace_bytes(C.byref(self.ix.view), C.byref(self.params), self.world)
        if nb == 0:
            raise ValueError("invalid search parameters")
        self._ws = self.torch.empty(nb, dtype=self.torch.uint8, device=self.ix.factor1.device)
        self.ws_bytes = nb

    def search_device(self, queries, results=None, num_results=None, timed=False):
        torch = self.torch
        q = queries.contiguous()
        nq = int(q.shape[0])
        k = self.params.k
        if results is None:
            results = torch.empty(nq, k, dtype=torch.int64, device=q.device)
        if num_results is None:
            num_results = torch.empty(nq, dtype=torch.int32, device=q.device)
        capi.check(self.L.chm_search_sharded(C.byref(self.ix.view), C.byref(self.params), C.byref(self.shard),
                                             self.comm, capi._ptr(q), nq, capi._ptr(results),
                                             capi._ptr(num_results), capi._ptr(self._ws), self.ws_bytes,
                                             capi._stream(torch),
                                             C.cast(self.timing, C.c_void_p) if timed else None),
                   "search_sharded")
        return results, num_results

    def step_ms(self):
        """Per-step device milliseconds of the last batch of a timed call."""
        return {n: float(self.timing[i]) for i, n in enumerate(capi.SH_STEPS)}

    def search(self, queries):
        """search_device with the overflow retry (every rank sees the same
        counts: the flags were all-reduced)."""
        res, nres = self.search_device(queries)
        extra = 0
        bad = (nres < 0).nonzero().flatten()
        while bad.numel() > 0 and extra < 6:
            extra += 1
            saved = self.params.table_log2_extra
            self.params.table_log2_extra = extra
            self._alloc()
            r2, n2 = self.search_device(queries[bad])
            res[bad], nres[bad] = r2, n2
            self.params.table_log2_extra = saved
            self._alloc()
            bad = (nres < 0).nonzero().flatten()
        if bad.numel() > 0:
            raise capi.ChmError(capi.CHM_ERR_CAPACITY, "search_sharded")
        return res, nres

    def close(self):
        if self.comm:
            capi.nccl_lib().chm_comm_destroy(self.comm)
            self.comm = C.c_void_p()


class CudaShardBackend:
    """The stage kernels of one rank (C ABI, current CUDA stream)."""

    def __init__(self, index, doc_bases, rank, *, nprobe, k_refine, k_full_bit, num_chunks, k, batch):
        import torch
        self.torch = torch
        self.ix = index
        self.v = C.byref(index.view)
        self.L = capi.lib()
        self.rank = rank
        self.base = int(doc_bases[rank])
        self.doc_bases = torch.tensor(doc_bases[:-1], dtype=torch.int64, device=index.factor1.device)
        self.nprobe, self.kr, self.kfb, self.nch, self.k = nprobe, k_refine, k_full_bit, num_chunks, k
        self.use_tc = bool(index.view.centroids_bf16) and nprobe <= 448
        self.batch = 0
        self._s1_extra = None
        self._alloc(batch)

    def _alloc(self, B):
        torch, dev = self.torch, self.ix.factor1.device
        self.batch = B
        ntok = 32 * B
        e = lambda *s, dt=torch.float32: torch.empty(*s, dtype=dt, device=dev)
        self.rot, self.cb1, self.cbex, self.lut = e(ntok, 128), e(ntok), e(ntok), e(ntok, 512)
        self.rd, self.rp = e(B, self.kr, dt=torch.int32), e(B, self.kr)
        self.nr, self.flags = e(B, dt=torch.int32), e(B, dt=torch.int32)
        self.mdocs, self.mpart, self.mcount = e(B, self.kr, dt=torch.int32), e(B, self.kr), e(B, dt=torch.int32)
        self.local = e(B, self.kr, dt=torch.int32)
        self.onebit = e(B, self.kr)
        self.fd, self.nf, self.fs = e(B, self.kr, dt=torch.int32), e(B, dt=torch.int32), e(B, self.kr)
        self.res, self.nres = e(B, self.k, dt=torch.int64), e(B, dt=torch.int32)
        self.fb_bytes = self.L.chm_refine_tc_workspace_bytes(self.v, B, self.kr)
        self.fb_ws = e(max(self.fb_bytes, 1), dt=torch.uint8)
        self._probe_ws = {}
        self._s1_extra = None

    def _stream(self):
        return capi._stream(self.torch)

    def _chk(self, st, what):
        capi.check(st, what)

    def prepare(self, queries):
        q = queries.contiguous()
        B = int(q.shape[0])
        if B > self.batch:
            self._alloc(B)
        self.B = B
        P = capi._ptr
        self._chk(self.L.chm_prepare_queries(P(self.ix.flips), self.ix.dim, self.ix.ex_bits, P(q), 32 * B,
                                             P(self.rot), P(self.cb1), P(self.cbex), P(self.lut), self._stream()),
                  "prepare")
        return None

    def probe(self, st, lo, hi, per):
        torch, P, L = self.torch, capi._ptr, self.L
        out = torch.zeros(per, self.nprobe, dtype=torch.int32, device=self.rot.device)
        n = hi - lo
        if n <= 0:
            return out
        key = n
        if key not in self._probe_ws:
            f = L.chm_probe_tc_workspace_bytes if self.use_tc else L.chm_probe_workspace_bytes
            nb = f(n, self.ix.n_clusters, self.nprobe)
            self._probe_ws[key] = (torch.empty(max(nb, 1), dtype=torch.uint8, device=self.rot.device), nb)
        ws, nb = self._probe_ws[key]
        rows = self.rot[lo:hi]
        if self.use_tc:
            s = L.chm_probe_tc(P(rows), n, P(self.ix.centroids), P(self.ix.centroids_bf16),
                               P(self.ix.centroid_norms), P(self.ix.centroid_norm_max), self.ix.n_clusters,
                               self.nprobe, P(out), P(ws), nb, self._stream())
        else:
            s = L.chm_probe(P(rows), n, P(self.ix.centroids), P(self.ix.centroid_norms), self.ix.n_clusters,
                            self.nprobe, P(out), P(ws), nb, self._stream())
        self._chk(s, "probe")
        return out

    def stage1(self, st, labels, extra):
        torch, P, L, B = self.torch, capi._ptr, self.L, self.B
        if self._s1_extra != extra:
            nb = L.chm_stage1_ex_workspace_bytes(self.v, self.batch, self.nprobe, extra)
            if nb == 0:
                raise ValueError("invalid stage-1 parameters")
            self._s1_ws = torch.empty(nb, dtype=torch.uint8, device=self.rot.device)
            self._s1_bytes = nb
            self._s1_extra = extra
        lab = labels.contiguous()
        self._chk(L.chm_stage1_ex(self.v, B, P(self.lut), P(self.cb1), P(lab), self.nprobe, self.kr,
                                  P(self.rd), P(self.rp), P(self.nr), P(self.flags), extra, P(self._s1_ws),
                                  self._s1_bytes, self._stream()), "stage1")
        return self.rd[:B], self.rp[:B], self.nr[:B], self.flags[:B]

    def merge_refined(self, g_docs, g_partial, g_counts):
        P, B = capi._ptr, self.B
        shards = int(g_docs.shape[0])
        self._chk(self.L.chm_merge_refined(B, shards, self.kr, P(g_docs), P(g_partial), P(g_counts),
                                           P(self.doc_bases), P(self.mdocs), P(self.mpart), P(self.mcount),
                                           self._stream()), "merge_refined")
        return self.mdocs[:B], self.mpart[:B], self.mcount[:B]

    def localize(self, gdocs, counts):
        P, B = capi._ptr, self.B
        out = self.torch.empty_like(gdocs)
        self._chk(self.L.chm_shard_localize(B, self.kr, P(gdocs), P(counts), self.base, self.ix.num_docs, P(out),
                                            self._stream()), "localize")
        return out

    def refine_1bit(self, st, local, counts):
        P, B = capi._ptr, self.B
        if B >= 16:  # chm_search's choice: the tensor-core filter on batches (same scores either way)
            self._chk(self.L.chm_refine_1bit_tc(self.v, B, P(self.lut), P(self.cb1), P(self.rot), P(local),
                                                P(counts), self.kr, P(self.onebit), P(self.fb_ws), self.fb_bytes,
                                                self._stream()), "refine_1bit")
        else:
            self._chk(self.L.chm_refine_1bit(self.v, B, P(self.lut), P(self.cb1), P(local), P(counts), self.kr,
                                             P(self.onebit), self._stream()), "refine_1bit")
        return self.onebit[:B]

    def select_fullbit(self, rdocs, onebit, counts):
        P, B = capi._ptr, self.B
        self._chk(self.L.chm_select_fullbit(B, P(rdocs), P(onebit), P(counts), self.kr, self.kfb, self.nch,
                                            P(self.fd), P(self.nf), self.kr, self._stream()), "select_fullbit")
        return self.fd[:B], self.nf[:B]

    def fullbit(self, st, fb_local, nf):
        P, B = capi._ptr, self.B
        self._chk(self.L.chm_fullbit_score_tc(self.v, B, P(self.rot), P(self.cbex), P(fb_local), P(nf), self.kr,
                                              P(self.fs), P(self.fb_ws), self.fb_bytes, self._stream()), "fullbit")
        return self.fs[:B]

    def final(self, fb_docs, fbs, nf):
        P, B = capi._ptr, self.B
        self._chk(self.L.chm_final_topk(B, P(fb_docs), P(fbs), P(nf), self.kr, self.k, P(self.res), P(self.nres),
                                        self._stream()), "final_topk")
        return self.res[:B], self.nres[:B]

    def fold_flags(self, nres, flags):
        return self.torch.where(flags != 0, self.torch.full_like(nres, -1), nres)
