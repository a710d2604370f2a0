"""Document-sharded search on the GPU: the CUDA stage backend under the
sharding protocol must return exactly what chm_search returns on the whole
index.

* one GPU: G shards as host threads sharing the device, exchanging tensors
  through a host barrier (no kernel waits on another kernel);
* two GPUs (skipped with fewer): one process per GPU over NCCL, through the
  Python protocol and through chm_search_sharded (native);
* one GPU, native: chm_search_sharded as a world of one.
"""
import os
import socket
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class ThreadComm:
    """all_gather / all_reduce(max) between threads of one process."""

    def __init__(self, world):
        self.world = world
        self.bar = threading.Barrier(world)
        self.slots = [None] * world

    def view(self, rank):
        comm = self

        class _V:
            def __init__(self):
                self.rank, self.world = rank, comm.world

            def all_gather(self, t):
                torch.cuda.current_stream().synchronize()
                comm.slots[rank] = t.contiguous()
                comm.bar.wait()
                out = torch.stack([s for s in comm.slots])
                torch.cuda.current_stream().synchronize()
                comm.bar.wait()
                return out

            def all_reduce_max(self, t):
                g = self.all_gather(t)
                t.copy_(g.max(dim=0).values)
                return t
        return _V()


def _full_index_arrays(d):
    return {k: getattr(d, k) for k in ("cluster_pos", "codes1", "factor1", "doc_ids", "tok2pos", "doc_ptrs",
                                       "full_codes", "full_factors")}


def _shard_device_index(d, lo, hi):
    from chimera_b200 import capi
    from chimera_b200 import sharded as SH
    sh = SH.shard_index_arrays(_full_index_arrays(d), lo, hi)
    return capi.DeviceIndex(dim=d.dim, ex_bits=d.ex_bits, centroids=d.centroids, centroid_norms=d.centroid_norms,
                            flips=d.flips, **sh)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_threads_match_chm_search(world):
    from chimera_b200 import capi
    from chimera_b200 import sharded as SH
    from tests._corpus import corpus, device_index
    c = corpus("small")
    cfg = c["cfg"]
    d = device_index(c, torch)
    q = torch.from_numpy(np.ascontiguousarray(c["queries"], np.float32)).cuda()
    want, wn = capi.Searcher(d, k=cfg.k, batch=q.shape[0], **cfg.search_kwargs()).search(q)
    torch.cuda.synchronize()
    bases = SH.shard_bounds(cfg.num_docs, world)
    shards = [_shard_device_index(d, bases[r], bases[r + 1]) for r in range(world)]
    comm = ThreadComm(world)
    params = dict(nprobe=cfg.nprobe, k_refine=cfg.k_refine, k_full_bit=cfg.k_full_bit, num_chunks=cfg.num_chunks,
                  k=cfg.k)
    out = [None] * world
    err = []

    def run(r):
        try:
            be = SH.CudaShardBackend(shards[r], bases, r, batch=q.shape[0], **params)
            res, nres = SH.ShardedPipeline(be, comm.view(r), params).search(q)
            torch.cuda.synchronize()
            out[r] = (res.clone(), nres.clone())
        except Exception as e:  # surfaced below
            err.append(e)
            comm.bar.abort()

    th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    assert not err, err
    for r in range(world):
        res, nres = out[r]
        assert torch.equal(nres, wn), r
        assert torch.equal(res, want), r


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    from chimera_b200 import capi
    from chimera_b200 import sharded as SH
    from tests._corpus import corpus, device_index
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        c = corpus("small")
        cfg = c["cfg"]
        d = device_index(c, torch)
        q = torch.from_numpy(np.ascontiguousarray(c["queries"], np.float32)).cuda()
        want, wn = capi.Searcher(d, k=cfg.k, batch=q.shape[0], **cfg.search_kwargs()).search(q)
        bases = SH.shard_bounds(cfg.num_docs, world)
        shard = _shard_device_index(d, bases[rank], bases[rank + 1])
        params = dict(nprobe=cfg.nprobe, k_refine=cfg.k_refine, k_full_bit=cfg.k_full_bit,
                      num_chunks=cfg.num_chunks, k=cfg.k)
        be = SH.CudaShardBackend(shard, bases, rank, batch=q.shape[0], **params)
        res, nres = SH.ShardedPipeline(be, SH.TorchComm(), params).search(q)
        torch.cuda.synchronize()
        ok = torch.equal(res, want) and torch.equal(nres, wn)
        # the same protocol in native code (chm_search_sharded)
        ns = SH.NativeShardSearcher(shard, bases, rank, world, batch=q.shape[0], **params)
        res2, nres2 = ns.search(q)
        torch.cuda.synchronize()
        ns.close()
        ok = ok and torch.equal(res2, want) and torch.equal(nres2, wn)
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_native_sharded_single_rank_matches_chm_search():
    """chm_search_sharded (the protocol in native code, NCCL collectives on
    the search stream) as a world of one: the same results as chm_search, in
    batches of 5 and 16 (both refinement paths), and per-step timings."""
    from chimera_b200 import capi
    from chimera_b200 import sharded as SH
    from tests._corpus import corpus, device_index
    c = corpus("small")
    cfg = c["cfg"]
    d = device_index(c, torch)
    q = torch.from_numpy(np.ascontiguousarray(c["queries"], np.float32)).cuda()
    want, wn = capi.Searcher(d, k=cfg.k, batch=q.shape[0], **cfg.search_kwargs()).search(q)
    for batch in (5, 16):
        s = SH.NativeShardSearcher(d, [0, cfg.num_docs], 0, 1, batch=batch, k=cfg.k, **cfg.search_kwargs())
        try:
            res, nres = s.search(q)
            torch.cuda.synchronize()
            assert torch.equal(nres, wn) and torch.equal(res, want), batch
            s.search_device(q, timed=True)
            ms = s.step_ms()
            assert set(ms) == set(capi.SH_STEPS) and all(v >= 0 for v in ms.values())
        finally:
            s.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_nccl_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"
