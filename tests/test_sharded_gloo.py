"""The document-sharded search protocol (chimera_b200.sharded.ShardedPipeline)
on world_size 2 and 3 CPU ranks over gloo, every stage computed by the oracle
on the rank's shard: the merged results must equal the oracle's search over
the whole corpus, bit for bit, on every rank."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    from chimera_b200 import sharded as SH
    from oracle import oracle as O
    from tests._corpus import corpus, oracle_search
    from tests._shard_oracle import OracleShardBackend

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        c = corpus("mini")
        cfg = c["cfg"]
        ix = c["index"]
        full = {k: torch.from_numpy(np.ascontiguousarray(getattr(ix, k))) for k in
                ("cluster_pos", "codes1", "factor1", "doc_ids", "tok2pos", "doc_ptrs", "full_codes",
                 "full_factors")}
        bases = SH.shard_bounds(cfg.num_docs, world)
        sh = SH.shard_index_arrays(full, bases[rank], bases[rank + 1])
        shard = O.Index(**{k: v.numpy() for k, v in sh.items()}, ex_bits=cfg.ex_bits)
        params = dict(nprobe=cfg.nprobe, k_refine=cfg.k_refine, k_full_bit=cfg.k_full_bit,
                      num_chunks=cfg.num_chunks, k=cfg.k)
        be = OracleShardBackend(shard, bases, rank, flips=c["flips"], centroids_rot=c["centroids_rot"],
                                cnorm=c["cnorm"], ex_bits=cfg.ex_bits, **params)
        pipe = SH.ShardedPipeline(be, SH.TorchComm(), params)
        q = torch.from_numpy(np.ascontiguousarray(c["queries"], np.float32))
        res, nres = pipe.search(q)
        want = [oracle_search(c, i)["result"] for i in range(q.shape[0])]
        ok = True
        for i, w in enumerate(want):
            got = res[i, :int(nres[i])].numpy()
            if not np.array_equal(got, np.asarray(w, np.int64)):
                ok = False
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_protocol_matches_single_index(world, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok"


def test_shard_index_arrays_partition():
    """Shards partition the tokens; local ids, offsets and cluster lists are
    consistent with the whole index."""
    from chimera_b200 import sharded as SH
    from tests._corpus import corpus
    c = corpus("mini")
    ix = c["index"]
    full = {k: torch.from_numpy(np.ascontiguousarray(getattr(ix, k))) for k in
            ("cluster_pos", "codes1", "factor1", "doc_ids", "tok2pos", "doc_ptrs", "full_codes", "full_factors")}
    bases = SH.shard_bounds(c["cfg"].num_docs, 3)
    total = 0
    for r in range(3):
        sh = SH.shard_index_arrays(full, bases[r], bases[r + 1])
        n = sh["factor1"].numel()
        total += n
        assert int(sh["cluster_pos"][-1]) == n
        assert int(sh["doc_ptrs"][-1]) == sh["full_factors"].numel() == n
        assert int(sh["doc_ids"].min()) >= 0 and int(sh["doc_ids"].max()) < bases[r + 1] - bases[r]
        # token t of the shard sits at cluster position tok2pos[t] and belongs to its doc
        owner = torch.repeat_interleave(torch.arange(bases[r + 1] - bases[r]),
                                        sh["doc_ptrs"][1:] - sh["doc_ptrs"][:-1])
        assert torch.equal(sh["doc_ids"][sh["tok2pos"].long()].long(), owner)
    assert total == full["factor1"].numel()
