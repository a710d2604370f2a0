#!/usr/bin/env python3
"""Benchmark of the B200 Chimera search path (QPS at Recall@100).

A step is one batch of `--batch` queries through the whole search hot path
(rotate + LUT, exact centroid probe, stage-1 LUT scoring + aggregation +
top-k_refine, 1-bit MaxSim refinement, progressive selection, full-bit
MaxSim, final ordering) over a synthetic corpus with BASELINE config C3's
shapes (1M docs, ~64M tokens, 262,144 clusters, ex-bits 4, nprobe 128,
k_refine 3000, k_full_bit 300, 5 chunks, k 100), built on the GPU.

value : queries/s with the queries already in HBM, device-timed (CUDA events
        on the launching stream, barrier + synchronize on both sides, max over
        ranks).
e2e   : queries/s through the public search entry point from pinned host
        buffers, the query H2D copy and the result D2H copy inside the timed
        region.
--impl reference : the CPU implementation (the oracle restatement of the
        same path with the reference's full-bit scorer order), all host
        threads, on a bounded sample of the same workload.

The corpus (≈8 GB of index) is larger than L2, so no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


class ClockSampler:
    """SM clocks and clock-event reasons sampled during the timed region:
    through NVML every 10 ms (read-only queries), else through nvidia-smi
    (about one sample per 200 ms)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index=0):
        self.gpu = gpu_index
        self.rows = []
        self._stop = threading.Event()
        self._t = None
        self._nv = None
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(gpu_index).uuid)
                self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
            self._nv = pynvml
        except Exception:
            self._nv = None

    def _sample_nvml(self):
        nv, h = self._nv, self._h
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        why = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        flags = ["Active" if why & b else "Not Active" for b in bits]
        return [str(self.gpu), str(sm), str(mx), "", hex(why)] + flags

    def _run(self):
        while not self._stop.is_set():
            try:
                if self._nv is not None:
                    self.rows.append(self._sample_nvml())
                    self._stop.wait(0.01)
                    continue
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q,
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.rows.append([x.strip() for x in out.split(",")])
            except Exception:
                self._nv = None
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "source": "nvml" if self._nv else "nvidia-smi"}


# DRAM bytes per unit of work of the dominant kernel, from one ncu capture of
# it on the c3s corpus with 32 queries (the 1-bit tensor-core refinement over
# token-order codes read + wrote 153.9 MB for 6.30 M refined tokens), scaled
# here by this run's refined tokens.
NCU_TRAFFIC_PER_UNIT = {"refine_1bit": 24.4}

METRIC = {"c3": "QPS at Recall@100 (C3 passage corpus)", "c4": "QPS at Recall@100 (C4 long-document corpus)",
          "c5": "QPS at Recall@100 (C5 large sharded corpus)", "c1": "QPS at Recall@100 (C1 small corpus)"}


def peaks():
    try:
        p = json.load(open(PEAKS))
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def ground_truth(torch, emb, doc_ptrs, queries, k, qsel):
    """Exact fp32 MaxSim top-k for the selected queries (brute force, GPU)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    n = emb.shape[0]
    m = doc_ptrs.shape[0] - 1
    owner = torch.repeat_interleave(torch.arange(m, device=emb.device), doc_ptrs[1:] - doc_ptrs[:-1])
    out = []
    chunk = 1 << 23
    for q in qsel:
        qt = queries[q]                                    # [32, d]
        best = torch.full((qt.shape[0], m), -float("inf"), device=emb.device)
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            sc = qt @ emb[s:e].T                           # [32, chunk]
            best.scatter_reduce_(1, owner[s:e].unsqueeze(0).expand(qt.shape[0], -1), sc, reduce="amax")
        score = best.sum(0)
        out.append(torch.topk(score, k).indices.cpu().numpy())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c3")
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--inflight", type=int, default=1,
                    help="batches in flight at once (one GPU): each on its own stream with its own workspace")
    ap.add_argument("--recall-queries", type=int, default=256)
    ap.add_argument("--cpu-sample", type=int, default=32,
                    help="queries whose full-bit stage the CPU baseline times")
    ap.add_argument("--parity-queries", type=int, default=8,
                    help="queries searched by the CPU oracle and compared with the GPU results")
    ap.add_argument("--ref-sample", type=int, default=16, help="queries per step of the reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--streamed", action="store_true",
                    help="generate and build the corpus chunk by chunk (always on for c5)")
    ap.add_argument("--micro", choices=["probe", "lut"], default=None,
                    help="operator microbench (BASELINE config C2) instead of the search bench")
    ap.add_argument("--lut-codes", type=int, default=1 << 26, help="codes scored per step by --micro lut")
    args = ap.parse_args()
    if args.micro == "probe":
        return micro_probe(args)
    if args.micro == "lut":
        return micro_lut(args)

    import torch
    from chimera_b200 import capi, workloads as W, sharded as SH

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and rank != 0:
        return  # the CPU reference arm runs on rank 0 alone
    torch.cuda.set_device(local)
    dist = None
    if world > 1 and args.impl == "ours":
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    cfg = W.CONFIGS[args.config]
    t0 = time.time()
    # corpora whose raw embeddings do not fit one device (C5: 600M tokens x
    # 512 B) are generated chunk by chunk (the same values) and built in chunks
    streamed = args.streamed or cfg.name == "c5"
    sc = None
    if streamed:
        sc = W.StreamedCorpus(cfg, seed=0)
        emb, doclens = None, sc.doclens
        queries = sc.queries()
        n_tok = sc.n
    else:
        emb, doclens, queries = W.generate_torch(cfg, seed=0)
        n_tok = int(emb.shape[0])
    log(f"[bench] corpus {cfg.name}: {n_tok} tokens, {cfg.num_docs} docs ({time.time() - t0:.1f}s)"
        + (", streamed" if streamed else ""))
    dl_host = doclens.cpu().numpy()
    ptr_full = torch.from_numpy(W.doc_ptrs(dl_host)).to(queries.device)
    t0 = time.time()
    whole = world == 1 or args.impl == "reference"
    if whole:
        bases = [0, cfg.num_docs]
    else:
        # document shard: docs [bases[rank], bases[rank+1]) with the centroids
        # sampled from the whole corpus (the single-GPU build's centroids)
        bases = SH.shard_bounds(cfg.num_docs, world)
    lo, hi = bases[rank if not whole else 0], bases[rank + 1 if not whole else 1]
    t_lo, t_hi = int(ptr_full[lo]), int(ptr_full[hi])
    ids = torch.from_numpy(capi.sample_centroids(n_tok, cfg.n_clusters, 42)).to(queries.device)
    cents = emb[ids].contiguous() if emb is not None else sc.gather(ids)
    if emb is not None:
        chunks = lambda: iter([(0, t_hi - t_lo, emb[t_lo:t_hi])])
    else:
        chunks = lambda: ((s - t_lo, e - t_lo, x) for s, e, x in sc.chunks(t_lo, t_hi))
    index = capi.build_index_streamed(chunks, t_hi - t_lo, cfg.dim, dl_host[lo:hi], cfg.n_clusters, cfg.ex_bits,
                                      cents)[0]
    del cents, ids
    torch.cuda.synchronize()
    log(f"[bench] index built in {time.time() - t0:.1f}s (rank {rank}, docs {lo}..{hi})")

    if args.impl == "reference":
        run_reference(args, cfg, index, queries, torch, emb, ptr_full, sc)
        return

    # exact MaxSim ground truth for the recall check, before the corpus is freed
    nq_total = queries.shape[0]
    nrec = min(args.recall_queries, nq_total)
    gt = None
    if nrec > 0 and rank == 0:
        gt = (ground_truth(torch, emb, ptr_full, queries, cfg.k, list(range(nrec))) if emb is not None else
              W.ground_truth_streamed(sc, queries[:nrec], cfg.k))
    del emb
    torch.cuda.empty_cache()

    B = args.batch
    params = dict(nprobe=cfg.nprobe, k_refine=cfg.k_refine, k_full_bit=cfg.k_full_bit, num_chunks=cfg.num_chunks,
                  k=cfg.k)
    inflight = max(1, args.inflight) if world == 1 else 1
    main_stream = torch.cuda.current_stream()
    lanes = [main_stream] + [torch.cuda.Stream() for _ in range(inflight - 1)]
    if world == 1:
        searchers = [capi.Searcher(index, k=cfg.k, batch=B, **cfg.search_kwargs()) for _ in range(inflight)]
        searcher = searchers[0]
        # one result buffer per step, so that every timed step's counts can be
        # checked after the timed region
        nbuf = args.warmup + args.steps
        res_bufs = [torch.empty(B, cfg.k, dtype=torch.int64, device="cuda") for _ in range(nbuf)]
        nres_bufs = [torch.empty(B, dtype=torch.int32, device="cuda") for _ in range(nbuf)]
        # step i runs on lane i % inflight (its own stream and workspace)
        search_device = lambda qb, i: searchers[i % inflight].search_device(qb, res_bufs[i], nres_bufs[i],
                                                                            stream=lanes[i % inflight])
        search_full = searcher.search
        parallelism = "single GPU" if inflight == 1 else f"single GPU, {inflight} batches in flight"
    else:
        # the sharded protocol in native code: stage kernels and NCCL
        # collectives on one stream, one host call per batch
        pipe = SH.NativeShardSearcher(index, bases, rank, world, batch=B, **params)
        search_device = lambda qb, i: pipe.search_device(qb)
        search_full = pipe.search
        parallelism = f"document shards x{world} (chm_search_sharded: NCCL all_gather/all_reduce on the stream)"

    # every rank serves the same query stream (strong scaling: the corpus and
    # the queries are fixed, the documents are split across the ranks)
    def batch_at(i):
        s = (i * B) % nq_total
        idx = torch.arange(s, s + B, device=queries.device) % nq_total
        return queries[idx].contiguous()

    stream = torch.cuda.current_stream()
    batches = [batch_at(i) for i in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        _, nres = search_device(batches[i], i)
    torch.cuda.synchronize()
    if nres.min().item() < 0:
        raise RuntimeError("stage-1 table overflow during warmup")

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    # ---- device-timed value -------------------------------------------------
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.nvtx.range_push("timed")
        ev0.record(stream)
        for ln in lanes[1:]:
            ln.wait_stream(stream)
        timed_counts = []
        for i in range(args.steps):
            timed_counts.append(search_device(batches[args.warmup + i], args.warmup + i)[1])
        for ln in lanes[1:]:
            stream.wait_stream(ln)
        ev1.record(stream)
        torch.cuda.nvtx.range_pop()
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_per_step = ms / args.steps
    qps = B * args.steps / (ms / 1e3)
    # every timed query must have completed without a stage-1 overflow
    # (an overflowed query would have been timed with an incomplete result)
    bad_timed = int(sum(int((c < 0).sum().item()) for c in timed_counts))
    if bad_timed:
        raise RuntimeError(f"{bad_timed} timed queries overflowed their stage-1 tables")

    # ---- end-to-end through the public entry point, host buffers -----------
    hq = [batches[args.warmup + i].cpu().pin_memory() for i in range(args.steps)]
    hres = [torch.empty(B, cfg.k, dtype=torch.int64).pin_memory() for _ in lanes]
    dq = [torch.empty_like(batches[0]) for _ in lanes]
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for ln in lanes[1:]:
        ln.wait_stream(stream)
    e2e_counts = []
    for i in range(args.steps):
        j = (args.warmup + i) % len(lanes)
        with torch.cuda.stream(lanes[j]):
            dq[j].copy_(hq[i], non_blocking=True)
            r, c = search_device(dq[j], args.warmup + i)
            hres[j].copy_(r, non_blocking=True)
        e2e_counts.append(c)
    for ln in lanes[1:]:
        stream.wait_stream(ln)
    e1.record(stream)
    barrier()
    ems = max_over_ranks(e0.elapsed_time(e1))
    e2e_qps = B * args.steps / (ems / 1e3)
    bad_e2e = int(sum(int((c < 0).sum().item()) for c in e2e_counts))
    if bad_e2e:
        raise RuntimeError(f"{bad_e2e} end-to-end queries overflowed their stage-1 tables")

    # ---- latency percentiles (one query per call, as gpu_search times it) --
    lat = latency_percentiles(torch, queries, lambda q: search_device(q, 0), barrier, n=64)

    # ---- recall ------------------------------------------------------------
    recall = None
    r_all = None
    if nrec > 0:
        r_all, _ = search_full(queries[:nrec].contiguous())
        r_all = r_all.cpu().numpy()
        if rank == 0:
            recall = round(W.recall_at_k(np.stack(gt), r_all, cfg.k), 4)

    # ---- per-step device times of one sharded batch (exchange included) -----
    shard_steps = None
    if world > 1:
        barrier()
        pipe.search_device(batches[args.warmup], timed=True)
        torch.cuda.synchronize()
        loc = pipe.step_ms()
        shard_steps = {k: round(max_over_ranks(v), 3) for k, v in loc.items()}
        tot = sum(shard_steps.values())
        xch = sum(v for k, v in shard_steps.items() if k.startswith(("gather", "reduce")))
        shard_steps["exchange_share"] = round(xch / tot, 4) if tot > 0 else None

    # ---- per-stage profile on this rank's (shard) index, exchange excluded --
    # (one GPU: the timed searcher itself, whose workspace is the largest
    # allocation of a big batch)
    torch.cuda.empty_cache()
    prof_searcher = searcher if world == 1 else capi.Searcher(index, k=cfg.k, batch=B, **cfg.search_kwargs())
    stages, stages_extra = profile_stages(torch, capi, index, prof_searcher, batches[args.warmup], cfg)
    del prof_searcher

    hbm, bf16, kind = peaks()
    # the dominant single kernel: probe and stage1 are pipelines of several
    # comparable kernels; the other stages are one main kernel each
    dom = max((s for s in stages if s["name"] not in ("probe", "stage1")), key=lambda s: s["ms"])
    achieved = dom["algo_bytes"] / (dom["ms"] / 1e3) / 1e9 if dom["bound"] == "hbm" else \
        dom["algo_flops"] / (dom["ms"] / 1e3) / 1e12
    peak = hbm if dom["bound"] == "hbm" else bf16
    probe_launches = next(s["launches"] for s in stages if s["name"] == "probe")
    if world == 1:
        launches = sum(s["launches"] for s in stages) + 1  # + chm_search's status fold
    else:
        # chm_search's kernels plus the sharded path's merge, two localizes and
        # label memset-free fold (the collectives are NCCL's own kernels)
        launches = sum(s["launches"] for s in stages) + 1 + 3
    line = {
        "metric": METRIC.get(cfg.name, f"QPS at Recall@100 ({cfg.name})"),
        "value": round(qps, 2), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32+u8", "data": "synthetic",
        "config": {"workload": f"{cfg.name}: {cfg.num_docs} docs, {int(ptr_full[-1])} tokens, "
                               f"{cfg.n_clusters} clusters, ex_bits {cfg.ex_bits}, nprobe {cfg.nprobe}, "
                               f"k_refine {cfg.k_refine}, k_full_bit {cfg.k_full_bit}, k {cfg.k}",
                   "batch_queries": B, "batches_in_flight": inflight,
                   "l2": "inputs larger than L2 (index >> 126 MB)",
                   "recall@100": recall, "recall_queries": nrec,
                   "latency_ms_single_query": lat, "parallelism": parallelism,
                   "stages_scope": "rank 0 index" + (" shard, exchange excluded" if world > 1 else "")},
        "e2e": {"value": round(e2e_qps, 2), "unit": "queries/s",
                "h2d_bytes_per_step": int(world * B * 32 * cfg.dim * 4), "d2h_bytes_per_step": int(world * B * cfg.k * 8)},
        "roofline": {"kernel": dom["name"], "bound": dom["bound"], "achieved": round(achieved, 2),
                     "peak": peak, "unit": "GB/s" if dom["bound"] == "hbm" else "TFLOP/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": (round(NCU_TRAFFIC_PER_UNIT[dom["name"]] * dom["units"])
                                 if dom["name"] in NCU_TRAFFIC_PER_UNIT and dom.get("units") else None),
                     "traffic_source": "ncu capture of the same kernel on the c3s case, scaled by refined tokens",
                     "peak_kind": kind},
        "stages_ms_per_step": {s["name"]: round(s["ms"], 3) for s in stages},
        "stage1_table_path_queries": next(s.get("table_path_queries") for s in stages if s["name"] == "stage1"),
        "sharded_steps_ms_max_over_ranks": shard_steps,
        "stages_algo_gbs": {s["name"]: round(s["algo_bytes"] / (s["ms"] / 1e3) / 1e9, 1)
                            for s in stages if s["algo_bytes"]},
        "gpu_launches": int(launches * args.steps),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, cfg, index, queries, torch, stages_extra)
        if args.parity_queries > 0:
            line["parity"] = oracle_parity(args, cfg, index, queries, torch, r_all, gt)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        pipe.close()
        dist.destroy_process_group()


def micro_probe(args):
    """C2 centroid-probe microbench: 1,024 queries x 32 tokens of unit-norm
    random vectors against 262,144 unit-norm random centroids, exact top-128
    per token through chm_probe_tc (bf16 tcgen05 candidates, exact fp32
    re-rank).  One step = the whole 32,768-row batch."""
    import ctypes as C
    import torch
    from chimera_b200 import capi
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    g = torch.Generator(device="cuda").manual_seed(0)
    rows, nc, nprobe = 1024 * 32, 262144, 128
    q = torch.randn(rows, 128, device="cuda", generator=g)
    q /= q.norm(dim=1, keepdim=True)
    cents = torch.randn(nc, 128, device="cuda", generator=g)
    cents /= cents.norm(dim=1, keepdim=True)
    L, P, st = capi.lib(), capi._ptr, capi._stream(torch)
    cn = torch.empty(nc, device="cuda")
    capi.check(L.chm_row_norms(P(cents), nc, P(cn), st), "norms")
    cb = torch.empty(nc, 128, dtype=torch.bfloat16, device="cuda")
    capi.check(L.chm_to_bf16(P(cents), nc * 128, P(cb), st), "bf16")
    cmax = torch.empty(1, device="cuda")
    capi.check(L.chm_max_value(P(cn), nc, P(cmax), st), "max")
    labels = torch.empty(rows, nprobe, dtype=torch.int32, device="cuda")
    wb = L.chm_probe_tc_workspace_bytes(rows, nc, nprobe)
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    run = lambda: capi.check(L.chm_probe_tc(P(q), rows, P(cents), P(cb), P(cn), P(cmax), nc, nprobe, P(labels),
                                            P(ws), wb, st), "probe_tc")
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        torch.cuda.synchronize()
        e0.record(torch.cuda.current_stream())
        for _ in range(args.steps):
            run()
        e1.record(torch.cuda.current_stream())
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    flops = 2.0 * rows * nc * 128
    tf = flops / (ms / 1e3) / 1e12
    hbm, bf16, kind = peaks()
    # exactness spot check against a fp32 brute force on a few rows
    sel = torch.arange(0, rows, rows // 16, device="cuda")
    d = cn[None, :] - 2.0 * (q[sel] @ cents.T)
    ref = torch.topk(-d, nprobe, dim=1).indices.sort(dim=1).values
    got = labels[sel].long().sort(dim=1).values
    agree = float((ref == got).float().mean().item())
    print(json.dumps({"metric": "centroid probe TFLOP/s (C2 operator microbench)", "value": round(tf, 2),
                      "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(ms, 3), "higher_is_better": True, "dtype": "bf16 candidates + fp32 re-rank",
                      "data": "synthetic",
                      "config": {"workload": "C2: 1,024 queries x 32 tokens x 128 dims vs 262,144 centroids, top-128",
                                 "rows": rows, "centroids": nc, "nprobe": nprobe,
                                 "top128_agreement_with_torch_fp32": agree},
                      "roofline": {"kernel": "chm_probe_tc (all launches)", "bound": "tensor", "achieved": round(tf, 2),
                                   "peak": bf16, "unit": "TFLOP/s", "frac": round(tf / bf16, 4), "traffic": None,
                                   "peak_kind": kind},
                      "clocks": clk.summary()}), flush=True)


def micro_lut(args):
    """C2 LUT-scoring microbench: `--lut-codes` (64M) uniform random codes at
    ex_bits 1, 2, 4 and 7 (stored widths w = 2, 3, 5, 8 bits per dim, the
    doc_full.bin layout) and the 1-bit cluster code (w = 1), grouped in lists
    of 64 codes with one fp32 scale factor per list (broadcast to its codes).
    Every code is scored by the 32 tokens of one query, and each list keeps
    the MaxSim over its codes: 128 queries x 8,192 lists, through
    chm_fullbit_score_tc (w = 2..7), chm_fullbit_score (w = 8) and
    chm_refine_1bit_tc (w = 1).  A step scores all codes once; value = code
    bytes read (16 w + 4 per code) / time."""
    import ctypes as C
    import torch
    from chimera_b200 import capi
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    L, P, st = capi.lib(), capi._ptr, capi._stream(torch)
    g = torch.Generator(device="cuda").manual_seed(0)
    nq, per, tok = 128, 8192, 64
    n = args.lut_codes
    docs = n // tok
    per = min(per, docs // nq)
    n = nq * per * tok
    dptr = torch.arange(0, n + 1, tok, dtype=torch.int64, device="cuda")
    fb_docs = torch.arange(nq * per, dtype=torch.int32, device="cuda").view(nq, per)
    num = torch.full((nq,), per, dtype=torch.int32, device="cuda")
    scale = torch.rand(nq * per, generator=g, device="cuda") * 0.5 + 0.05
    factors = scale.repeat_interleave(tok).contiguous()
    q = torch.randn(nq * 32, 128, generator=g, device="cuda")
    q /= q.norm(dim=1, keepdim=True)
    hbm, _, kind = peaks()
    out = {}
    for ex in (0, 1, 2, 4, 7):
        w = 1 + ex if ex else 1
        codes = torch.randint(0, 256, (n, 16 * w), dtype=torch.uint8, generator=g, device="cuda")
        rot = q.contiguous()
        cb = torch.empty(nq * 32, device="cuda")
        cbx = torch.empty(nq * 32, device="cuda")
        lut = torch.empty(nq * 32, 512, device="cuda")
        flips = torch.zeros(64, dtype=torch.uint8, device="cuda")
        capi.check(L.chm_prepare_queries(P(flips), 128, max(ex, 1), P(q), nq * 32, P(rot), P(cb), P(cbx), P(lut), st),
                   "prepare")
        view = capi.ChmIndex()
        view.n_tokens, view.num_docs, view.ex_bits, view.dim = n, nq * per, max(ex, 1), 128
        view.doc_ptrs = dptr.data_ptr()
        scores = torch.empty(nq, per, device="cuda")
        if w == 1:
            view.codes1_tok, view.factor1_tok = codes.data_ptr(), factors.data_ptr()
            wb = L.chm_refine_1bit_tc_workspace_bytes(nq, per)
            ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
            run = lambda: capi.check(L.chm_refine_1bit_tc(C.byref(view), nq, P(lut), P(cb), P(rot), P(fb_docs),
                                                          P(num), per, P(scores), P(ws), wb, st), "1-bit")
        else:
            view.full_codes, view.full_factors = codes.data_ptr(), factors.data_ptr()
            wb = L.chm_fullbit_score_tc_workspace_bytes(nq, per)
            ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
            run = lambda: capi.check(L.chm_fullbit_score_tc(C.byref(view), nq, P(rot), P(cbx), P(fb_docs), P(num),
                                                            per, P(scores), P(ws), wb, st), "full-bit")
        for _ in range(args.warmup):
            run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
            e0.record(torch.cuda.current_stream())
            for _ in range(args.steps):
                run()
            e1.record(torch.cuda.current_stream())
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        gbs = n * (16 * w + 4) / (ms / 1e3) / 1e9
        out[f"w{w}"] = {"ex_bits": ex if ex else None, "ms": round(ms, 3), "gbs": round(gbs, 1),
                        "frac": round(gbs / hbm, 4), "clocks": clk.summary()}
        del codes, ws
        torch.cuda.empty_cache()
    print(json.dumps({"metric": "LUT scoring HBM GB/s (C2 operator microbench)", "value": out["w5"]["gbs"],
                      "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "higher_is_better": True, "dtype": "u8 codes, f32 math", "data": "synthetic",
                      "config": {"workload": f"C2: {n} uniform random codes per width, lists of {tok} codes with "
                                             f"per-list fp32 factors, 32 query tokens x {nq} queries",
                                 "value_width": "w5 (ex_bits 4)"},
                      "widths": out, "peak": hbm, "peak_kind": kind, "l2": "inputs larger than L2"}), flush=True)


def profile_stages(torch, capi, index, searcher, q, cfg):
    """Runs the pipeline stage by stage on the launching stream with CUDA
    events between stages (same kernels as chm_search) and returns per-stage
    device time with each stage's algorithmic bytes / flops."""
    import ctypes as C
    L = capi.lib()
    B = q.shape[0]
    P = capi._ptr
    st = capi._stream(torch)
    dev = q.device
    p = searcher.params
    ntok = B * 32
    rot = torch.empty(ntok, 128, device=dev)
    cb1 = torch.empty(ntok, device=dev)
    cbex = torch.empty(ntok, device=dev)
    lut = torch.empty(ntok, 512, device=dev)
    labels = torch.empty(ntok, p.nprobe, dtype=torch.int32, device=dev)
    use_tc = bool(index.view.centroids_bf16) and p.nprobe <= 448
    pb = (L.chm_probe_tc_workspace_bytes if use_tc else L.chm_probe_workspace_bytes)(ntok, index.n_clusters, p.nprobe)
    pws = torch.empty(pb, dtype=torch.uint8, device=dev)

    def probe():
        if use_tc:
            return L.chm_probe_tc(P(rot), ntok, P(index.centroids), P(index.centroids_bf16), P(index.centroid_norms),
                                  P(index.centroid_norm_max), index.n_clusters, p.nprobe, P(labels), P(pws), pb, st)
        return L.chm_probe(P(rot), ntok, P(index.centroids), P(index.centroid_norms), index.n_clusters, p.nprobe,
                           P(labels), P(pws), pb, st)
    sb = L.chm_stage1_workspace_bytes(C.byref(index.view), B, p.nprobe, p.k_refine)
    # the search workspace (idle here) holds stage 1's, which dominates it
    ws_search = getattr(searcher, "_ws", None)
    sws = ws_search if ws_search is not None and ws_search.numel() >= sb else \
        torch.empty(sb, dtype=torch.uint8, device=dev)
    rd = torch.empty(B, p.k_refine, dtype=torch.int32, device=dev)
    rp = torch.empty(B, p.k_refine, device=dev)
    nr = torch.empty(B, dtype=torch.int32, device=dev)
    ob = torch.empty(B, p.k_refine, device=dev)
    fd = torch.empty(B, p.k_refine, dtype=torch.int32, device=dev)
    nf = torch.empty(B, dtype=torch.int32, device=dev)
    fs = torch.empty(B, p.k_refine, device=dev)
    res = torch.empty(B, p.k, dtype=torch.int64, device=dev)
    nres = torch.empty(B, dtype=torch.int32, device=dev)
    v = C.byref(index.view)
    fbb = L.chm_refine_tc_workspace_bytes(v, B, p.k_refine)  # room for long docs' parts, as chm_search
    fbws = torch.empty(max(fbb, 1), dtype=torch.uint8, device=dev)
    stages = [
        ("prepare", 1, lambda: L.chm_prepare_queries(P(index.flips), index.dim, index.ex_bits, P(q), ntok, P(rot),
                                                    P(cb1), P(cbex), P(lut), st)),
        ("probe", 6 if use_tc else 2, probe),
        ("stage1", stage1_launches(index, p), lambda: L.chm_stage1(v, B, P(lut), P(cb1), P(labels), p.nprobe,
                                                                   p.k_refine, P(rd), P(rp),
                                           P(nr), None, P(sws), sb, st)),
        # chm_search's choice: the tensor-core filter on batches of 16 or more
        ("refine_1bit", 7, lambda: L.chm_refine_1bit_tc(v, B, P(lut), P(cb1), P(rot), P(rd), P(nr), p.k_refine, P(ob),
                                                        P(fbws), fbb, st)) if B >= 16 else
        ("refine_1bit", 1, lambda: L.chm_refine_1bit(v, B, P(lut), P(cb1), P(rd), P(nr), p.k_refine, P(ob), st)),
        ("select_fullbit", 1, lambda: L.chm_select_fullbit(B, P(rd), P(ob), P(nr), p.k_refine, p.k_full_bit,
                                                           p.num_chunks, P(fd), P(nf), p.k_refine, st)),
        ("fullbit", 8, lambda: L.chm_fullbit_score_tc(v, B, P(rot), P(cbex), P(fd), P(nf), p.k_refine, P(fs),
                                                      P(fbws), fbb, st)),
        ("final_topk", 1, lambda: L.chm_final_topk(B, P(fd), P(fs), P(nf), p.k_refine, p.k, P(res), P(nres), st)),
    ]
    times = {n: 0.0 for n, _, _ in stages}
    # (after the runs) which queries stage 1's hash-table path redid
    table_q = torch.empty(B, dtype=torch.int32, device=dev)
    reps = 3
    stream = torch.cuda.current_stream()
    for r in range(reps + 1):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(stages) + 1)]
        evs[0].record(stream)
        for i, (n, _, f) in enumerate(stages):
            capi.check(f(), n)
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
        if r > 0:
            for i, (n, _, _) in enumerate(stages):
                times[n] += evs[i].elapsed_time(evs[i + 1]) / reps
    # algorithmic work per step
    cp = index.cluster_pos
    lens = (cp[1:] - cp[:-1]).to(torch.int64)
    lab = labels.view(B, 32, p.nprobe).to(torch.int64)
    uniq_bytes = 0
    for b in range(B):
        u = torch.unique(lab[b])
        uniq_bytes += int(lens[u].sum().item()) * 24
    nrh = nr.cpu().numpy()
    dp = index.doc_ptrs
    ref_tok = 0
    for b in range(B):
        d = rd[b, :nrh[b]].to(torch.int64)
        ref_tok += int((dp[d + 1] - dp[d]).sum().item())
    nfh = nf.cpu().numpy()
    fb_tok = 0
    for b in range(B):
        d = fd[b, :nfh[b]].to(torch.int64)
        fb_tok += int((dp[d + 1] - dp[d]).sum().item())
    w = 1 + index.ex_bits
    out = []
    for n, launches, _ in stages:
        s = {"name": n, "ms": times[n], "launches": launches, "bound": "hbm", "algo_bytes": 0, "algo_flops": 0}
        if n == "probe":
            s.update(bound="tensor", algo_flops=2.0 * ntok * index.n_clusters * 128)
        elif n == "stage1":
            s["algo_bytes"] = uniq_bytes
        elif n == "refine_1bit":
            s["algo_bytes"] = ref_tok * 24
            s["units"] = ref_tok
        elif n == "fullbit":
            s["algo_bytes"] = fb_tok * (16 * w + 4)
        out.append(s)
    capi.check(L.chm_stage1_table_queries(v, B, p.nprobe, p.k_refine, 0, P(sws), sb, P(table_q), st), "table q")
    torch.cuda.synchronize()
    for s in out:
        if s["name"] == "stage1":
            s["table_path_queries"] = int(table_q.sum().item())
    # the batch's full-bit selection and scores, for the CPU baseline's check
    extra = dict(rot=rot.view(B, 32, 128), cbex=cbex.view(B, 32), fb_docs=fd, num_fb=nf, fb_scores=fs)
    return out, extra


def stage1_launches(index, p):
    """Kernels one chm_stage1 call launches: the hash-table path's 8 (clear or
    memset, score, combine, mark, hist, pivot, compact, select; masked to the
    queries it redoes), and with the dense-bound path enabled its score and
    histogram plus pivot, compact, select, exact and final per round (a
    second round when 12,288 candidates exceed the first round's)."""
    v = index.view
    if not (v.tok_cluster and v.codes1_tok and v.max_doc_len > 0 and p.nprobe <= 128):
        return 7  # the hash-table path alone (its tables cleared by a memset)
    kc = min(max(p.k_refine + max(p.k_refine // 2, 64), p.k_refine), 12288, index.num_docs)
    rounds = 2 if min(12288, index.num_docs) > kc else 1
    return 8 + 2 + 5 * rounds


def latency_percentiles(torch, queries, search_device, barrier, n=64):
    """Wall-clock latency of one query per call (as gpu_search times it),
    synchronised on every rank."""
    lat = []
    for i in range(n + 3):
        q = queries[i % queries.shape[0]:i % queries.shape[0] + 1].contiguous()
        barrier()
        t = time.perf_counter()
        search_device(q)
        torch.cuda.synchronize()
        if i >= 3:
            lat.append((time.perf_counter() - t) * 1e3)
    lat = np.sort(np.array(lat))
    pct = lambda p: float(np.interp(p / 100 * (len(lat) - 1), np.arange(len(lat)), lat))
    return {"p50": round(pct(50), 3), "p99": round(pct(99), 3), "mean": round(float(lat.mean()), 3)}


def _host_index(index):
    from oracle import oracle as O
    return O.Index(**index.to_host())


def cpu_baseline(args, cfg, index, queries, torch, extra):
    """The reference's own CPU stage: its AVX-512 full-bit MaxSim
    (compute_full_bit_scores, search_impl.cu:510-574, through
    oracle/_ref/libchimera_ref.so) on all host cores over the docs that the
    GPU run selected for full-bit scoring, for `--cpu-sample` queries of the
    profiled batch.  The GPU full-bit scores of the same docs must equal it
    bit for bit."""
    from oracle import oracle as O
    if not O.ref_available():
        return {"value": None, "unit": "queries/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref/libchimera_ref.so not built"}
    R = O.ref()
    threads = os.cpu_count()
    S = min(args.cpu_sample, int(extra["num_fb"].shape[0]))
    full = index.full_codes.cpu().numpy().reshape(-1)
    ff = index.full_factors.cpu().numpy()
    dp = index.doc_ptrs.cpu().numpy()
    rot = extra["rot"][:S].cpu().numpy()
    cbex = extra["cbex"][:S].cpu().numpy()
    nfh = extra["num_fb"][:S].cpu().numpy()
    fd = extra["fb_docs"][:S].cpu().numpy()
    fs = extra["fb_scores"][:S].cpu().numpy()
    w = 1 + index.ex_bits
    secs, toks, docs, exact = 0.0, 0, 0, 0
    for q in range(S):
        d = np.ascontiguousarray(fd[q, :nfh[q]], np.int32)
        out = np.zeros(len(d), np.float32)
        t0 = time.perf_counter()
        R.cref_fullbit_doc_scores(np.ascontiguousarray(rot[q]), np.ascontiguousarray(cbex[q]), full, ff, dp, d,
                                  len(d), index.ex_bits, out, threads)
        secs += time.perf_counter() - t0
        toks += int((dp[d.astype(np.int64) + 1] - dp[d]).sum())
        docs += len(d)
        exact += int(np.array_equal(out.view(np.uint32), fs[q, :nfh[q]].view(np.uint32)))
    gbytes = toks * (16 * w + 4) / 1e9
    return {"value": round(S / secs, 3), "unit": "queries/s (full-bit stage)", "cores": threads,
            "kind": "reference",
            "sample": f"the reference's AVX-512 full-bit MaxSim over the docs the GPU selected, {S} queries "
                      f"({docs} docs, {toks} tokens)",
            "per_query_ms": round(secs / S * 1e3, 3), "docs_per_s": round(docs / secs, 1),
            "code_gbs": round(gbytes / secs, 3), "gpu_scores_bit_exact_queries": exact}


def oracle_parity(args, cfg, index, queries, torch, gpu_results, gt):
    """The CPU oracle (exact probe + every stage of the path, oracle/) on the
    first `--parity-queries` queries of the recall set, over the same index:
    its results against the GPU's, and both recalls on those queries."""
    from oracle import oracle as O
    P = min(args.parity_queries, 0 if gpu_results is None else gpu_results.shape[0])
    if P == 0:
        return None
    threads = os.cpu_count()
    hidx = _host_index(index)
    q = queries[:P].contiguous()
    rot = O.rotate(index.flips.cpu().numpy(), q.reshape(-1, q.shape[-1]).cpu().numpy()).reshape(P, 32, 128)
    cb1, cbex = O.query_state(rot, cfg.ex_bits)
    labels = O.probe(rot.reshape(P * 32, 128), index.centroids.cpu().numpy(), index.centroid_norms.cpu().numpy(),
                     cfg.nprobe, threads).reshape(P, 32, cfg.nprobe)
    t0 = time.perf_counter()
    res, nres = hidx.search_batch(rot, cb1, cbex, labels, cfg.nprobe, cfg.k_refine, cfg.k_full_bit,
                                  cfg.num_chunks, cfg.k, threads)
    secs = time.perf_counter() - t0
    same = sum(int(np.array_equal(res[i, :nres[i]], gpu_results[i, :nres[i]])) for i in range(P))
    return {"queries": P, "bit_exact": same,
            "oracle_recall@100": round(W_recall(np.stack(gt[:P]), res, cfg.k), 4),
            "gpu_recall@100": round(W_recall(np.stack(gt[:P]), gpu_results[:P], cfg.k), 4),
            "oracle": "plain-C restatement (oracle/), exact probe, all host threads",
            "oracle_qps": round(P / secs, 3)}


def W_module():
    from chimera_b200 import workloads
    return workloads


def W_recall(gt, res, k):
    from chimera_b200 import workloads as W
    return W.recall_at_k(gt, res, k)


def run_reference(args, cfg, index, queries, torch, emb, ptr_full, sc=None):
    """The reference's own search path (oracle/ref_search.cu: its CUDA kernels,
    host flow and AVX-512 full-bit scorer; an exact cuBLAS probe stands in for
    cuVS CAGRA, which is not installable here), one query per call as
    gpu_search times it (cpp/apps/search.cpp:96-106).  A step is
    `--ref-sample` queries; value = queries / sum of their latencies."""
    from oracle import oracle as O
    import torch.cuda
    W = args.warmup
    steps = args.steps
    per = args.ref_sample
    wl = (f"{cfg.name}: {cfg.num_docs} docs, {int(index.n_tokens)} tokens, {cfg.n_clusters} clusters, "
          f"ex_bits {cfg.ex_bits}, nprobe {cfg.nprobe}, k_refine {cfg.k_refine}, k_full_bit {cfg.k_full_bit}, "
          f"k {cfg.k}")
    base = {"impl": "reference", "metric": METRIC.get(cfg.name, f"QPS at Recall@100 ({cfg.name})"), "unit": "queries/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": steps, "warmup": W,
            "higher_is_better": True, "data": "synthetic"}
    if not O.ref_search_available():
        print(json.dumps({**base, "unavailable": "oracle/_ref/libchimera_ref_search.so was not built "
                                                 "(the reference tree was absent at build time)"}), flush=True)
        return
    nq_total = queries.shape[0]
    # warm-up on the last queries; the timed steps run queries 0, 1, 2, ...,
    # so that recall covers the first --recall-queries queries like our arm's
    timed_idx = [i % nq_total for i in range(steps * per)]
    warm_idx = [(nq_total - 1 - i) % nq_total for i in range(W * per)]
    qidx = warm_idx + timed_idx
    timed = sorted(set(timed_idx))
    if emb is not None:
        gt_list = ground_truth(torch, emb, ptr_full, queries, cfg.k, timed)
    else:
        gt_list = W_module().ground_truth_streamed(sc, queries[timed], cfg.k)
    gt = dict(zip(timed, gt_list))
    del emb
    torch.cuda.empty_cache()
    hidx = _host_index(index)
    threads = os.cpu_count()
    sess = O.RefSearchSession(hidx, index.centroids.cpu().numpy(), index.centroid_norms.cpu().numpy(), cfg.dim,
                              cfg.nprobe, cfg.k_refine, threads)
    qh = queries.cpu().numpy()
    lat, res, hit = [], {}, 0
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        for n, qi in enumerate(qidx):
            t0 = time.perf_counter()
            r, _, _ = sess.search(qh[qi], cfg.nprobe, cfg.k_refine, cfg.k_full_bit, cfg.num_chunks, cfg.k)
            dt = time.perf_counter() - t0
            if n >= W * per:
                lat.append(dt)
                res[qi] = r
    sess.close()
    v = len(lat) / sum(lat)
    ls = np.sort(np.array(lat) * 1e3)
    pct = lambda p: float(np.interp(p / 100 * (len(ls) - 1), np.arange(len(ls)), ls))
    rec = W_recall(np.stack([gt[q] for q in timed]), [res[q] for q in timed], cfg.k)
    same = [q for q in timed if q < args.recall_queries]
    rec_same = W_recall(np.stack([gt[q] for q in same]), [res[q] for q in same], cfg.k) if same else None
    line = {**base, "value": round(v, 3), "ms_per_step": round(float(np.sum(ls)) / steps, 3),
            "config": {"workload": wl, "implementation":
                       "reference kernels (kernels.cu, unchanged) + exact-probe shim (cuBLAS SGEMM + select, "
                       "standing in for cuVS CAGRA) + the reference's AVX-512 full-bit scorer on the host, "
                       "one query per call (search_impl.cu:46-574)",
                       "queries_per_step": per, "recall@100": round(rec_same, 4) if same else None,
                       "recall_queries": len(same), "recall@100_all_timed": round(rec, 4),
                       "timed_queries": len(timed),
                       "latency_ms_single_query": {"p50": round(pct(50), 3), "p99": round(pct(99), 3),
                                                   "mean": round(float(ls.mean()), 3)}},
            "cpu_baseline": {"value": round(v, 3), "unit": "queries/s", "cores": threads, "kind": "reference",
                             "sample": f"{per} queries per step, one per call; the full-bit stage on "
                                       f"{threads} host threads"},
            "e2e": {"value": round(v, 3), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
