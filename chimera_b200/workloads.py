"""Seeded synthetic corpora for the benchmark configurations.

No public dataset ships with the reference (its CLI expects LoTTE-style
files that are not available here), so every configuration is a synthetic
stand-in with the shapes and distributions the benchmark plan names:

* doc lengths: clip(round(N(mu, sd)), lo, hi), or a clipped log-normal for
  the long-document corpus;
* token embeddings: a K-component isotropic Gaussian mixture (centres
  N(0, 1)^128, within-component sd 0.3, component drawn uniformly per
  token), L2-normalised;
* queries: a random target document's first <= 32 tokens plus N(0, 0.1)
  noise, renormalised, padded with fresh unit-norm random tokens.

``generate_numpy`` is the reference generator (numpy PCG64, used for the
small configurations and the test fixtures).  ``generate_torch`` follows
the same recipe with torch's CUDA generator for the corpora that are too
large to build on the host; its streams differ from numpy's, so the two are
separate seeded corpora of identical distribution.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np


@dataclasses.dataclass(frozen=True)
class Config:
    name: str
    num_docs: int
    doclen: tuple  # ("normal", mu, sd, lo, hi) | ("lognormal", median, sigma, lo, hi)
    components: int
    num_queries: int
    n_clusters: int
    ex_bits: int
    nprobe: int
    k_refine: int
    k_full_bit: int
    num_chunks: int = 5
    k: int = 100
    dim: int = 128
    qlen: int = 32
    within_sd: float = 0.3
    query_noise: float = 0.1

    def search_kwargs(self):
        return dict(nprobe=self.nprobe, k_refine=self.k_refine, k_full_bit=self.k_full_bit,
                    num_chunks=self.num_chunks)


CONFIGS = {
    # small CPU-runnable corpus
    "c1": Config("c1", 10_000, ("normal", 64, 20, 8, 180), 1024, 64, 4096, 4, 32, 1000, 100),
    # single-GPU passage-scale corpus (the headline)
    "c3": Config("c3", 1_000_000, ("normal", 64, 20, 8, 180), 16384, 1024, 262144, 4, 128,
                 3000, 300),
    # long-document corpus
    "c4": Config("c4", 200_000, ("lognormal", 600, 0.55, 300, 2000), 32768, 4096, 700_000, 2,
                 64, 2000, 200),
    # large sharded corpus
    "c5": Config("c5", 8_800_000, ("normal", 68, 22, 8, 180), 65536, 8192, 4_194_304, 4, 128,
                 3000, 300),
    # C3's per-query shape (mean list length 244, nprobe 128, k_refine 3000) on 1/8 of its corpus:
    # the small case for full ncu captures (about 1 GB on the device)
    "c3s": Config("c3s", 125_000, ("normal", 64, 20, 8, 180), 2048, 128, 32768, 4, 128, 3000, 300),
    # C5's density of centroids per mixture component (64) and its query and
    # search shape on 1/64 of its documents: the probe's near-ties as at C5
    "c5s": Config("c5s", 137_500, ("normal", 68, 22, 8, 180), 1024, 1024, 65_536, 4, 128, 3000, 300),
    # test-sized corpora with the same recipe
    "mini": Config("mini", 300, ("normal", 64, 20, 8, 180), 64, 6, 128, 4, 16, 60, 20, 5, 10),
    "small": Config("small", 2000, ("normal", 64, 20, 8, 180), 256, 16, 512, 4, 24, 300, 60,
                    5, 20),
    # sparse probing (4 of 4,096 lists per query token, as C3 probes 128 of
    # 262,144): a doc rarely has two tokens in one query token's lists
    "sparse": Config("sparse", 1500, ("normal", 64, 20, 8, 180), 256, 16, 4096, 4, 4, 100, 30, 5, 20),
    # long documents (several 128-token tiles each), ex_bits 2
    "long": Config("long", 300, ("lognormal", 200, 0.6, 100, 600), 64, 6, 256, 2, 16, 120, 30, 5, 10),
}


def doclens_numpy(cfg: Config, rng: np.random.Generator) -> np.ndarray:
    kind = cfg.doclen[0]
    if kind == "normal":
        _, mu, sd, lo, hi = cfg.doclen
        x = np.rint(rng.normal(mu, sd, cfg.num_docs))
    else:
        _, median, sigma, lo, hi = cfg.doclen
        x = np.rint(rng.lognormal(math.log(median), sigma, cfg.num_docs))
    return np.clip(x, lo, hi).astype(np.int32)


def _normalise(x: np.ndarray) -> np.ndarray:
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


def generate_numpy(cfg: Config, seed: int = 0, chunk: int = 1 << 20):
    """Returns (embeddings [N, dim] f32, doclens [M] i32, queries [Q, 32, dim] f32)."""
    rng = np.random.default_rng(seed)
    doclens = doclens_numpy(cfg, rng)
    n = int(doclens.sum())
    centres = rng.standard_normal((cfg.components, cfg.dim)).astype(np.float32)
    emb = np.empty((n, cfg.dim), np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        comp = rng.integers(0, cfg.components, e - s)
        x = centres[comp] + np.float32(cfg.within_sd) * rng.standard_normal(
            (e - s, cfg.dim)).astype(np.float32)
        emb[s:e] = _normalise(x)
    ptr = np.zeros(cfg.num_docs + 1, np.int64)
    np.cumsum(doclens, out=ptr[1:])
    queries = np.empty((cfg.num_queries, cfg.qlen, cfg.dim), np.float32)
    targets = rng.integers(0, cfg.num_docs, cfg.num_queries)
    for i, d in enumerate(targets):
        take = min(cfg.qlen, int(doclens[d]))
        base = emb[ptr[d]:ptr[d] + take]
        noisy = base + np.float32(cfg.query_noise) * rng.standard_normal(base.shape).astype(np.float32)
        queries[i, :take] = _normalise(noisy)
        if take < cfg.qlen:
            queries[i, take:] = _normalise(
                rng.standard_normal((cfg.qlen - take, cfg.dim)).astype(np.float32))
    return emb, doclens, queries


def generate_torch(cfg: Config, seed: int = 0, device: str = "cuda", chunk: int = 1 << 22):
    """Same recipe on the GPU (torch CUDA generator); returns device tensors
    (embeddings [N, dim] f32, doclens [M] i32, queries [Q, 32, dim] f32)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    kind = cfg.doclen[0]
    if kind == "normal":
        _, mu, sd, lo, hi = cfg.doclen
        x = torch.randn(cfg.num_docs, generator=g, device=device, dtype=torch.float64) * sd + mu
    else:
        _, median, sigma, lo, hi = cfg.doclen
        x = torch.exp(torch.randn(cfg.num_docs, generator=g, device=device,
                                  dtype=torch.float64) * sigma + math.log(median))
    doclens = torch.clamp(torch.round(x), lo, hi).to(torch.int32)
    n = int(doclens.sum().item())
    centres = torch.randn(cfg.components, cfg.dim, generator=g, device=device)
    emb = torch.empty(n, cfg.dim, device=device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        comp = torch.randint(0, cfg.components, (e - s,), generator=g, device=device)
        v = centres[comp] + cfg.within_sd * torch.randn(e - s, cfg.dim, generator=g, device=device)
        emb[s:e] = v / v.norm(dim=1, keepdim=True)
    ptr = torch.zeros(cfg.num_docs + 1, dtype=torch.int64, device=device)
    ptr[1:] = torch.cumsum(doclens.to(torch.int64), 0)
    targets = torch.randint(0, cfg.num_docs, (cfg.num_queries,), generator=g, device=device)
    take = torch.clamp(doclens[targets].to(torch.int64), max=cfg.qlen)
    j = torch.arange(cfg.qlen, device=device)
    src = ptr[targets][:, None] + torch.minimum(j[None, :], take[:, None] - 1)
    base = emb[src]                                               # [Q, 32, dim]
    noisy = base + cfg.query_noise * torch.randn(base.shape, generator=g, device=device)
    noisy = noisy / noisy.norm(dim=2, keepdim=True)
    pad = torch.randn(base.shape, generator=g, device=device)
    pad = pad / pad.norm(dim=2, keepdim=True)
    queries = torch.where((j[None, :] < take[:, None])[..., None], noisy, pad)
    return emb, doclens, queries.contiguous()


class StreamedCorpus:
    """generate_torch's corpus, produced chunk by chunk for corpora whose
    embeddings do not fit on one device (C5: about 600M tokens x 512 B).

    A first pass draws everything in generate_torch's order and records the
    generator state at the start of every embedding chunk; any chunk can then
    be regenerated with the same values.  The doc lengths, the embeddings
    (chunk by chunk) and the queries equal generate_torch's with the same
    seed and chunk size."""

    def __init__(self, cfg: Config, seed: int = 0, device: str = "cuda", chunk: int = 1 << 22):
        import torch
        self.cfg, self.chunk, self.device = cfg, chunk, device
        self._torch = torch
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        kind = cfg.doclen[0]
        if kind == "normal":
            _, mu, sd, lo, hi = cfg.doclen
            x = torch.randn(cfg.num_docs, generator=g, device=device, dtype=torch.float64) * sd + mu
        else:
            _, median, sigma, lo, hi = cfg.doclen
            x = torch.exp(torch.randn(cfg.num_docs, generator=g, device=device,
                                      dtype=torch.float64) * sigma + math.log(median))
        self.doclens = torch.clamp(torch.round(x), lo, hi).to(torch.int32)
        self.n = int(self.doclens.sum().item())
        self.centres = torch.randn(cfg.components, cfg.dim, generator=g, device=device)
        # the chunks' draws, recorded and skipped (the values are drawn and dropped
        # so that the generator advances exactly as generate_torch's does)
        self.states = []
        for s in range(0, self.n, chunk):
            e = min(self.n, s + chunk)
            self.states.append(g.get_state())
            torch.randint(0, cfg.components, (e - s,), generator=g, device=device)
            torch.randn(e - s, cfg.dim, generator=g, device=device)
        self.ptr = torch.zeros(cfg.num_docs + 1, dtype=torch.int64, device=device)
        self.ptr[1:] = torch.cumsum(self.doclens.to(torch.int64), 0)
        targets = torch.randint(0, cfg.num_docs, (cfg.num_queries,), generator=g, device=device)
        self._take = torch.clamp(self.doclens[targets].to(torch.int64), max=cfg.qlen)
        j = torch.arange(cfg.qlen, device=device)
        self._src = self.ptr[targets][:, None] + torch.minimum(j[None, :], self._take[:, None] - 1)
        shape = (cfg.num_queries, cfg.qlen, cfg.dim)
        self._noise = torch.randn(shape, generator=g, device=device)
        self._pad = torch.randn(shape, generator=g, device=device)
        self._queries = None

    @property
    def num_chunks(self) -> int:
        return len(self.states)

    def chunk_at(self, i: int):
        """Tokens [i * chunk, min(n, (i + 1) * chunk)) as a [m, dim] f32 tensor."""
        torch = self._torch
        cfg = self.cfg
        s = i * self.chunk
        e = min(self.n, s + self.chunk)
        g = torch.Generator(device=self.device)
        g.set_state(self.states[i])
        comp = torch.randint(0, cfg.components, (e - s,), generator=g, device=self.device)
        v = self.centres[comp] + cfg.within_sd * torch.randn(e - s, cfg.dim, generator=g, device=self.device)
        return v / v.norm(dim=1, keepdim=True)

    def chunks(self, lo: int = 0, hi: int | None = None):
        """Yields (s, e, x): the tokens of [lo, hi) in order, x = rows s..e-1."""
        hi = self.n if hi is None else hi
        for i in range(lo // self.chunk, (hi + self.chunk - 1) // self.chunk):
            s0 = i * self.chunk
            x = self.chunk_at(i)
            s, e = max(lo, s0), min(hi, s0 + x.shape[0])
            if s < e:
                yield s, e, x[s - s0:e - s0]

    def gather(self, ids):
        """Rows `ids` (device int64 tensor of token ids) in one pass over the chunks."""
        torch = self._torch
        ids = ids.to(self.device)
        out = torch.empty(ids.shape[0], self.cfg.dim, device=self.device)
        order = torch.argsort(ids)
        sid = ids[order]
        for i in range(self.num_chunks):
            s0 = i * self.chunk
            a = int(torch.searchsorted(sid, s0).item())
            b = int(torch.searchsorted(sid, s0 + self.chunk).item())
            if a < b:
                out[order[a:b]] = self.chunk_at(i)[sid[a:b] - s0]
        return out

    def queries(self):
        """generate_torch's queries [Q, 32, dim]."""
        if self._queries is None:
            torch = self._torch
            cfg = self.cfg
            base = self.gather(self._src.reshape(-1)).reshape(cfg.num_queries, cfg.qlen, cfg.dim)
            noisy = base + cfg.query_noise * self._noise
            noisy = noisy / noisy.norm(dim=2, keepdim=True)
            pad = self._pad / self._pad.norm(dim=2, keepdim=True)
            j = torch.arange(cfg.qlen, device=self.device)
            self._queries = torch.where((j[None, :] < self._take[:, None])[..., None], noisy, pad).contiguous()
        return self._queries


def ground_truth_streamed(corpus: "StreamedCorpus", queries, k: int, group: int = 32):
    """Exact fp32 MaxSim top-k of `queries` ([Q, 32, dim] device tensor) over
    the streamed corpus, one pass over its chunks: per chunk and group of
    queries the token scores, a per-(query token, doc) max, and per complete
    doc the sum over query tokens, merged into a running top-k.  A doc that
    continues into the next chunk carries its partial maxima over."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    Q, L, D = queries.shape
    ptr = corpus.ptr
    groups = [list(range(a, min(Q, a + group))) for a in range(0, Q, group)]
    top_v = [torch.full((len(gq), k), -float("inf"), device=queries.device) for gq in groups]
    top_i = [torch.zeros((len(gq), k), dtype=torch.int64, device=queries.device) for gq in groups]
    carry = [None] * len(groups)
    for s, e, x in corpus.chunks():
        d0 = int(torch.searchsorted(ptr, s, right=True).item()) - 1
        d1 = int(torch.searchsorted(ptr, e - 1, right=True).item()) - 1
        owner = torch.repeat_interleave(torch.arange(d1 - d0 + 1, device=x.device),
                                        torch.clamp(torch.minimum(ptr[d0 + 1:d1 + 2], torch.tensor(e, device=x.device))
                                                    - torch.maximum(ptr[d0:d1 + 1], torch.tensor(s, device=x.device)),
                                                    min=0))
        last_complete = int(ptr[d1 + 1].item()) == e
        ndoc = d1 - d0 + 1
        for gi, gq in enumerate(groups):
            qg = queries[gq].reshape(-1, D)
            sc = qg @ x.T                                                  # [G*32, m]
            best = torch.full((qg.shape[0], ndoc), -float("inf"), device=x.device)
            best.scatter_reduce_(1, owner.unsqueeze(0).expand(qg.shape[0], -1), sc, reduce="amax")
            del sc
            if carry[gi] is not None:
                best[:, 0] = torch.maximum(best[:, 0], carry[gi])
            nc = ndoc if last_complete else ndoc - 1
            carry[gi] = None if last_complete else best[:, ndoc - 1].clone()
            if nc > 0:
                score = best[:, :nc].view(len(gq), L, nc).sum(1)
                v = torch.cat([top_v[gi], score], 1)
                i = torch.cat([top_i[gi], torch.arange(d0, d0 + nc, device=x.device).expand(len(gq), -1)], 1)
                tv, ti = torch.topk(v, k, dim=1)
                top_v[gi], top_i[gi] = tv, torch.gather(i, 1, ti)
    return [row.cpu().numpy() for gi in range(len(groups)) for row in top_i[gi]]


def doc_ptrs(doclens) -> np.ndarray:
    d = np.asarray(doclens, np.int64)
    p = np.zeros(d.shape[0] + 1, np.int64)
    np.cumsum(d, out=p[1:])
    return p


def maxsim_ground_truth_numpy(emb, doclens, queries, k=100):
    """Exact fp32 MaxSim top-k (brute force, small corpora only)."""
    ptr = doc_ptrs(doclens)
    m = len(doclens)
    owner = np.repeat(np.arange(m), doclens)
    out = np.zeros((queries.shape[0], k), np.int64)
    for i, q in enumerate(queries):
        s = emb @ q.T                                   # [N, 32]
        best = np.full((m, q.shape[0]), -np.inf, np.float32)
        np.maximum.at(best, owner, s)
        score = best.sum(1)
        order = np.lexsort((np.arange(m), -score))
        out[i] = order[:k]
    del ptr
    return out


def recall_at_k(gt: np.ndarray, results, k: int) -> float:
    """|top-k ∩ GT top-k| / (Q * k), as cpp/apps/utils.cpp:265-290 computes it."""
    hit = 0
    for g, r in zip(gt, results):
        hit += len(set(int(x) for x in list(r)[:k]) & set(int(x) for x in g[:k]))
    return hit / (len(results) * k)
