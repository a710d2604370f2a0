"""A stage backend for chimera_b200.sharded.ShardedPipeline built from the
oracle (CPU, test infrastructure): each stage of one rank computed by the
plain-C restatement on that rank's document shard.  With it the sharding
protocol (exchange steps, merge rule, ownership masks, overflow folding) runs
over gloo on CPU ranks and is compared with the oracle's single-index search.
"""
import numpy as np
import torch

from oracle import oracle as O


class OracleShardBackend:
    def __init__(self, shard_index, doc_bases, rank, *, flips, centroids_rot, cnorm, ex_bits, nprobe, k_refine,
                 k_full_bit, num_chunks, k):
        self.ix = shard_index
        self.bases = list(doc_bases)
        self.base = int(doc_bases[rank])
        self.n_local = int(doc_bases[rank + 1] - doc_bases[rank])
        self.flips, self.cents, self.cnorm, self.ex_bits = flips, centroids_rot, cnorm, ex_bits
        self.nprobe, self.kr, self.kfb, self.nch, self.k = nprobe, k_refine, k_full_bit, num_chunks, k

    def prepare(self, queries):
        q = queries.numpy()
        self.B = q.shape[0]
        self.rot = O.rotate(self.flips, q.reshape(-1, q.shape[-1])).reshape(self.B * 32, 128)
        self.cb1, self.cbex = O.query_state(self.rot, self.ex_bits)
        self.luts = O.build_lut(self.rot)
        return None

    def probe(self, st, lo, hi, per):
        out = torch.zeros(per, self.nprobe, dtype=torch.int32)
        if hi > lo:
            lab = O.probe(self.rot[lo:hi], self.cents, self.cnorm, self.nprobe)
            out[:hi - lo] = torch.from_numpy(lab.astype(np.int64).astype(np.int32))
        return out

    def stage1(self, st, labels, extra):
        B, kr = self.B, self.kr
        lab = labels.numpy().astype(np.uint32).reshape(B, 32, self.nprobe)
        docs = torch.zeros(B, kr, dtype=torch.int32)
        part = torch.zeros(B, kr, dtype=torch.float32)
        cnt = torch.zeros(B, dtype=torch.int32)
        for b in range(B):
            s = slice(32 * b, 32 * (b + 1))
            tr = self.ix.search_one(self.rot[s], self.cb1[s], self.cbex[s], lab[b], self.nprobe, kr,
                                    min(self.kfb, kr), self.nch, self.k)
            n = tr["n_refined"]
            cnt[b] = n
            docs[b, :n] = torch.from_numpy(tr["refined_docs"])
            part[b, :n] = torch.from_numpy(tr["refined_partial"])
        return docs, part, cnt, torch.zeros(B, dtype=torch.int32)

    def merge_refined(self, g_docs, g_partial, g_counts):
        G, B, kr = g_docs.shape
        out_d = torch.zeros(B, kr, dtype=torch.int32)
        out_p = torch.zeros(B, kr, dtype=torch.float32)
        out_c = torch.zeros(B, dtype=torch.int32)
        for q in range(B):
            d, p = [], []
            for s in range(G):
                n = int(g_counts[s, q])
                d.append(g_docs[s, q, :n].numpy().astype(np.int64) + self.bases[s])
                p.append(g_partial[s, q, :n].numpy())
            d, p = np.concatenate(d), np.concatenate(p)
            order = np.lexsort((d, -p))[:kr]  # partial desc, doc asc
            out_c[q] = len(order)
            out_d[q, :len(order)] = torch.from_numpy(d[order].astype(np.int32))
            out_p[q, :len(order)] = torch.from_numpy(p[order])
        return out_d, out_p, out_c

    def localize(self, gdocs, counts):
        g = gdocs.numpy().astype(np.int64)
        out = np.full(g.shape, -1, np.int32)
        for q in range(g.shape[0]):
            n = int(counts[q])
            own = (g[q, :n] >= self.base) & (g[q, :n] < self.base + self.n_local)
            out[q, :n][own] = (g[q, :n][own] - self.base).astype(np.int32)
        return torch.from_numpy(out)

    def refine_1bit(self, st, local, counts):
        out = torch.full((self.B, self.kr), -np.inf, dtype=torch.float32)
        for q in range(self.B):
            s = slice(32 * q, 32 * (q + 1))
            for r in range(int(counts[q])):
                d = int(local[q, r])
                if d >= 0:
                    out[q, r] = self.ix.onebit_doc_score(self.luts[s], self.cb1[s], d)
        return out

    def select_fullbit(self, rdocs, onebit, counts):
        """Progressive chunked selection (search_impl.cu:341-494), ties to
        the lower refined index, as the oracle's search_one does it."""
        fd = torch.zeros(self.B, self.kr, dtype=torch.int32)
        nf = torch.zeros(self.B, dtype=torch.int32)
        for q in range(self.B):
            R = int(counts[q])
            if R == 0:
                continue
            sc = onebit[q, :R].numpy()
            T = min(self.kfb, R)
            nch = min(self.nch, R)
            cs = (R + nch - 1) // nch
            order = np.lexsort((np.arange(R), -sc))
            chosen = np.zeros(R, bool)
            for c in range(nch):
                end = min((c + 1) * cs, R)
                cum = min(T * (c + 1) // nch, min(T, end))
                chosen[order[order < end][:cum]] = True
            sel = np.nonzero(chosen)[0]
            nf[q] = len(sel)
            fd[q, :len(sel)] = rdocs[q, torch.from_numpy(sel)]
        return fd, nf

    def fullbit(self, st, fb_local, nf):
        out = torch.full((self.B, self.kr), -np.inf, dtype=torch.float32)
        for q in range(self.B):
            s = slice(32 * q, 32 * (q + 1))
            for i in range(int(nf[q])):
                d = int(fb_local[q, i])
                if d >= 0:
                    out[q, i] = self.ix.fullbit_doc_score(self.rot[s], self.cbex[s], d)
        return out

    def final(self, fb_docs, fbs, nf):
        res = torch.full((self.B, self.k), -1, dtype=torch.int64)
        nres = torch.zeros(self.B, dtype=torch.int32)
        for q in range(self.B):
            n = int(nf[q])
            d = fb_docs[q, :n].numpy().astype(np.int64)
            s = fbs[q, :n].numpy()
            order = np.lexsort((-d, -s))[:self.k]  # score desc, doc desc
            nres[q] = len(order)
            res[q, :len(order)] = torch.from_numpy(d[order])
        return res, nres

    def fold_flags(self, nres, flags):
        return torch.where(flags != 0, torch.full_like(nres, -1), nres)
