"""Shared test corpora: seeded synthetic data (chimera_b200.workloads) and an
index built on the CPU by the oracle (exact assignment, reference-order
rotation and RaBitQ encoding), cached per session."""
import ctypes as C
import functools
import os

import numpy as np

from chimera_b200 import capi, workloads as W
from oracle import oracle as O


@functools.lru_cache(maxsize=None)
def corpus(name="small", seed=0, dim=128, ex_bits=None):
    cfg = W.CONFIGS[name]
    if ex_bits is not None:
        import dataclasses
        cfg = dataclasses.replace(cfg, ex_bits=ex_bits)
    emb, dl, qs = W.generate_numpy(cfg, seed)
    if dim != 128:
        emb = np.ascontiguousarray(emb[:, :dim])
        emb /= np.linalg.norm(emb, axis=1, keepdims=True)
        qs = np.ascontiguousarray(qs[:, :, :dim])
        qs /= np.linalg.norm(qs, axis=2, keepdims=True)
    n = emb.shape[0]
    flips = capi.fhtkac_flips(42)
    ids = capi.sample_centroids(n, cfg.n_clusters, 42)
    cent = np.ascontiguousarray(emb[ids])
    assign = O.assign(emb, cent)
    pos, inv = O.cluster_order(assign, cfg.n_clusters)
    L = O.lib()
    L.orc_rotate_batch.argtypes = [O._u8p, O._f32p, C.c_int64, C.c_int, O._f32p, C.c_int]
    L.orc_encode_batch.argtypes = [O._f32p, C.c_int64, C.c_int, O._u8p, O._f32p, O._u8p, O._f32p, C.c_int]
    rot = np.zeros((n, 128), np.float32)
    L.orc_rotate_batch(flips, np.ascontiguousarray(emb), n, dim, rot, os.cpu_count())
    fb = 128 * (1 + cfg.ex_bits) // 8
    c1 = np.zeros((n, 16), np.uint8)
    f1 = np.zeros(n, np.float32)
    full = np.zeros((n, fb), np.uint8)
    ff = np.zeros(n, np.float32)
    L.orc_encode_batch(rot, n, cfg.ex_bits, c1, f1, full, ff, os.cpu_count())
    ptr = W.doc_ptrs(dl)
    owner = np.repeat(np.arange(len(dl)), dl).astype(np.int32)
    tok2pos = np.zeros(n, np.uint32)
    tok2pos[inv] = np.arange(n, dtype=np.uint32)
    crot = np.zeros((cfg.n_clusters, 128), np.float32)
    L.orc_rotate_batch(flips, cent, cfg.n_clusters, dim, crot, os.cpu_count())
    cnorm = O.dot_norms(crot)
    qrot = np.zeros((qs.shape[0] * 32, 128), np.float32)
    L.orc_rotate_batch(flips, np.ascontiguousarray(qs.reshape(-1, dim)), qs.shape[0] * 32, dim, qrot,
                       os.cpu_count())
    qrot = qrot.reshape(qs.shape[0], 32, 128)
    cb1, cbex = O.query_state(qrot, cfg.ex_bits)
    labels = O.probe(qrot.reshape(-1, 128), crot, cnorm, cfg.nprobe).reshape(qs.shape[0], 32, cfg.nprobe)
    index = O.Index(cluster_pos=pos, codes1=c1[inv], factor1=f1[inv], doc_ids=owner[inv], tok2pos=tok2pos,
                    doc_ptrs=ptr, full_codes=full, full_factors=ff, ex_bits=cfg.ex_bits)
    return dict(cfg=cfg, emb=emb, doclens=dl, queries=qs, flips=flips, centroid_ids=ids, assign=assign,
                cluster_pos=pos, inv=inv, rot=rot, codes1_tok=c1, f1_tok=f1, full=full, ff=ff,
                centroids_rot=crot, cnorm=cnorm, qrot=qrot, cb1=cb1, cbex=cbex, labels=labels,
                index=index, dim=dim, ptr=ptr, owner=owner, tok2pos=tok2pos)


def oracle_search(c, q, **over):
    cfg = c["cfg"]
    kw = dict(nprobe=cfg.nprobe, k_refine=cfg.k_refine, k_full_bit=cfg.k_full_bit,
              num_chunks=cfg.num_chunks, k=cfg.k)
    kw.update(over)
    labels = c["labels"][q]
    if kw["nprobe"] != cfg.nprobe:
        labels = O.probe(c["qrot"][q], c["centroids_rot"], c["cnorm"], kw["nprobe"])
    return c["index"].search_one(c["qrot"][q], c["cb1"][q], c["cbex"][q], labels, kw["nprobe"],
                                 kw["k_refine"], kw["k_full_bit"], kw["num_chunks"], kw["k"])


def device_index(c, torch):
    return capi.DeviceIndex.from_host(
        cluster_pos=c["cluster_pos"], codes1=c["index"].codes1, factor1=c["index"].factor1,
        doc_ids=c["index"].doc_ids, tok2pos=c["tok2pos"], doc_ptrs=c["ptr"], full_codes=c["full"],
        full_factors=c["ff"], centroids_rot=c["centroids_rot"], flips=c["flips"], dim=c["dim"],
        ex_bits=c["cfg"].ex_bits)
