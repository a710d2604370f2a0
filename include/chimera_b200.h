/*
 * chimera_b200 -- C ABI of the B200-native Chimera search path.
 *
 * Every entry point takes plain device pointers and sizes, runs
 * asynchronously on the given CUDA stream, allocates nothing (scratch is a
 * caller-provided workspace), and returns a chm_status instead of throwing.
 * The host C++ layer (include/chimera/chimera_index.cuh) turns statuses into
 * the reference's exception types.
 *
 * Each function names the reference interface it replaces (paths inside the
 * Chimera project, https://github.com/iidyc/Chimera).
 */
#ifndef CHIMERA_B200_H
#define CHIMERA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CHM_PADDED_DIM 128  /* cpp/include/chimera/config.cuh:7 */
#define CHM_QLEN 32         /* cpp/include/chimera/config.cuh:8 */
#define CHM_MAX_NPROBE 1024 /* reference: 512 and unchecked (kernels.cuh:64) */
#define CHM_MAX_K_REFINE 8192
#define CHM_MAX_K 8192

typedef enum {
    CHM_OK = 0,
    CHM_ERR_INVALID = 1,   /* bad argument (reference: std::invalid_argument) */
    CHM_ERR_CAPACITY = 2,  /* workspace or table too small */
    CHM_ERR_CUDA = 3,      /* CUDA launch/runtime failure */
    CHM_ERR_TIMEOUT = 4,   /* a bounded wait ran out */
    CHM_ERR_UNSUPPORTED = 5
} chm_status;

/* Device-resident index (all pointers are device memory).
 * Layouts are the reference's on-disk layouts (build_index.cu:470-498):
 * 1-bit data in cluster order, full codes in token order. */
typedef struct {
    int64_t n_tokens;
    int64_t num_docs;
    int64_t n_clusters;
    int32_t ex_bits;             /* 1..7; full codes use 1 + ex_bits bits/dim */
    int32_t dim;                 /* raw embedding dimension, 64..128 */
    int32_t max_list_len;        /* longest inverted list */
    int32_t max_doc_len;         /* longest document (0: unknown; stage 1 then
                                    uses its hash-table path only) */
    const int64_t* cluster_pos;  /* [n_clusters + 1] list offsets (ivf.bin) */
    const uint8_t* codes1;       /* [n_tokens * 16] 1-bit codes, cluster order */
    const float* factor1;        /* [n_tokens] 1-bit factors, cluster order */
    const int32_t* doc_ids;      /* [n_tokens] owning doc, cluster order */
    const uint32_t* tok2pos;     /* [n_tokens] token id -> cluster position */
    const int64_t* doc_ptrs;     /* [num_docs + 1] token offsets of documents */
    const uint8_t* full_codes;   /* [n_tokens * 16 * (1 + ex_bits)] token order */
    const float* full_factors;   /* [n_tokens] token order */
    const float* centroids;      /* [n_clusters * 128] rotated centroids, fp32 */
    const float* centroid_norms; /* [n_clusters] ||c||^2 (sequential fma) */
    const uint8_t* flips;        /* [64] FhtKac sign flips (doc_1bit.bin) */
    const void* centroids_bf16;  /* [n_clusters * 128] bf16 copy for the tensor-core
                                    probe; NULL selects the exact SIMT probe */
    const float* centroid_norm_max; /* device scalar max ||c||^2 (with centroids_bf16) */
    /* The 1-bit codes and factors again in token order (a document's tokens
     * contiguous), read by the refinement stage as one span per document.
     * Built from the cluster-ordered arrays by chm_token_order_1bit.  NULL:
     * refinement gathers through tok2pos (the reference's layout,
     * kernels.cu:580-600). */
    const uint8_t* codes1_tok;   /* [n_tokens * 16] */
    const float* factor1_tok;    /* [n_tokens] */
    /* Cluster of every token, token order (IVF_PG's assignment,
     * ivf_pg.cpp:110-126).  With codes1_tok, factor1_tok and max_doc_len it
     * enables stage 1's dense-bound path; NULL: hash-table path only. */
    const uint32_t* tok_cluster; /* [n_tokens] */
} chm_index;

typedef struct {
    int32_t nprobe;      /* SearchOptions::nprobe (chimera_index.cuh:27) */
    int32_t k_refine;    /* SearchOptions::k_refine */
    int32_t k_full_bit;  /* SearchOptions::k_full_bit */
    int32_t num_chunks;  /* SearchOptions::num_chunks */
    int32_t k;           /* results per query */
    int32_t batch;       /* queries processed per pipeline pass */
    int32_t table_log2_extra; /* grow stage-1 tables by 2^x (retry on overflow) */
} chm_search_params;

/* Library version and the last CUDA error string seen on this thread. */
const char* chm_version(void);
const char* chm_last_error(void);

/* Workspace bytes chm_search needs for `params` on `index`. */
size_t chm_search_workspace_bytes(const chm_index* index, const chm_search_params* params);

/*
 * Full search of `num_queries` raw queries ([num_queries, 32, index->dim]
 * fp32, device).  Writes up to k doc ids per query (best first, -1 padded)
 * into `results` ([num_queries, k] int64, device) and the count into
 * `num_results` ([num_queries] int32, device).  A query whose stage-1 table
 * overflowed gets a negative count (-flags); rerun it with a larger
 * table_log2_extra.
 * Replaces chimera_index::search / search_one (cpp/src/search_impl.cu:46-116),
 * one query per call there, `params->batch` queries per pass here.
 */
chm_status chm_search(const chm_index* index, const chm_search_params* params,
                      const float* queries, int64_t num_queries, int64_t* results,
                      int32_t* num_results, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * Stage entry points (each replaces the named reference kernels / calls).
 */

/* FhtKacRotator::rotate over every query token (rotator.hpp:281-334,
 * called at search_impl.cu:73-75), QueryState (chimera_index_internal.cuh:
 * 58-64) and precompute_one_bit_lut_kernel (kernels.cu:402-428).
 * rot [ntok*128], cb1/cbex [ntok], lut [ntok*512] (lut may be NULL). */
chm_status chm_prepare_queries(const uint8_t* flips, int32_t dim, int32_t ex_bits,
                               const float* raw, int64_t ntok, float* rot, float* cb1,
                               float* cbex, float* lut, void* stream);

/* Exact top-nprobe centroids per rotated query token
 * (replaces IVF_PG::search_centroids -> cuVS CAGRA, ivf_pg.cpp:37-65, 96-108).
 * labels [nrows * nprobe], nearest first. */
size_t chm_probe_workspace_bytes(int64_t nrows, int64_t n_clusters, int32_t nprobe);
chm_status chm_probe(const float* rot_queries, int64_t nrows, const float* centroids,
                     const float* centroid_norms, int64_t n_clusters, int32_t nprobe,
                     uint32_t* labels, void* workspace, size_t workspace_bytes, void* stream);

/* chm_probe without allocation.  No counterpart in the reference: an addition
 * for callers that must not allocate device memory per call.  Same result as
 * chm_probe; the [nrows x n_clusters] fp32 distance scratch is a file-scope
 * device array of CHM_PROBE_NOALLOC_MAX_ELEMENTS floats (16 MiB per device,
 * reserved when the module loads), e.g. one 32-token query against up to
 * 131,072 centroids.  Larger nrows * n_clusters returns CHM_ERR_CAPACITY
 * (message in chm_last_error) and launches nothing.  The first call on each
 * device performs a one-time setup (cudaGetSymbolAddress with that device
 * current); make it before any stream capture begins.  The address it caches
 * does not survive cudaDeviceReset of that device, so do not call this entry
 * point on a device after resetting it in the same process.  The scratch needs no
 * zeroing (it is fully written before it is read).  There is one scratch per
 * device: calls that overlap on one device (two streams or two host threads)
 * race, so serialise them. */
#define CHM_PROBE_NOALLOC_MAX_ELEMENTS (1 << 22)
chm_status chm_probe_noalloc(const float* rot_queries, int64_t nrows, const float* centroids,
                             const float* centroid_norms, int64_t n_clusters, int32_t nprobe,
                             uint32_t* labels, void* stream);

/* Tensor-core probe with the same exact result: a bf16 tcgen05 pass proposes
 * candidates and exact fp32 re-ranking with an error-bound certificate (or an
 * exact recomputation of the row) decides.  nprobe <= 448. */
size_t chm_probe_tc_workspace_bytes(int64_t nrows, int64_t n_clusters, int32_t nprobe);
chm_status chm_probe_tc(const float* rot_queries, int64_t nrows, const float* centroids,
                        const void* centroids_bf16, const float* centroid_norms,
                        const float* centroid_norm_max, int64_t n_clusters, int32_t nprobe,
                        uint32_t* labels, void* workspace, size_t workspace_bytes, void* stream);

/* fp32 -> bf16 (round to nearest even) and the max of n values (device). */
chm_status chm_to_bf16(const float* x, int64_t n, void* out, void* stream);
chm_status chm_max_value(const float* x, int64_t n, float* out, void* stream);

/* Stage 1 for `nq` queries: candidate scoring of every probed list with the
 * 1-bit LUT, per-(doc, query token) max aggregation, per-doc partial score
 * and the ordered top-k_refine
 * (replaces mark/count/materialize/partial_score/sum_partial_scores kernels
 * + CUB scan/sort, kernels.cu:117-400, search_impl.cu:118-262).
 * refined_docs/refined_partial [nq * k_refine]; num_refined [nq];
 * num_candidates [nq] (may be NULL). */
size_t chm_stage1_workspace_bytes(const chm_index* index, int32_t nq, int32_t nprobe,
                                  int32_t k_refine);
chm_status chm_stage1(const chm_index* index, int32_t nq, const float* lut, const float* cb1,
                      const uint32_t* labels, int32_t nprobe, int32_t k_refine,
                      int32_t* refined_docs, float* refined_partial, int32_t* num_refined,
                      int64_t* num_candidates, void* workspace, size_t workspace_bytes,
                      void* stream);

/* chm_stage1 with the per-query status flags (nonzero: the stage-1 table or
 * key buffer overflowed; rerun with table_log2_extra + 1) and an explicit
 * table size, for callers that drive the stages themselves (document-sharded
 * search).  flags [nq]. */
size_t chm_stage1_ex_workspace_bytes(const chm_index* index, int32_t nq, int32_t nprobe,
                                     int32_t table_log2_extra);
chm_status chm_stage1_ex(const chm_index* index, int32_t nq, const float* lut, const float* cb1,
                         const uint32_t* labels, int32_t nprobe, int32_t k_refine,
                         int32_t* refined_docs, float* refined_partial, int32_t* num_refined,
                         uint32_t* flags, int32_t table_log2_extra, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Which queries of the last chm_stage1 / chm_stage1_ex call on `workspace`
 * (same index, nq, nprobe, k_refine and table_log2_extra) took the hash-table
 * path: out[q] = 1 when the dense-bound path flagged query q (fewer positive
 * docs than k_refine, an unproven boundary or a compaction overflow) or did
 * not run, 0 when it produced the refined list.  Diagnostics; no reference
 * counterpart.  out [nq] (device). */
chm_status chm_stage1_table_queries(const chm_index* index, int32_t nq, int32_t nprobe, int32_t k_refine,
                                    int32_t table_log2_extra, const void* workspace, size_t workspace_bytes,
                                    uint32_t* out, void* stream);

/* Segmented 1-bit MaxSim of the refined docs (replaces
 * gather_refined_doc_lengths/positions + one_bit_token_score +
 * one_bit_document_score kernels, kernels.cu:430-617,
 * search_impl.cu:278-403).  scores [nq * k_refine].  A negative doc id
 * marks a slot another document shard owns; its score is -inf. */
chm_status chm_refine_1bit(const chm_index* index, int32_t nq, const float* lut,
                           const float* cb1, const int32_t* refined_docs,
                           const int32_t* num_refined, int32_t k_refine, float* scores,
                           void* stream);

/* chm_refine_1bit with an int8 tensor-core filter: tcgen05.mma.kind::i8 of
 * the code bits against the query in 16-bit fixed point gives each (token,
 * query token) an estimate with a proven error bound; only tokens that can
 * hold a document's maximum get the exact LUT sum (about 1.01 per document
 * and query token).  Same scores as chm_refine_1bit, bit for bit.  chm_search
 * uses it for batches of 16 or more queries and chm_refine_1bit (one launch,
 * no planning) for smaller ones.  rot [nq*32*128] rotated queries;
 * workspace from chm_refine_1bit_tc_workspace_bytes. */
size_t chm_refine_1bit_tc_workspace_bytes(int32_t nq, int32_t k_refine);
chm_status chm_refine_1bit_tc(const chm_index* index, int32_t nq, const float* lut,
                              const float* cb1, const float* rot, const int32_t* refined_docs,
                              const int32_t* num_refined, int32_t k_refine, float* scores,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Progressive chunked selection of the docs to full-bit score
 * (search_impl.cu:341-494).  fb_docs [nq * fb_cap], num_fb [nq]. */
chm_status chm_select_fullbit(int32_t nq, const int32_t* refined_docs, const float* onebit,
                              const int32_t* num_refined, int32_t k_refine, int32_t k_full_bit,
                              int32_t num_chunks, int32_t* fb_docs, int32_t* num_fb,
                              int32_t fb_cap, void* stream);

/* (1+ex_bits)-bit MaxSim of the selected docs (replaces the AVX-512
 * compute_full_bit_scores, search_impl.cu:510-574).
 * rot [nq*32*128], cbex [nq*32], scores [nq * fb_cap].  A negative doc id
 * marks a slot another document shard owns; its score is -inf. */
chm_status chm_fullbit_score(const chm_index* index, int32_t nq, const float* rot,
                             const float* cbex, const int32_t* fb_docs, const int32_t* num_fb,
                             int32_t fb_cap, float* scores, void* stream);

/* chm_fullbit_score with the int8 tensor-core filter of chm_refine_1bit_tc:
 * the code levels (0..2^w-1) against the query in 16-bit fixed point give each
 * (token, query token) an estimate with a proven error bound; only tokens that
 * can hold a document's maximum get the exact sum in the AVX-512 lane order.
 * Same scores as chm_fullbit_score, bit for bit.  Widths w = 1 + ex_bits of 2
 * to 7 (w = 8 runs chm_fullbit_score).  Workspace from
 * chm_fullbit_score_tc_workspace_bytes. */
size_t chm_fullbit_score_tc_workspace_bytes(int32_t nq, int32_t fb_cap);

/* Workspace for chm_refine_1bit_tc or chm_fullbit_score_tc on `index` with
 * room to score its documents longer than one 128-token tile on the tensor
 * cores as 128-token parts (up to 16 parts; their maxima merge across parts).
 * The two sizes above give long documents that room only when the batch's
 * other items leave it, and otherwise the SIMT kernels.  Any of the three
 * sizes works with either call. */
size_t chm_refine_tc_workspace_bytes(const chm_index* index, int32_t nq, int32_t cap);
chm_status chm_fullbit_score_tc(const chm_index* index, int32_t nq, const float* rot,
                                const float* cbex, const int32_t* fb_docs, const int32_t* num_fb,
                                int32_t fb_cap, float* scores, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Final ordering of the full-bit scored docs, best first, ties to the larger
 * doc id (std::priority_queue<pair<float,size_t>> pops, search_impl.cu:
 * 496-500).  results [nq * k] (-1 padded), num_results [nq]. */
chm_status chm_final_topk(int32_t nq, const int32_t* fb_docs, const float* fb_scores,
                          const int32_t* num_fb, int32_t fb_cap, int32_t k, int64_t* results,
                          int32_t* num_results, void* stream);

/* Merge per-shard top-k lists (score, global doc id) into a global top-k with
 * the same ordering rule (document-sharded multi-GPU search; no reference
 * counterpart).  scores/docs [nq * shards * k] as gathered by NCCL. */
chm_status chm_merge_topk(int32_t nq, int32_t shards, int32_t k, const float* scores,
                          const int64_t* docs, const int32_t* counts, int64_t* results,
                          float* result_scores, int32_t* num_results, void* stream);

/* Document-sharded search (no reference counterpart; the reference runs on
 * one GPU).  Shard s holds docs [doc_base[s], doc_base[s] + its num_docs)
 * with local ids.
 *
 * chm_merge_refined: the gathered stage-1 lists of all shards
 * (docs/partial [shards][nq][k_refine] local ids, counts [shards][nq],
 * doc_base [shards] device array) -> the refined list of the whole corpus,
 * global ids, ordered by (partial score desc, doc asc) as the reference's
 * stable radix sort orders it (search_impl.cu:245-261).
 * out_docs/out_partial [nq][k_refine], out_counts [nq]. */
chm_status chm_merge_refined(int32_t nq, int32_t shards, int32_t k_refine, const int32_t* docs,
                             const float* partial, const int32_t* counts, const int64_t* doc_base,
                             int32_t* out_docs, float* out_partial, int32_t* out_counts,
                             void* stream);

/* Global doc ids [nq][cap] (first counts[q] valid) -> this shard's local ids,
 * -1 for documents outside [doc_base, doc_base + num_docs) and past counts. */
chm_status chm_shard_localize(int32_t nq, int32_t cap, const int32_t* global_docs,
                              const int32_t* counts, int64_t doc_base, int64_t num_docs,
                              int32_t* local_docs, void* stream);

/*
 * Index build (replaces build_index.cu:186-363 and quantization.cpp).
 */

/* Exact nearest centroid (min ||c||^2 - 2<x,c>, sequential fp32 fma dots,
 * ties to the lower id) for n vectors stored as [n, 128] rows (raw dims
 * first, zero padded); a bf16 tcgen05 pass proposes 16 candidates per row,
 * exact re-ranking with an error-bound certificate decides, uncertified rows
 * are recomputed exactly.  Stand-in for the CAGRA k=1 assignment
 * (build_index.cu:186-230).  assign [n]. */
size_t chm_build_assign_workspace_bytes(int64_t n, int64_t n_clusters);
chm_status chm_build_assign(const float* x, int64_t n, int32_t dim, const float* centroids,
                            const float* centroid_norms, int64_t n_clusters, uint32_t* assign,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Rotate + RaBitQ-encode n raw vectors (encode_embeddings,
 * build_index.cu:258-303; quantization.cpp:47-193).
 * codes1 [n*16], f1 [n], full [n*16*(1+ex_bits)], ff [n]; rot may be NULL. */
chm_status chm_build_encode(const uint8_t* flips, const float* x, int64_t n, int32_t dim,
                            int32_t ex_bits, uint8_t* codes1, float* f1, uint8_t* full,
                            float* ff, float* rot, void* stream);

/* IVF lists and the cluster-ordered 1-bit arrays from the assignment
 * (IVF_PG::build_from_assignments, ivf_pg.cpp:110-126: a stable counting sort
 * of the tokens by cluster; reorder_by_cluster, build_index.cu:328-363).
 * assign [n] cluster of every token; doc_ptrs [num_docs + 1]; codes_tok
 * [n*16] and factor_tok [n] the encoder's 1-bit output in token order.
 * Writes cluster_pos [n_clusters + 1], inv [n] (position -> token, ivf.bin),
 * codes1 [n*16], factor1 [n], doc_ids [n] (cluster order) and tok2pos [n].
 * status (device u32, may be NULL): bit 0 an assignment out of range (its
 * token gets no position), bit 1 a list longer than 32,768 tokens (left
 * unsorted); 0 on success.
 * n_clusters <= 16,777,216. */
size_t chm_build_cluster_order_workspace_bytes(int64_t n, int64_t n_clusters);
chm_status chm_build_cluster_order(const uint32_t* assign, int64_t n, int64_t n_clusters, const int64_t* doc_ptrs,
                                   int64_t num_docs, const uint8_t* codes_tok, const float* factor_tok,
                                   int64_t* cluster_pos, uint32_t* inv, uint8_t* codes1, float* factor1,
                                   int32_t* doc_ids, uint32_t* tok2pos, uint32_t* status, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Token-order copy of the cluster-ordered 1-bit arrays:
 * codes_tok[t] = codes1[tok2pos[t]], factor_tok[t] = factor1[tok2pos[t]]
 * (the inverse of reorder_by_cluster's permutation, build_index.cu:328-363).
 * codes_tok [n*16], factor_tok [n]. */
chm_status chm_token_order_1bit(const uint8_t* codes1, const float* factor1, const uint32_t* tok2pos, int64_t n,
                                uint8_t* codes_tok, float* factor_tok, void* stream);

/* Cluster of every token from the IVF layout: tok_cluster[t] = the cluster
 * whose list [cluster_pos[c], cluster_pos[c+1]) holds position tok2pos[t].
 * tok_cluster [n]. */
chm_status chm_token_clusters(const int64_t* cluster_pos, int64_t n_clusters, const uint32_t* tok2pos, int64_t n,
                              uint32_t* tok_cluster, void* stream);

/* ||x||^2 of n rows of width 128 as a sequential fma chain. */
chm_status chm_row_norms(const float* x, int64_t n, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CHIMERA_B200_H */
