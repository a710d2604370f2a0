/*
 * chimera_b200 -- document-sharded search over NCCL (lib/libchimera_nccl.so).
 *
 * No counterpart in the reference, which runs on device 0 only
 * (cpp/src/chimera_index.cu:68).  The corpus's documents are split into
 * contiguous ranges, one per rank (one GPU each); every rank holds its docs'
 * index (chm_index with local doc ids, global cluster ids) and calls
 * chm_search_sharded with the same queries.  The exchange steps run as NCCL
 * collectives on the search stream, between the stage kernels of
 * include/chimera_b200.h, with no host synchronisation:
 *
 *   prepare (every rank) -> probe of this rank's share of the query-token rows
 *   -> all_gather labels -> stage 1 on the shard -> all_gather of the local
 *   top-k_refine lists + all_reduce(max) of the overflow flags -> merge into
 *   the corpus-wide refined list -> 1-bit scores of the docs this rank owns
 *   -> all_reduce(max) -> progressive selection (every rank) -> full-bit
 *   scores of the owned docs -> all_reduce(max) -> final top-k (every rank)
 *
 * so every rank returns the results one GPU holding the whole corpus returns,
 * bit for bit.
 */
#ifndef CHIMERA_B200_SHARDED_H
#define CHIMERA_B200_SHARDED_H

#include "chimera_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

#define CHM_COMM_ID_BYTES 128

/* An NCCL communicator with its rank, size and device. */
typedef struct chm_comm chm_comm;

/* A new NCCL unique id (ncclGetUniqueId), to be shared with every rank. */
chm_status chm_comm_unique_id(uint8_t id[CHM_COMM_ID_BYTES]);

/* Rank `rank` of `world` on CUDA device `device` (ncclCommInitRank; every
 * rank calls it with the same id). */
chm_status chm_comm_init(const uint8_t id[CHM_COMM_ID_BYTES], int32_t world, int32_t rank, int32_t device,
                         chm_comm** out);

/* One process driving `ndev` GPUs: comms[i] is rank i on devices[i]
 * (ncclCommInitAll). */
chm_status chm_comm_init_all(int32_t ndev, const int32_t* devices, chm_comm** comms);

chm_status chm_comm_destroy(chm_comm* comm);

/* This rank's documents: [doc_base[rank], doc_base[rank + 1]) of the corpus
 * (doc_base: world + 1 host values). */
typedef struct {
    int32_t rank;
    int32_t world;
    const int64_t* doc_base;
} chm_shard;

/* Device milliseconds of the steps of the last batch (timing != NULL). */
typedef enum {
    CHM_SH_PREPARE = 0,
    CHM_SH_PROBE,
    CHM_SH_GATHER_LABELS,
    CHM_SH_STAGE1,
    CHM_SH_GATHER_LISTS,
    CHM_SH_MERGE,
    CHM_SH_REFINE,
    CHM_SH_REDUCE_ONEBIT,
    CHM_SH_SELECT,
    CHM_SH_FULLBIT,
    CHM_SH_REDUCE_FULLBIT,
    CHM_SH_FINAL,
    CHM_SH_STEPS
} chm_sharded_step;

size_t chm_search_sharded_workspace_bytes(const chm_index* shard_index, const chm_search_params* params,
                                          int32_t world);

/* chm_search over a document-sharded corpus.  shard_index holds this rank's
 * docs with local ids; results are global doc ids (identical on every rank).
 * A query whose stage-1 table overflowed on any rank gets a negative count on
 * every rank: rerun it with a larger table_log2_extra.  timing: NULL, or
 * CHM_SH_STEPS floats receiving the per-step device milliseconds of the last
 * batch (events on `stream`). */
chm_status chm_search_sharded(const chm_index* shard_index, const chm_search_params* params,
                              const chm_shard* shard, chm_comm* comm, const float* queries, int64_t num_queries,
                              int64_t* results, int32_t* num_results, void* workspace, size_t workspace_bytes,
                              void* stream, float* timing);

#ifdef __cplusplus
}
#endif
#endif /* CHIMERA_B200_SHARDED_H */
