/* Test infrastructure only (never linked by the product).
 *
 * Plain-C restatement of the Chimera search hot path and of its index
 * encoder, used as the parity checker for the CUDA kernels.  Every function
 * cites the reference file:line it follows (paths inside the Chimera
 * project).  Floating-point steps follow the reference's operation order;
 * the file is compiled with -ffp-contract=off and every fused multiply-add
 * the reference performs is written as an explicit fmaf()/fma().
 */
#ifndef CHIMERA_ORACLE_H
#define CHIMERA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_DIM 128 /* PADDED_DIM, cpp/include/chimera/config.cuh:7 */
#define ORC_QLEN 32 /* Q_DOCLEN,   cpp/include/chimera/config.cuh:8 */
#define ORC_LUT_PER_Q 512

typedef struct {
    int64_t n_tokens;
    int64_t num_docs;
    int64_t n_clusters;
    int32_t ex_bits;
    const int64_t* cluster_pos;  /* [n_clusters + 1] */
    const uint8_t* codes1;       /* [n_tokens * 16], cluster order */
    const float* factor1;        /* [n_tokens], cluster order */
    const int32_t* doc_ids;      /* [n_tokens], cluster order */
    const uint32_t* tok2pos;     /* [n_tokens], token id -> cluster position */
    const int64_t* doc_ptrs;     /* [num_docs + 1] */
    const uint8_t* full_codes;   /* [n_tokens * 16 * (1 + ex_bits)], token order */
    const float* full_factors;   /* [n_tokens], token order */
} orc_index;

typedef struct {
    int32_t nprobe, k_refine, k_full_bit, num_chunks, k;
} orc_params;

/* Per-query trace of every stage (caller-allocated arrays). */
typedef struct {
    int64_t n_candidates;       /* unique candidate documents (stage 1) */
    int32_t n_refined;          /* min(k_refine, n_candidates) */
    int32_t* refined_docs;      /* [k_refine] ordered by partial score desc */
    float* refined_partial;     /* [k_refine] */
    float* onebit_scores;       /* [k_refine] 1-bit MaxSim per refined doc */
    int32_t fullbit_cap;
    int32_t n_fullbit;          /* docs full-bit scored */
    int32_t* fullbit_docs;      /* [fullbit_cap] ascending refined index */
    float* fullbit_scores;      /* [fullbit_cap] */
    int32_t n_result;
    int64_t* result;            /* [k] best first */
} orc_trace;

/* rotation / query state / LUT */
void orc_fht(float* x, int n);
void orc_rotate(const uint8_t* flips /*64 B*/, const float* src, int dim, float* dst /*128*/);
void orc_query_state(const float* rot /*128*/, int ex_bits, float* cb1, float* cbex);
void orc_build_lut(const float* rot /*128*/, float* lut /*512*/);
float orc_lut_ip(const float* lut, const uint8_t* code16);

/* centroid probe (exact fp32) */
void orc_probe(const float* queries /*nq x 128*/, int64_t nq, const float* centroids,
               const float* centroid_norms, int64_t nc, int nprobe, uint32_t* labels,
               int threads);
float orc_dot128(const float* a, const float* b);

/* search */
int orc_search_one(const orc_index* idx, const float* rot_q /*32x128*/, const float* cb1,
                   const float* cbex, const uint32_t* labels /*32 x nprobe*/,
                   const orc_params* p, orc_trace* tr);
int orc_search_batch(const orc_index* idx, const float* rot_q, const float* cb1,
                     const float* cbex, const uint32_t* labels, int64_t nq,
                     const orc_params* p, int64_t* results /*nq x k*/,
                     int32_t* n_results, int threads);
float orc_fullbit_doc_score(const orc_index* idx, const float* rot_q, const float* cbex,
                            int64_t doc);
float orc_onebit_doc_score(const orc_index* idx, const float* luts /*32x512*/,
                           const float* cb1, int64_t doc);

/* packing of (1..8)-bit codes */
void orc_pack(const uint8_t* raw, uint8_t* packed, int dim, int bits);
void orc_unpack(const uint8_t* packed, uint8_t* raw, int dim, int bits);

/* encoder */
double orc_best_rescale_factor(const float* o_abs, int dim, int ex_bits);
void orc_encode(const float* rot, int dim, int ex_bits, uint8_t* code1 /*dim/8*/,
                float* f1, uint8_t* full /*dim*(1+ex)/8*/, float* ff);

/* build helpers */
void orc_assign(const float* x, int64_t n, int dim, const float* centroids,
                const float* centroid_norms, int64_t nc, uint32_t* assign, int threads);
void orc_cluster_order(const uint32_t* assign, int64_t n, int64_t nc, int64_t* cluster_pos,
                       uint32_t* inv_list);

/* batched helpers */
void orc_rotate_batch(const uint8_t* flips, const float* src, int64_t n, int dim, float* dst,
                      int threads);
void orc_encode_batch(const float* rot, int64_t n, int ex_bits, uint8_t* code1, float* f1,
                      uint8_t* full, float* ff, int threads);
void orc_query_prep(const float* rot, int64_t ntok, int ex_bits, float* cb1, float* cbex,
                    float* lut);
void orc_dot_norms(const float* x, int64_t n, float* out);

#ifdef __cplusplus
}
#endif
#endif
