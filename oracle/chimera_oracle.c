/* Test infrastructure only: plain-C restatement of the Chimera search path
 * and encoder.  The CUDA product never calls this file; tests/, the smoke
 * check and bench.py's CPU-baseline leg use it as the checker.
 *
 * Parity is pinned two ways: (1) rotation, encoding, packing and the
 * full-bit scorer are compared bit-for-bit with the reference's own CPU code
 * (oracle/_ref, built from the reference sources by oracle/Makefile); (2) the
 * GPU-stage restatements follow kernels.cu / search_impl.cu line by line in
 * operation order.  See the header for the data layout.
 */
#include "chimera_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* Rotation: FhtKacRotator::rotate, rabitqlib/utils/rotator.hpp:281-334.     */
/* FFHT helper_float_{6,7} (rabitqlib/utils/fht_avx.cpp:396-591) applies    */
/* radix-2 butterflies (a+b, a-b) in ascending stride order 1,2,...,n/2.     */
/* ------------------------------------------------------------------------ */
void orc_fht(float* x, int n) {
    for (int h = 1; h < n; h <<= 1) {
        for (int i = 0; i < n; i += 2 * h) {
            for (int j = i; j < i + h; ++j) {
                const float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
        }
    }
}

/* flip_sign, rotator.hpp:129-172: element i of a 64-float chunk flips when
 * bit i of the little-endian u64 at flip[i/8] is set. */
static void flip_sign(const uint8_t* flip, float* data, int dim) {
    for (int i = 0; i < dim; ++i)
        if ((flip[i >> 3] >> (i & 7)) & 1u) data[i] = -data[i];
}

static void rescale(float* x, int n, float f) {
    for (int i = 0; i < n; ++i) x[i] = x[i] * f;
}

/* kacs_walk, rotator.hpp:257-270 */
static void kacs_walk(float* x, int len) {
    const int half = len / 2;
    for (int i = 0; i < half; ++i) {
        const float a = x[i], b = x[i + half];
        x[i] = a + b;
        x[i + half] = a - b;
    }
}

void orc_rotate(const uint8_t* flips, const float* src, int dim, float* dst) {
    const int padded = ORC_DIM;
    int log = 0;
    while ((2 << log) <= dim) ++log;          /* floor_log2(dim) */
    const int trunc = 1 << log;
    const float fac = 1.0f / sqrtf((float)trunc);
    memcpy(dst, src, sizeof(float) * (size_t)dim);
    for (int i = dim; i < padded; ++i) dst[i] = 0.0f;
    const int fb = padded / 8;                /* flip bytes per round */
    if (trunc == padded) {                    /* rotator.hpp:284-306 */
        for (int r = 0; r < 4; ++r) {
            flip_sign(flips + r * fb, dst, padded);
            orc_fht(dst, trunc);
            rescale(dst, trunc, fac);
        }
        return;
    }
    const int start = padded - trunc;         /* rotator.hpp:308-333 */
    for (int r = 0; r < 4; ++r) {
        flip_sign(flips + r * fb, dst, padded);
        float* base = (r & 1) ? dst + start : dst;
        orc_fht(base, trunc);
        rescale(base, trunc, fac);
        kacs_walk(dst, padded);
    }
    rescale(dst, padded, 0.25f);
}

/* QueryState, cpp/src/chimera_index_internal.cuh:58-64 (std::accumulate is a
 * left-to-right sum starting at 0.0f). */
void orc_query_state(const float* rot, int ex_bits, float* cb1, float* cbex) {
    float sumq = 0.0f;
    for (int i = 0; i < ORC_DIM; ++i) sumq = sumq + rot[i];
    *cb1 = (sumq * (float)((1 << 1) - 1)) / 2.0f;
    *cbex = (sumq * (float)((1 << (ex_bits + 1)) - 1)) / 2.0f;
}

/* precompute_one_bit_lut_kernel, cpp/src/kernels.cu:402-428 */
void orc_build_lut(const float* q, float* lut) {
    for (int idx = 0; idx < ORC_LUT_PER_Q; ++idx) {
        const int chunk = idx / 16, e = idx % 16;
        float s = 0.0f;
        for (int b = 0; b < 4; ++b)
            if ((e >> b) & 1) s = s + q[chunk * 4 + b];
        lut[idx] = s;
    }
}

/* ip accumulation of partial_score_kernel (kernels.cu:361-373) and
 * one_bit_token_score_kernel (kernels.cu:497-500): chunks 0..31 in order;
 * chunk c is nibble (c & 1) of code byte c / 2. */
float orc_lut_ip(const float* lut, const uint8_t* code) {
    float ip = 0.0f;
    for (int c = 0; c < 32; ++c) {
        const int nib = (code[c >> 1] >> ((c & 1) * 4)) & 0xF;
        ip = ip + lut[c * 16 + nib];
    }
    return ip;
}

/* ------------------------------------------------------------------------ */
/* Exact centroid probe (stand-in for cuVS CAGRA, ivf_pg.cpp:37-65).         */
/* Key: dist = ||c||^2 - 2<q,c>, both dots as sequential fmaf over the 128  */
/* rotated dims; smallest nprobe, ties to the lower centroid id.            */
/* ------------------------------------------------------------------------ */
float orc_dot128(const float* a, const float* b) {
    float acc = 0.0f;
    for (int i = 0; i < ORC_DIM; ++i) acc = fmaf(a[i], b[i], acc);
    return acc;
}

static float dotn(const float* a, const float* b, int n) {
    float acc = 0.0f;
    for (int i = 0; i < n; ++i) acc = fmaf(a[i], b[i], acc);
    return acc;
}

typedef struct { float d; uint32_t id; } dist_id;

static int worse(dist_id a, dist_id b) { /* a ranks after b */
    return a.d > b.d || (a.d == b.d && a.id > b.id);
}

/* bounded max-heap of the best k (root = worst kept) */
static void heap_push_bounded(dist_id* h, int* n, int k, dist_id v) {
    if (*n < k) {
        int i = (*n)++;
        h[i] = v;
        while (i > 0) {
            int p = (i - 1) / 2;
            if (!worse(h[i], h[p])) break;
            dist_id t = h[i]; h[i] = h[p]; h[p] = t; i = p;
        }
        return;
    }
    if (!worse(h[0], v)) return;
    h[0] = v;
    int i = 0;
    for (;;) {
        int l = 2 * i + 1, r = l + 1, m = i;
        if (l < k && worse(h[l], h[m])) m = l;
        if (r < k && worse(h[r], h[m])) m = r;
        if (m == i) break;
        dist_id t = h[i]; h[i] = h[m]; h[m] = t; i = m;
    }
}

static int cmp_dist_id(const void* a, const void* b) {
    const dist_id* x = (const dist_id*)a;
    const dist_id* y = (const dist_id*)b;
    if (worse(*x, *y)) return 1;
    if (worse(*y, *x)) return -1;
    return 0;
}

void orc_probe(const float* queries, int64_t nq, const float* centroids,
               const float* cnorm, int64_t nc, int nprobe, uint32_t* labels, int threads) {
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
    for (int64_t q = 0; q < nq; ++q) {
        dist_id* h = (dist_id*)malloc(sizeof(dist_id) * (size_t)nprobe);
        int n = 0;
        const float* qv = queries + q * ORC_DIM;
        for (int64_t c = 0; c < nc; ++c) {
            const float dot = orc_dot128(qv, centroids + c * ORC_DIM);
            dist_id v = { cnorm[c] - 2.0f * dot, (uint32_t)c };
            heap_push_bounded(h, &n, nprobe, v);
        }
        qsort(h, (size_t)n, sizeof(dist_id), cmp_dist_id);
        for (int i = 0; i < nprobe; ++i) labels[q * nprobe + i] = i < n ? h[i].id : 0xFFFFFFFFu;
        free(h);
    }
}

/* ------------------------------------------------------------------------ */
/* Search                                                                    */
/* ------------------------------------------------------------------------ */

/* sum_partial_scores_kernel's shuffle-down tree, kernels.cu:192-198 */
static float tree32(const float* v) {
    float a[32];
    memcpy(a, v, sizeof(a));
    for (int off = 16; off >= 1; off >>= 1)
        for (int i = 0; i < off; ++i) a[i] = a[i] + a[i + off];
    return a[0];
}

/* one_bit_document_score_kernel's 128-thread shared-memory tree,
 * kernels.cu:557-570: each of the first 32 threads holds 0.0f + max_vals[j];
 * strides 64 and 32 add zeros; strides 16..1 are the pairwise tree. */
static float tree32_block128(const float* m) {
    float a[32];
    for (int i = 0; i < 32; ++i) a[i] = ((0.0f + m[i]) + 0.0f) + 0.0f;
    for (int off = 16; off >= 1; off >>= 1)
        for (int i = 0; i < off; ++i) a[i] = a[i] + a[i + off];
    return a[0];
}

typedef struct { float s; int32_t doc; int32_t idx; } scored;

static int cmp_partial(const void* a, const void* b) { /* score desc, doc asc */
    const scored* x = (const scored*)a;
    const scored* y = (const scored*)b;
    if (x->s > y->s) return -1;
    if (x->s < y->s) return 1;
    return (x->doc > y->doc) - (x->doc < y->doc);
}

static int cmp_onebit(const void* a, const void* b) { /* score desc, idx asc */
    const scored* x = (const scored*)a;
    const scored* y = (const scored*)b;
    if (x->s > y->s) return -1;
    if (x->s < y->s) return 1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}

static int cmp_final(const void* a, const void* b) { /* priority_queue<pair<float,size_t>> pop order */
    const scored* x = (const scored*)a;
    const scored* y = (const scored*)b;
    if (x->s > y->s) return -1;
    if (x->s < y->s) return 1;
    return (x->doc < y->doc) - (x->doc > y->doc);
}

float orc_onebit_doc_score(const orc_index* idx, const float* luts, const float* cb1,
                           int64_t doc) {
    float m[32];
    for (int t = 0; t < 32; ++t) m[t] = -FLT_MAX;
    for (int64_t tok = idx->doc_ptrs[doc]; tok < idx->doc_ptrs[doc + 1]; ++tok) {
        const uint32_t pos = idx->tok2pos[tok];
        const uint8_t* code = idx->codes1 + (size_t)pos * 16;
        const float f = idx->factor1[pos];
        for (int t = 0; t < 32; ++t) {
            const float d = (orc_lut_ip(luts + t * ORC_LUT_PER_Q, code) - cb1[t]) * f;
            m[t] = fmaxf(m[t], d);
        }
    }
    return tree32_block128(m);
}

/* Code of dimension i in the packed layouts of
 * rabitqlib/quantization/pack_excode.hpp:13-260 (w = bits per dimension). */
static inline int code_at(const uint8_t* p, int i, int w) {
    switch (w) {
        case 1: return (p[2 * (i / 16) + (i % 16) / 8] >> (i % 8)) & 1;
        case 2: return (p[4 * (i / 16) + (i % 4)] >> (2 * ((i % 16) / 4))) & 3;
        case 3: {
            const uint8_t* g = p + 24 * (i / 64);
            const int r = i % 64;
            return ((g[r % 16] >> (2 * (r / 16))) & 3) | (((g[16 + r % 8] >> (r / 8)) & 1) << 2);
        }
        case 4: return (p[8 * (i / 16) + (i % 8)] >> (4 * ((i % 16) / 8))) & 15;
        case 5: {
            const uint8_t* g = p + 40 * (i / 64);
            const int r = i % 64;
            const int lo = (g[16 * (r / 32) + (r % 16)] >> (4 * ((r / 16) % 2))) & 15;
            return lo | (((g[32 + r % 8] >> (r / 8)) & 1) << 4);
        }
        case 6: {
            const uint8_t* g = p + 12 * (i / 16);
            const int j = i % 16;
            return ((g[j % 8] >> (4 * (j / 8))) & 15) | (((g[8 + j % 4] >> (2 * (j / 4))) & 3) << 4);
        }
        case 7: {
            const uint8_t* g = p + 56 * (i / 64);
            const int r = i % 64;
            int lo;
            if (r < 48) {
                lo = g[r] & 63;
            } else {
                const int j = r - 48;
                lo = ((g[j] >> 6) & 3) | (((g[16 + j] >> 6) & 3) << 2) | (((g[32 + j] >> 6) & 3) << 4);
            }
            return lo | (((g[48 + r % 8] >> (r / 8)) & 1) << 6);
        }
        default: return p[i];
    }
}

void orc_unpack(const uint8_t* packed, uint8_t* raw, int dim, int bits) {
    for (int i = 0; i < dim; ++i) raw[i] = (uint8_t)code_at(packed, i, bits);
}

void orc_pack(const uint8_t* raw, uint8_t* packed, int dim, int bits) {
    int bytes = dim * bits / 8;
    memset(packed, 0, (size_t)bytes);
    for (int i = 0; i < dim; ++i) {
        const int v = raw[i];
        switch (bits) {
            case 1: packed[2 * (i / 16) + (i % 16) / 8] |= (uint8_t)((v & 1) << (i % 8)); break;
            case 2: packed[4 * (i / 16) + (i % 4)] |= (uint8_t)((v & 3) << (2 * ((i % 16) / 4))); break;
            case 3: {
                uint8_t* g = packed + 24 * (i / 64);
                const int r = i % 64;
                g[r % 16] |= (uint8_t)((v & 3) << (2 * (r / 16)));
                g[16 + r % 8] |= (uint8_t)(((v >> 2) & 1) << (r / 8));
                break;
            }
            case 4: packed[8 * (i / 16) + (i % 8)] |= (uint8_t)((v & 15) << (4 * ((i % 16) / 8))); break;
            case 5: {
                uint8_t* g = packed + 40 * (i / 64);
                const int r = i % 64;
                g[16 * (r / 32) + (r % 16)] |= (uint8_t)((v & 15) << (4 * ((r / 16) % 2)));
                g[32 + r % 8] |= (uint8_t)(((v >> 4) & 1) << (r / 8));
                break;
            }
            case 6: {
                uint8_t* g = packed + 12 * (i / 16);
                const int j = i % 16;
                g[j % 8] |= (uint8_t)((v & 15) << (4 * (j / 8)));
                g[8 + j % 4] |= (uint8_t)(((v >> 4) & 3) << (2 * (j / 4)));
                break;
            }
            case 7: {
                uint8_t* g = packed + 56 * (i / 64);
                const int r = i % 64;
                if (r < 48) {
                    g[r] |= (uint8_t)(v & 63);
                } else {
                    const int j = r - 48;
                    g[j] |= (uint8_t)((v & 3) << 6);
                    g[16 + j] |= (uint8_t)(((v >> 2) & 3) << 6);
                    g[32 + j] |= (uint8_t)(((v >> 4) & 3) << 6);
                }
                g[48 + r % 8] |= (uint8_t)(((v >> 6) & 1) << (r / 8));
                break;
            }
            default: packed[i] = (uint8_t)v; break;
        }
    }
}

/* _mm512_reduce_add_ps as GCC implements it (avx512fintrin.h,
 * __MM512_REDUCE_OP): halves, quarters, then (0+2)+(1+3). */
static float reduce16(const float* s) {
    float t3[8], t6[4];
    for (int i = 0; i < 8; ++i) t3[i] = s[8 + i] + s[i];
    for (int i = 0; i < 4; ++i) t6[i] = t3[4 + i] + t3[i];
    const float a = t6[0] + t6[2];
    const float b = t6[1] + t6[3];
    return a + b;
}

/* compute_full_bit_scores, cpp/src/search_impl.cu:525-572, with
 * gemv_batch8_avx512 (space.hpp:806-851): per query token 16 lane
 * accumulators, s[l] = fma(decoded[16b+l], q[16b+l], s[l]) for b = 0..7,
 * then the 512-bit reduction; combined = (ip - cbex) * factor; max over
 * tokens; final sum of the two 16-lane halves reduced the same way. */
float orc_fullbit_doc_score(const orc_index* idx, const float* q, const float* cbex,
                            int64_t doc) {
    const int w = 1 + idx->ex_bits;
    const size_t stride = (size_t)ORC_DIM * (size_t)w / 8;
    float m[32];
    for (int t = 0; t < 32; ++t) m[t] = -INFINITY;
    float dec[ORC_DIM];
    for (int64_t tok = idx->doc_ptrs[doc]; tok < idx->doc_ptrs[doc + 1]; ++tok) {
        const uint8_t* code = idx->full_codes + (size_t)tok * stride;
        for (int i = 0; i < ORC_DIM; ++i) dec[i] = (float)code_at(code, i, w);
        const float f = idx->full_factors[tok];
        for (int t = 0; t < 32; ++t) {
            const float* qt = q + t * ORC_DIM;
            float s[16];
            for (int l = 0; l < 16; ++l) s[l] = 0.0f;
            for (int b = 0; b < ORC_DIM / 16; ++b)
                for (int l = 0; l < 16; ++l) s[l] = fmaf(dec[16 * b + l], qt[16 * b + l], s[l]);
            const float ip = reduce16(s);
            const float comb = (ip - cbex[t]) * f;
            m[t] = m[t] > comb ? m[t] : comb;   /* _mm512_max_ps(m, comb) */
        }
    }
    float s[16];
    for (int l = 0; l < 16; ++l) s[l] = m[l] + m[16 + l];
    return reduce16(s);
}

/* Stage 1 (search_impl.cu:118-262; kernels.cu:206-400):
 * candidate docs = every doc with a token in a list probed by any query
 * token; partial[doc][t] = max(0, max positive (ip - cb1[t]) * factor over
 * the doc's tokens in t's probed lists); doc partial score = tree32;
 * stable descending sort of (ascending-doc) candidates, keep k_refine. */
typedef struct {
    int32_t* row_of_doc;   /* [num_docs], -1 when not a candidate */
    float* rows;           /* [cap * 32] */
    int32_t* cand;         /* [cap] */
    int64_t cap, n;
} stage1_ws;

static int stage1(const orc_index* idx, const float* luts, const float* cb1,
                  const uint32_t* labels, int nprobe, stage1_ws* ws) {
    ws->n = 0;
    for (int t = 0; t < 32; ++t) {
        const float* lut = luts + t * ORC_LUT_PER_Q;
        for (int p = 0; p < nprobe; ++p) {
            const uint32_t label = labels[t * nprobe + p];
            if ((int64_t)label >= idx->n_clusters) continue;
            for (int64_t pos = idx->cluster_pos[label]; pos < idx->cluster_pos[label + 1]; ++pos) {
                const int32_t doc = idx->doc_ids[pos];
                if (doc < 0 || (int64_t)doc >= idx->num_docs) continue;
                int32_t row = ws->row_of_doc[doc];
                if (row < 0) {
                    if (ws->n == ws->cap) {
                        const int64_t nc = ws->cap ? ws->cap * 2 : 4096;
                        float* r = (float*)realloc(ws->rows, sizeof(float) * 32 * (size_t)nc);
                        int32_t* c = (int32_t*)realloc(ws->cand, sizeof(int32_t) * (size_t)nc);
                        if (!r || !c) return -1;
                        ws->rows = r; ws->cand = c; ws->cap = nc;
                    }
                    row = (int32_t)ws->n++;
                    ws->row_of_doc[doc] = row;
                    ws->cand[row] = doc;
                    memset(ws->rows + (size_t)row * 32, 0, sizeof(float) * 32);
                }
                const float ip = orc_lut_ip(lut, idx->codes1 + (size_t)pos * 16);
                const float dist = (ip - cb1[t]) * idx->factor1[pos];
                float* cell = ws->rows + (size_t)row * 32 + t;
                if (dist > 0.0f && dist > *cell) *cell = dist;
            }
        }
    }
    return 0;
}

int orc_search_one(const orc_index* idx, const float* rot_q, const float* cb1,
                   const float* cbex, const uint32_t* labels, const orc_params* p,
                   orc_trace* tr) {
    float* luts = (float*)malloc(sizeof(float) * 32 * ORC_LUT_PER_Q);
    stage1_ws ws = { 0 };
    ws.row_of_doc = (int32_t*)malloc(sizeof(int32_t) * (size_t)idx->num_docs);
    if (!luts || !ws.row_of_doc) return -1;
    for (int64_t d = 0; d < idx->num_docs; ++d) ws.row_of_doc[d] = -1;
    for (int t = 0; t < 32; ++t) orc_build_lut(rot_q + t * ORC_DIM, luts + t * ORC_LUT_PER_Q);
    if (stage1(idx, luts, cb1, labels, p->nprobe, &ws) != 0) return -1;

    tr->n_candidates = ws.n;
    tr->n_refined = 0;
    tr->n_fullbit = 0;
    tr->n_result = 0;
    int rc = 0;
    if (ws.n > 0) {
        scored* cs = (scored*)malloc(sizeof(scored) * (size_t)ws.n);
        for (int64_t i = 0; i < ws.n; ++i) {
            cs[i].s = tree32(ws.rows + (size_t)i * 32);
            cs[i].doc = ws.cand[i];
            cs[i].idx = 0;
        }
        qsort(cs, (size_t)ws.n, sizeof(scored), cmp_partial);
        const int R = (int)(ws.n < p->k_refine ? ws.n : p->k_refine);
        tr->n_refined = R;
        for (int r = 0; r < R; ++r) {
            tr->refined_docs[r] = cs[r].doc;
            tr->refined_partial[r] = cs[r].s;
        }
        free(cs);

        /* 1-bit refinement over all tokens of the refined docs */
        for (int r = 0; r < R; ++r)
            tr->onebit_scores[r] = orc_onebit_doc_score(idx, luts, cb1, tr->refined_docs[r]);

        /* progressive chunked selection, search_impl.cu:341-494 */
        const int T = p->k_full_bit < R ? p->k_full_bit : R;
        const int nch = p->num_chunks < R ? p->num_chunks : R;
        const int cs_sz = (R + nch - 1) / nch;
        scored* order = (scored*)malloc(sizeof(scored) * (size_t)R);
        for (int r = 0; r < R; ++r) { order[r].s = tr->onebit_scores[r]; order[r].idx = r; order[r].doc = 0; }
        qsort(order, (size_t)R, sizeof(scored), cmp_onebit);
        uint8_t* chosen = (uint8_t*)calloc((size_t)R, 1);
        for (int c = 0; c < nch; ++c) {
            const int end = (c + 1) * cs_sz < R ? (c + 1) * cs_sz : R;
            const int carry = T < end ? T : end;
            int cum = T * (c + 1) / nch;
            if (cum > carry) cum = carry;
            int taken = 0;
            for (int i = 0; i < R && taken < cum; ++i) {
                if (order[i].idx < end) { chosen[order[i].idx] = 1; ++taken; }
            }
        }
        int nf = 0;
        scored* fin = (scored*)malloc(sizeof(scored) * (size_t)R);
        for (int r = 0; r < R; ++r) {
            if (!chosen[r]) continue;
            const float s = orc_fullbit_doc_score(idx, rot_q, cbex, tr->refined_docs[r]);
            if (nf < tr->fullbit_cap) {
                tr->fullbit_docs[nf] = tr->refined_docs[r];
                tr->fullbit_scores[nf] = s;
            } else {
                rc = -2;
            }
            fin[nf].s = s; fin[nf].doc = tr->refined_docs[r]; fin[nf].idx = r;
            ++nf;
        }
        tr->n_fullbit = nf;
        qsort(fin, (size_t)nf, sizeof(scored), cmp_final);
        const int nk = nf < p->k ? nf : p->k;
        for (int i = 0; i < nk; ++i) tr->result[i] = fin[i].doc;
        tr->n_result = nk;
        free(fin); free(chosen); free(order);
    }
    free(ws.rows); free(ws.cand); free(ws.row_of_doc); free(luts);
    return rc;
}

int orc_search_batch(const orc_index* idx, const float* rot_q, const float* cb1,
                     const float* cbex, const uint32_t* labels, int64_t nq,
                     const orc_params* p, int64_t* results, int32_t* n_results, int threads) {
    int err = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1) reduction(|:err)
    for (int64_t q = 0; q < nq; ++q) {
        orc_trace tr;
        memset(&tr, 0, sizeof(tr));
        tr.refined_docs = (int32_t*)malloc(sizeof(int32_t) * (size_t)p->k_refine);
        tr.refined_partial = (float*)malloc(sizeof(float) * (size_t)p->k_refine);
        tr.onebit_scores = (float*)malloc(sizeof(float) * (size_t)p->k_refine);
        tr.fullbit_cap = p->k_refine;
        tr.fullbit_docs = (int32_t*)malloc(sizeof(int32_t) * (size_t)p->k_refine);
        tr.fullbit_scores = (float*)malloc(sizeof(float) * (size_t)p->k_refine);
        tr.result = results + q * p->k;
        const int rc = orc_search_one(idx, rot_q + q * 32 * ORC_DIM, cb1 + q * 32, cbex + q * 32,
                                      labels + q * 32 * p->nprobe, p, &tr);
        if (rc != 0) err |= 1;
        n_results[q] = tr.n_result;
        free(tr.refined_docs); free(tr.refined_partial); free(tr.onebit_scores);
        free(tr.fullbit_docs); free(tr.fullbit_scores);
    }
    return err ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* Encoder: cpp/src/quantization.cpp:47-193.                                 */
/* Eigen 3.4 reductions with AVX-512 packets (Redux.h:227-282, 64-byte       */
/* aligned input): two 16-lane accumulators over alternating packets, the    */
/* products fused into the adds, then predux (8+8, 4+4, (0+2)+(1+3)).        */
/* ------------------------------------------------------------------------ */
static float predux16(const float* p) {
    float x8[8], x4[4];
    for (int i = 0; i < 8; ++i) x8[i] = p[i] + p[8 + i];
    for (int i = 0; i < 4; ++i) x4[i] = x8[i] + x8[4 + i];
    const float a = x4[0] + x4[2];
    const float b = x4[1] + x4[3];
    return a + b;
}

static float eigen_dot128(const float* a, const float* b) {
    float r0[16], r1[16];
    for (int l = 0; l < 16; ++l) { r0[l] = a[l] * b[l]; r1[l] = a[16 + l] * b[16 + l]; }
    for (int base = 32; base < 128; base += 32)
        for (int l = 0; l < 16; ++l) {
            r0[l] = fmaf(a[base + l], b[base + l], r0[l]);
            r1[l] = fmaf(a[base + 16 + l], b[base + 16 + l], r1[l]);
        }
    for (int l = 0; l < 16; ++l) r0[l] = r0[l] + r1[l];
    return predux16(r0);
}

/* encode_one_bit, quantization.cpp:47-60 */
static void encode_one_bit(const float* o, int dim, uint8_t* code, float* factor) {
    float xu_cb[ORC_DIM];
    memset(code, 0, (size_t)dim / 8);
    for (int i = 0; i < dim; ++i) {
        const int bit = o[i] > 0.0f;
        code[i >> 3] |= (uint8_t)(bit << (i & 7));
        xu_cb[i] = (float)bit + -0.5f;
    }
    *factor = 1.0f / eigen_dot128(xu_cb, o);
}

/* best_rescale_factor, quantization.cpp:62-119.  The reference pops a
 * min-priority-queue of (t, dim) pairs; pops therefore follow ascending
 * (t, dim) order, which this binary heap reproduces. */
typedef struct { double t; int id; } tev;
static int tev_less(tev a, tev b) { return a.t < b.t || (a.t == b.t && a.id < b.id); }

static void tev_push(tev* h, int* n, tev v) {
    int i = (*n)++;
    h[i] = v;
    while (i > 0) {
        int p = (i - 1) / 2;
        if (!tev_less(h[i], h[p])) break;
        tev t = h[i]; h[i] = h[p]; h[p] = t; i = p;
    }
}

static tev tev_pop(tev* h, int* n) {
    tev top = h[0];
    h[0] = h[--(*n)];
    int i = 0;
    for (;;) {
        int l = 2 * i + 1, r = l + 1, m = i;
        if (l < *n && tev_less(h[l], h[m])) m = l;
        if (r < *n && tev_less(h[r], h[m])) m = r;
        if (m == i) break;
        tev t = h[i]; h[i] = h[m]; h[m] = t; i = m;
    }
    return top;
}

static const float kTightStart[9] = { 0.f, 0.15f, 0.20f, 0.52f, 0.59f, 0.71f, 0.75f, 0.77f, 0.81f };

double orc_best_rescale_factor(const float* o_abs, int dim, int ex_bits) {
    const double kEps = 1e-5;
    const int kNEnum = 10;
    float mx = o_abs[0];
    for (int i = 1; i < dim; ++i) if (o_abs[i] > mx) mx = o_abs[i];
    const double max_o = mx;
    const double t_end = (double)(((1 << ex_bits) - 1) + kNEnum) / max_o;
    const double t_start = t_end * (double)kTightStart[ex_bits];
    int cur[ORC_DIM];
    double sqr_den = (double)dim * 0.25;
    double num = 0.0;
    for (int i = 0; i < dim; ++i) {
        const int c = (int)fma(t_start, (double)o_abs[i], kEps);
        cur[i] = c;
        sqr_den = sqr_den + (double)(c * c + c);
        num = fma((double)c + 0.5, (double)o_abs[i], num);
    }
    tev heap[ORC_DIM];
    int n = 0;
    for (int i = 0; i < dim; ++i) {
        tev v = { (double)(cur[i] + 1) / (double)o_abs[i], i };
        tev_push(heap, &n, v);
    }
    double max_ip = 0.0, t = 0.0;
    while (n > 0) {
        const tev e = tev_pop(heap, &n);
        cur[e.id]++;
        const int upd = cur[e.id];
        sqr_den = sqr_den + (double)(2 * upd);
        num = num + (double)o_abs[e.id];
        const double ip = num / sqrt(sqr_den);
        if (ip > max_ip) { max_ip = ip; t = e.t; }
        if (upd < (1 << ex_bits) - 1) {
            const double tn = (double)(upd + 1) / (double)o_abs[e.id];
            if (tn < t_end) { tev v = { tn, e.id }; tev_push(heap, &n, v); }
        }
    }
    return t;
}

/* quantize_ex (quantization.cpp:121-146) + encode_full_code (:168-193). */
void orc_encode(const float* o, int dim, int ex_bits, uint8_t* code1, float* f1,
                uint8_t* full, float* ff) {
    encode_one_bit(o, dim, code1, f1);
    /* rowwise().normalized(): x / sqrt(squaredNorm) */
    const float nrm = sqrtf(eigen_dot128(o, o));
    float o_abs[ORC_DIM];
    for (int i = 0; i < dim; ++i) o_abs[i] = fabsf(o[i] / nrm);
    const double t = orc_best_rescale_factor(o_abs, dim, ex_bits);
    const int top = (1 << ex_bits) - 1;
    uint8_t total[ORC_DIM];
    float xu_cb[ORC_DIM];
    const float cb = -((float)(1 << ex_bits) - 0.5f);
    for (int i = 0; i < dim; ++i) {
        int c = (int)fma(t, (double)o_abs[i], 1e-5);
        if (c >= (1 << ex_bits)) c = top;
        if (o[i] < 0.0f) c = (~c) & top;
        const int tot = c + ((o[i] >= 0.0f) << ex_bits);
        total[i] = (uint8_t)tot;
        xu_cb[i] = (float)tot + cb;
    }
    *ff = 1.0f / eigen_dot128(xu_cb, o);
    orc_pack(total, full, dim, 1 + ex_bits);
}

/* ------------------------------------------------------------------------ */
/* Build helpers                                                             */
/* ------------------------------------------------------------------------ */

/* Exact nearest centroid (stand-in for the CAGRA k=1 search of
 * build_index.cu:186-230): min ||c||^2 - 2<x,c>, ties to the lower id. */
void orc_assign(const float* x, int64_t n, int dim, const float* c, const float* cn,
                int64_t nc, uint32_t* assign, int threads) {
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (int64_t i = 0; i < n; ++i) {
        float best = INFINITY;
        uint32_t bi = 0;
        for (int64_t k = 0; k < nc; ++k) {
            const float d = cn[k] - 2.0f * dotn(x + i * dim, c + k * dim, dim);
            if (d < best) { best = d; bi = (uint32_t)k; }
        }
        assign[i] = bi;
    }
}

/* IVF_PG::build_from_assignments, cpp/src/ivf_pg.cpp:110-126 */
void orc_cluster_order(const uint32_t* a, int64_t n, int64_t nc, int64_t* cluster_pos,
                       uint32_t* inv_list) {
    memset(cluster_pos, 0, sizeof(int64_t) * (size_t)(nc + 1));
    for (int64_t i = 0; i < n; ++i) cluster_pos[a[i] + 1]++;
    for (int64_t k = 0; k < nc; ++k) cluster_pos[k + 1] += cluster_pos[k];
    int64_t* w = (int64_t*)malloc(sizeof(int64_t) * (size_t)nc);
    memcpy(w, cluster_pos, sizeof(int64_t) * (size_t)nc);
    for (int64_t i = 0; i < n; ++i) inv_list[w[a[i]]++] = (uint32_t)i;
    free(w);
}

/* Batched helpers (OpenMP over rows). */
void orc_rotate_batch(const uint8_t* flips, const float* src, int64_t n, int dim, float* dst,
                      int threads) {
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (int64_t i = 0; i < n; ++i) orc_rotate(flips, src + i * dim, dim, dst + i * ORC_DIM);
}

void orc_encode_batch(const float* rot, int64_t n, int ex_bits, uint8_t* code1, float* f1,
                      uint8_t* full, float* ff, int threads) {
    const int fb = ORC_DIM * (1 + ex_bits) / 8;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (int64_t i = 0; i < n; ++i)
        orc_encode(rot + i * ORC_DIM, ORC_DIM, ex_bits, code1 + i * 16, f1 + i,
                   full + i * fb, ff + i);
}

void orc_query_prep(const float* rot, int64_t ntok, int ex_bits, float* cb1, float* cbex,
                    float* lut) {
    for (int64_t i = 0; i < ntok; ++i) {
        orc_query_state(rot + i * ORC_DIM, ex_bits, cb1 + i, cbex + i);
        if (lut) orc_build_lut(rot + i * ORC_DIM, lut + i * ORC_LUT_PER_Q);
    }
}

void orc_dot_norms(const float* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_dot128(x + i * ORC_DIM, x + i * ORC_DIM);
}
