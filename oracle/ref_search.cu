// Test and benchmark infrastructure only (never linked into the product):
// the reference's own search path, one query per call, as a persistent
// session -- the "reference kernels + exact-probe shim" arm that bench.py
// times against the product.
//
// What runs, per query, in the reference's order (cpp/src/search_impl.cu):
//   host  FhtKac rotation of the 32 tokens + QueryState      :72-82
//         (the reference rotator via libchimera_ref.so)
//   H2D   rotated queries + cb1 on the h2d stream, event      :84-91
//   GPU   precompute_one_bit_lut_kernel                       :93-95
//   GPU   probe (stand-in for cuVS CAGRA, which is absent here: exact
//         top-nprobe of ||c||^2 - 2<q,c> by cuBLAS SGEMM + a block select)
//   GPU   generate_and_refine_candidates: memsets on the d2h stream, mark,
//         count, ExclusiveSum, D2H + host sync, memset, materialize,
//         partial_score, sum_partial_scores, SortPairsDescending, copy  :118-262
//   mixed collaborative_document_scoring: gather lengths, InclusiveScan,
//         gather positions, D2H + host sync, per chunk token + document
//         scores with events and D2H on the d2h stream; on the host per
//         chunk nth_element x2, unseen-doc selection, the AVX-512 full-bit
//         MaxSim (OpenMP, the reference's unpack + gemv_batch8 via
//         cref_fullbit_doc_scores), heap, final top-k pops     :264-508
//
// The reference kernels come from kernels.cu, compiled unchanged beside this
// file by oracle/Makefile.  Device memory is allocated once per session
// (the reference's allocate_workspace, cpp/src/utils.cu:299-456), sized for
// the worst case of the index, so a search call allocates nothing on the GPU.
#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cub/cub.cuh>
#include <numeric>
#include <queue>
#include <string>
#include <thrust/device_ptr.h>
#include <thrust/functional.h>
#include <thrust/iterator/transform_iterator.h>
#include <vector>

#include "chimera/kernels.cuh"

using namespace Chimera;

// from libchimera_ref.so (oracle/ref_shim.cpp: the reference's rotator and
// its AVX-512 full-bit scorer loop around unpack_func / gemv_batch8_avx512)
extern "C" {
void* cref_rotator_create(size_t dim, size_t padded_dim, uint64_t seed);
void cref_rotator_destroy(void* r);
void cref_rotate(void* r, const float* src, float* dst, size_t count, size_t dim, size_t padded_dim);
void cref_query_state(const float* rotated, size_t padded_dim, size_t ex_bits, float* cb1, float* cbex);
void cref_fullbit_doc_scores(const float* rotated_queries, const float* cbex_sumq, const uint8_t* full_codes,
                             const float* full_factors, const int64_t* doc_ptrs, const int32_t* docs, int count,
                             size_t ex_bits, float* out_scores, int threads);
}

namespace {

struct to_size_t {
    __host__ __device__ size_t operator()(int x) const { return static_cast<size_t>(x); }
};

// ---- exact probe shim -----------------------------------------------------
// One CTA per query token: the nprobe smallest keys of ||c||^2 - 2 dot[c]
// (ties to the lower centroid id) by an 11/11/10-bit radix select over the
// order-preserving key, then one ordered pass that writes the labels.
__device__ __forceinline__ uint32_t probe_key(float cn, float dot) {
    const float d = cn - 2.0f * dot;
    const uint32_t b = __float_as_uint(d);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Exclusive scan of one value per thread over a 1024-thread block.
__device__ uint32_t block_scan_excl(uint32_t v, uint32_t* s_warp, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = s_warp[lane];
        uint32_t z = w;
        for (int off = 1; off < 32; off <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, z, off);
            if (lane >= off) z += y;
        }
        s_warp[lane] = z - w;
        if (lane == 31) s_warp[32] = z;
    }
    __syncthreads();
    const uint32_t r = s_warp[warp] + x - v;
    *total = s_warp[32];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(1024) probe_select_kernel(const float* __restrict__ dots,
                                                            const float* __restrict__ cnorm, int nc, int nprobe,
                                                            uint32_t* __restrict__ labels) {
    __shared__ uint32_t hist[2048];
    __shared__ uint32_t s_warp[33];
    __shared__ uint32_t s_prefix, s_mask, s_need, s_less, s_eq;
    const int row = blockIdx.x;
    const float* dr = dots + (size_t)row * nc;
    if (threadIdx.x == 0) { s_prefix = 0; s_mask = 0; s_need = (uint32_t)nprobe; }
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    for (int lv = 0; lv < 3; ++lv) {
        for (int i = threadIdx.x; i < 2048; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask, need = s_need;
        const uint32_t dm = (1u << widths[lv]) - 1;
        for (int c = threadIdx.x; c < nc; c += blockDim.x) {
            const uint32_t k = probe_key(cnorm[c], dr[c]);
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shifts[lv]) & dm], 1u);
        }
        __syncthreads();
        // thread t owns bins 2t, 2t + 1 (ascending)
        const uint32_t h0 = hist[2 * threadIdx.x], h1 = hist[2 * threadIdx.x + 1];
        uint32_t total;
        const uint32_t before = block_scan_excl(h0 + h1, s_warp, &total);
        if (before < need && before + h0 + h1 >= need) {
            const bool first = before + h0 >= need;
            const uint32_t b = 2 * threadIdx.x + (first ? 0 : 1);
            s_prefix = prefix | (b << shifts[lv]);
            s_mask = mask | (dm << shifts[lv]);
            s_need = need - (first ? before : before + h0);
        }
        __syncthreads();
    }
    // s_prefix is the nprobe-th smallest key; s_need of its copies are taken,
    // lowest ids first
    const uint32_t pivot = s_prefix;
    const uint32_t take_eq = s_need;
    const uint32_t n_less = (uint32_t)nprobe - take_eq;
    if (threadIdx.x == 0) { s_less = 0; s_eq = 0; }
    __syncthreads();
    uint32_t* out = labels + (size_t)row * nprobe;
    for (int base = 0; base < nc; base += blockDim.x) {
        const int c = base + threadIdx.x;
        const uint32_t k = c < nc ? probe_key(cnorm[c], dr[c]) : 0xFFFFFFFFu;
        if (c < nc && k < pivot) out[atomicAdd(&s_less, 1u)] = (uint32_t)c;
        // equal keys (rare) in id order
        const bool eq = c < nc && k == pivot;
        if (__syncthreads_or(eq)) {
            uint32_t tot;
            const uint32_t at = block_scan_excl(eq ? 1u : 0u, s_warp, &tot) + s_eq;
            if (eq && at < take_eq) out[n_less + at] = (uint32_t)c;
            __syncthreads();
            if (threadIdx.x == 0) s_eq += tot;
            __syncthreads();
        }
    }
}

struct Session {
    // index
    int dim = 0, ex_bits = 0, nprobe_max = 0, k_refine_max = 0;
    int64_t n_tokens = 0, num_docs = 0, n_clusters = 0;
    int max_cluster_size = 0;
    std::vector<uint8_t> full_codes;   // host, token order (full_bit_codes_)
    std::vector<float> full_factors;   // host, token order
    std::vector<int64_t> doc_ptrs64;   // host
    void* rotator = nullptr;
    // device
    char* d_codes = nullptr;
    float* d_factor = nullptr;
    int* d_doc_ids = nullptr;
    size_t* d_cpos = nullptr;
    int* d_doc_ptrs = nullptr;
    uint32_t* d_tok2pos = nullptr;
    float* d_cent = nullptr;
    float* d_cnorm = nullptr;
    float* d_queries = nullptr;
    float* d_cb1 = nullptr;
    float* d_lut = nullptr;
    float* d_dots = nullptr;
    uint32_t* d_labels = nullptr;
    uint32_t* d_bitmap = nullptr;
    uint32_t* d_offsets = nullptr;
    int* d_mat_ids = nullptr;
    float* d_pq = nullptr;
    float* d_ps = nullptr;
    int* d_cand_ids = nullptr;
    float* d_sps = nullptr;
    int* d_sids = nullptr;
    int* d_len = nullptr;
    size_t* d_off = nullptr;
    uint32_t* d_rpos = nullptr;
    float* d_tok_scores = nullptr;
    float* d_doc_scores = nullptr;
    void* d_temp = nullptr;
    size_t temp_bytes = 0;
    size_t nb = 0, noff = 0, max_ref_tokens = 0;
    // host pinned
    float* h_queries = nullptr;
    float* h_cb1 = nullptr;
    size_t* h_off = nullptr;
    int* h_ref_ids = nullptr;
    float* h_doc_scores = nullptr;
    uint32_t* h_ncand = nullptr;
    std::vector<char> seen;
    std::vector<int> order;
    cudaStream_t s_compute = nullptr, s_h2d = nullptr, s_d2h = nullptr;
    cudaEvent_t ev_h2d = nullptr;
    cublasHandle_t blas = nullptr;
    int threads = 1;
};

template <typename T>
bool dalloc(T** p, size_t n) {
    return cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T) + 16) == cudaSuccess;
}

void destroy(Session* s) {
    if (!s) return;
    cudaDeviceSynchronize();
    void* dev[] = {s->d_codes, s->d_factor, s->d_doc_ids, s->d_cpos, s->d_doc_ptrs, s->d_tok2pos, s->d_cent,
                   s->d_cnorm, s->d_queries, s->d_cb1, s->d_lut, s->d_dots, s->d_labels, s->d_bitmap,
                   s->d_offsets, s->d_mat_ids, s->d_pq, s->d_ps, s->d_cand_ids, s->d_sps, s->d_sids, s->d_len,
                   s->d_off, s->d_rpos, s->d_tok_scores, s->d_doc_scores, s->d_temp};
    for (void* p : dev)
        if (p) cudaFree(p);
    void* host[] = {s->h_queries, s->h_cb1, s->h_off, s->h_ref_ids, s->h_doc_scores, s->h_ncand};
    for (void* p : host)
        if (p) cudaFreeHost(p);
    if (s->s_compute) cudaStreamDestroy(s->s_compute);
    if (s->s_h2d) cudaStreamDestroy(s->s_h2d);
    if (s->s_d2h) cudaStreamDestroy(s->s_d2h);
    if (s->ev_h2d) cudaEventDestroy(s->ev_h2d);
    if (s->blas) cublasDestroy(s->blas);
    if (s->rotator) cref_rotator_destroy(s->rotator);
    delete s;
}

#define CK(x)                                                                  \
    do {                                                                       \
        cudaError_t e_ = (x);                                                  \
        if (e_ != cudaSuccess) {                                               \
            snprintf(err, errlen, "%s: %s", #x, cudaGetErrorString(e_));       \
            return 1;                                                          \
        }                                                                      \
    } while (0)

}  // namespace

// Uploads the index once.  Host arrays in the reference's layouts: codes1 /
// factor1 / doc_ids cluster ordered, tok2pos, cluster_pos, doc_ptrs, full
// codes and factors in token order (kept on the host for the CPU full-bit
// stage), rotated centroids [n_clusters x 128] and their norms (probe shim).
extern "C" void* cref_session_create(const uint8_t* codes1, const float* factor1, const int32_t* doc_ids,
                                     int64_t n_tokens, const uint64_t* cluster_pos, int64_t n_clusters,
                                     const int64_t* doc_ptrs, int64_t num_docs, const uint32_t* tok2pos,
                                     const uint8_t* full_codes, const float* full_factors, int ex_bits, int dim,
                                     const float* centroids_rot, const float* centroid_norms, int nprobe_max,
                                     int k_refine_max, int threads, char* err, int errlen) {
    err[0] = 0;
    if (nprobe_max <= 0 || nprobe_max > kCandidateRefinementMaxNprobe || k_refine_max <= 0 || num_docs <= 0 ||
        n_clusters <= 0 || n_tokens <= 0 || ex_bits < 1 || ex_bits > 7 || num_docs > (int64_t)INT32_MAX) {
        snprintf(err, errlen, "invalid arguments");
        return nullptr;
    }
    Session* s = new Session();
    auto fail = [&](const char* what) -> void* {
        if (!err[0]) snprintf(err, errlen, "%s", what);
        destroy(s);
        return nullptr;
    };
    s->dim = dim;
    s->ex_bits = ex_bits;
    s->nprobe_max = nprobe_max;
    s->k_refine_max = k_refine_max;
    s->n_tokens = n_tokens;
    s->num_docs = num_docs;
    s->n_clusters = n_clusters;
    s->threads = threads > 0 ? threads : 1;
    const size_t fb = (size_t)PADDED_DIM * (1 + ex_bits) / 8;
    s->full_codes.assign(full_codes, full_codes + (size_t)n_tokens * fb);
    s->full_factors.assign(full_factors, full_factors + n_tokens);
    s->doc_ptrs64.assign(doc_ptrs, doc_ptrs + num_docs + 1);
    int max_doc = 0;
    std::vector<int> dp32(num_docs + 1);
    for (int64_t i = 0; i <= num_docs; ++i) dp32[i] = (int)doc_ptrs[i];
    for (int64_t i = 0; i < num_docs; ++i) max_doc = std::max<int>(max_doc, (int)(doc_ptrs[i + 1] - doc_ptrs[i]));
    for (int64_t c = 0; c < n_clusters; ++c)
        s->max_cluster_size = std::max<int>(s->max_cluster_size, (int)(cluster_pos[c + 1] - cluster_pos[c]));
    s->rotator = cref_rotator_create((size_t)dim, PADDED_DIM, 42);
    if (!s->rotator) return fail("rotator");
    s->nb = candidate_bitmap_num_buckets((size_t)num_docs);
    s->noff = candidate_bitmap_num_offsets(s->nb);
    s->max_ref_tokens = (size_t)k_refine_max * (size_t)max_doc;
    bool ok = dalloc(&s->d_codes, (size_t)n_tokens * CODE_BYTES) && dalloc(&s->d_factor, n_tokens) &&
              dalloc(&s->d_doc_ids, n_tokens) && dalloc(&s->d_cpos, n_clusters + 1) &&
              dalloc(&s->d_doc_ptrs, num_docs + 1) && dalloc(&s->d_tok2pos, n_tokens) &&
              dalloc(&s->d_cent, (size_t)n_clusters * PADDED_DIM) && dalloc(&s->d_cnorm, n_clusters) &&
              dalloc(&s->d_queries, (size_t)Q_DOCLEN * PADDED_DIM) && dalloc(&s->d_cb1, Q_DOCLEN) &&
              dalloc(&s->d_lut, LUT_TOTAL_FLOATS) && dalloc(&s->d_dots, (size_t)Q_DOCLEN * n_clusters) &&
              dalloc(&s->d_labels, (size_t)Q_DOCLEN * nprobe_max) && dalloc(&s->d_bitmap, s->nb) &&
              dalloc(&s->d_offsets, s->noff) && dalloc(&s->d_mat_ids, num_docs) &&
              dalloc(&s->d_pq, (size_t)num_docs * Q_DOCLEN) && dalloc(&s->d_ps, num_docs) &&
              dalloc(&s->d_cand_ids, num_docs) && dalloc(&s->d_sps, num_docs) && dalloc(&s->d_sids, num_docs) &&
              dalloc(&s->d_len, k_refine_max) && dalloc(&s->d_off, (size_t)k_refine_max + 1) &&
              dalloc(&s->d_rpos, s->max_ref_tokens) && dalloc(&s->d_tok_scores, s->max_ref_tokens * Q_DOCLEN) &&
              dalloc(&s->d_doc_scores, k_refine_max);
    if (!ok) return fail("device allocation failed");
    ok = cudaMallocHost(&s->h_queries, sizeof(float) * Q_DOCLEN * PADDED_DIM) == cudaSuccess &&
         cudaMallocHost(&s->h_cb1, sizeof(float) * Q_DOCLEN) == cudaSuccess &&
         cudaMallocHost(&s->h_off, sizeof(size_t) * (k_refine_max + 1)) == cudaSuccess &&
         cudaMallocHost(&s->h_ref_ids, sizeof(int) * k_refine_max) == cudaSuccess &&
         cudaMallocHost(&s->h_doc_scores, sizeof(float) * k_refine_max) == cudaSuccess &&
         cudaMallocHost(&s->h_ncand, sizeof(uint32_t)) == cudaSuccess;
    if (!ok) return fail("pinned allocation failed");
    if (cudaMemcpy(s->d_codes, codes1, (size_t)n_tokens * CODE_BYTES, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->d_factor, factor1, sizeof(float) * n_tokens, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->d_doc_ids, doc_ids, sizeof(int) * n_tokens, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->d_cpos, cluster_pos, sizeof(size_t) * (n_clusters + 1), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(s->d_doc_ptrs, dp32.data(), sizeof(int) * (num_docs + 1), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(s->d_tok2pos, tok2pos, sizeof(uint32_t) * n_tokens, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->d_cent, centroids_rot, sizeof(float) * n_clusters * PADDED_DIM, cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(s->d_cnorm, centroid_norms, sizeof(float) * n_clusters, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail("upload failed");
    // CUB temporary storage: the largest of the three reference calls
    size_t b1 = 0, b2 = 0, b3 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, b1, s->d_offsets, s->d_offsets, (int)s->noff);
    cub::DeviceRadixSort::SortPairsDescending(nullptr, b2, s->d_ps, s->d_sps, s->d_cand_ids, s->d_sids,
                                              (int)num_docs, 0, 32);
    {
        auto it = thrust::make_transform_iterator(thrust::device_ptr<int>(s->d_len), to_size_t());
        cub::DeviceScan::InclusiveScan(nullptr, b3, it, s->d_off + 1, thrust::plus<size_t>(), k_refine_max);
    }
    s->temp_bytes = std::max(b1, std::max(b2, b3));
    if (cudaMalloc(&s->d_temp, s->temp_bytes) != cudaSuccess) return fail("device allocation failed");
    if (cudaStreamCreateWithFlags(&s->s_compute, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s->s_h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s->s_d2h, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->ev_h2d, cudaEventDisableTiming) != cudaSuccess)
        return fail("streams");
    if (cublasCreate(&s->blas) != CUBLAS_STATUS_SUCCESS) return fail("cublas");
    cublasSetMathMode(s->blas, CUBLAS_PEDANTIC_MATH);  // plain fp32, no TF32
    cublasSetStream(s->blas, s->s_compute);
    s->seen.assign((size_t)num_docs, 0);
    s->order.assign((size_t)k_refine_max, 0);
    if (cudaDeviceSynchronize() != cudaSuccess) return fail("synchronize");
    return s;
}

extern "C" void cref_session_destroy(void* h) { destroy(static_cast<Session*>(h)); }

// One search_one call: raw query [32 x dim] (host) -> up to k doc ids.
// n_candidates / n_refined (may be NULL) report the stage sizes.  labels_in
// (host [32 x nprobe], may be NULL) replaces the probe shim's labels, so that
// tests can drive the rest of the path with given probe lists.
extern "C" int cref_session_search(void* h, const float* query, const uint32_t* labels_in, int nprobe,
                                   int k_refine, int k_full_bit, int num_chunks_opt, int k, int64_t* out, int* n_out,
                                   int64_t* n_candidates, int* n_refined, char* err, int errlen) {
    err[0] = 0;
    Session* s = static_cast<Session*>(h);
    *n_out = 0;
    if (!s || nprobe <= 0 || nprobe > s->nprobe_max || k_refine <= 0 || k_refine > s->k_refine_max ||
        k_full_bit <= 0 || num_chunks_opt <= 0 || k <= 0) {
        snprintf(err, errlen, "invalid arguments");
        return 2;
    }
    // ---- search_one: host rotation + QueryState (search_impl.cu:72-82)
    cref_rotate(s->rotator, query, s->h_queries, Q_DOCLEN, (size_t)s->dim, PADDED_DIM);
    float cbex[Q_DOCLEN];
    for (int i = 0; i < Q_DOCLEN; ++i)
        cref_query_state(s->h_queries + (size_t)i * PADDED_DIM, PADDED_DIM, (size_t)s->ex_bits, &s->h_cb1[i],
                         &cbex[i]);
    cudaStream_t st = s->s_compute;
    CK(cudaMemcpyAsync(s->d_queries, s->h_queries, sizeof(float) * Q_DOCLEN * PADDED_DIM, cudaMemcpyHostToDevice,
                       s->s_h2d));
    CK(cudaMemcpyAsync(s->d_cb1, s->h_cb1, sizeof(float) * Q_DOCLEN, cudaMemcpyHostToDevice, s->s_h2d));
    CK(cudaEventRecord(s->ev_h2d, s->s_h2d));
    CK(cudaStreamWaitEvent(st, s->ev_h2d, 0));
    precompute_one_bit_lut_kernel<<<Q_DOCLEN, 256, 0, st>>>(s->d_queries, s->d_lut);
    CK(cudaGetLastError());

    // ---- generate_and_refine_candidates (search_impl.cu:118-262)
    CK(cudaMemsetAsync(s->d_bitmap, 0, s->nb * sizeof(uint32_t), s->s_d2h));
    CK(cudaMemsetAsync(s->d_offsets, 0, s->noff * sizeof(uint32_t), s->s_d2h));
    CK(cudaEventRecord(s->ev_h2d, s->s_d2h));
    if (labels_in) {
        CK(cudaMemcpyAsync(s->d_labels, labels_in, sizeof(uint32_t) * Q_DOCLEN * nprobe, cudaMemcpyHostToDevice, st));
    } else {  // exact probe shim in place of ivf->search_centroids (CAGRA)
        const float one = 1.0f, zero = 0.0f;
        if (cublasSgemm(s->blas, CUBLAS_OP_T, CUBLAS_OP_N, (int)s->n_clusters, Q_DOCLEN, PADDED_DIM, &one,
                        s->d_cent, PADDED_DIM, s->d_queries, PADDED_DIM, &zero, s->d_dots,
                        (int)s->n_clusters) != CUBLAS_STATUS_SUCCESS) {
            snprintf(err, errlen, "cublasSgemm failed");
            return 1;
        }
        probe_select_kernel<<<Q_DOCLEN, 1024, 0, st>>>(s->d_dots, s->d_cnorm, (int)s->n_clusters, nprobe,
                                                       s->d_labels);
        CK(cudaGetLastError());
    }
    CK(cudaStreamWaitEvent(st, s->ev_h2d, 0));
    const int tpb = 256;
    const dim3 grid(std::max((s->max_cluster_size + tpb - 1) / tpb, 16), Q_DOCLEN);
    mark_candidate_documents_kernel<<<grid, tpb, 0, st>>>(s->d_labels, s->d_cpos, s->d_doc_ids, s->d_bitmap,
                                                         (size_t)s->num_docs, nprobe, (size_t)s->n_clusters);
    CK(cudaGetLastError());
    count_candidate_bitmap_kernel<<<(unsigned)((s->nb + tpb - 1) / tpb), tpb, 0, st>>>(s->d_bitmap, s->nb,
                                                                                      s->d_offsets);
    CK(cudaGetLastError());
    size_t tb = s->temp_bytes;
    CK(cub::DeviceScan::ExclusiveSum(s->d_temp, tb, s->d_offsets, s->d_offsets, (int)s->noff, st));
    CK(cudaMemcpyAsync(s->h_ncand, s->d_offsets + s->noff - 1, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    const int n_cand = (int)*s->h_ncand;
    if (n_candidates) *n_candidates = n_cand;
    if (n_refined) *n_refined = 0;
    if (n_cand == 0) return 0;
    if ((int64_t)n_cand > s->num_docs) {
        snprintf(err, errlen, "candidate count exceeds num_docs");
        return 1;
    }
    CK(cudaMemsetAsync(s->d_pq, 0, (size_t)n_cand * Q_DOCLEN * sizeof(float), st));
    materialize_candidate_documents_kernel<<<(unsigned)((s->nb + tpb - 1) / tpb), tpb, 0, st>>>(
        s->d_bitmap, s->nb, s->d_offsets, s->d_mat_ids);
    CK(cudaGetLastError());
    partial_score_kernel<<<grid, tpb, 0, st>>>(s->d_lut, s->d_codes, s->d_factor, s->d_cb1, s->d_labels,
                                               s->d_cpos, s->d_doc_ids, s->d_pq, s->d_bitmap, s->d_offsets, n_cand,
                                               (size_t)s->num_docs, nprobe, (size_t)s->n_clusters);
    CK(cudaGetLastError());
    const int n_ref = std::min(k_refine, n_cand);
    sum_partial_scores_kernel<<<(n_cand + PARTIAL_SCORE_WARPS_PER_BLOCK - 1) / PARTIAL_SCORE_WARPS_PER_BLOCK,
                                PARTIAL_SCORE_WARPS_PER_BLOCK * 32, 0, st>>>(s->d_pq, s->d_mat_ids, s->d_ps,
                                                                             s->d_cand_ids, n_cand);
    CK(cudaGetLastError());
    tb = s->temp_bytes;
    CK(cub::DeviceRadixSort::SortPairsDescending(s->d_temp, tb, s->d_ps, s->d_sps, s->d_cand_ids, s->d_sids, n_cand,
                                                 0, 32, st));
    CK(cudaMemcpyAsync(s->d_cand_ids, s->d_sids, n_ref * sizeof(int), cudaMemcpyDeviceToDevice, st));
    if (n_refined) *n_refined = n_ref;

    // ---- collaborative_document_scoring (search_impl.cu:264-508)
    const int full_bit_target = std::min(k_full_bit, n_ref);
    gather_refined_doc_lengths_kernel<<<(n_ref + 255) / 256, 256, 0, st>>>(s->d_cand_ids, s->d_doc_ptrs, s->d_len,
                                                                         n_ref);
    CK(cudaGetLastError());
    CK(cudaMemsetAsync(s->d_off, 0, sizeof(size_t), st));
    {
        auto it = thrust::make_transform_iterator(thrust::device_ptr<int>(s->d_len), to_size_t());
        tb = s->temp_bytes;
        CK(cub::DeviceScan::InclusiveScan(s->d_temp, tb, it, s->d_off + 1, thrust::plus<size_t>(), n_ref, st));
    }
    gather_refined_token_positions_kernel<<<n_ref, 256, 0, st>>>(s->d_cand_ids, s->d_doc_ptrs, s->d_tok2pos,
                                                                s->d_off, s->d_rpos, n_ref);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(s->h_off, s->d_off, (n_ref + 1) * sizeof(size_t), cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(s->h_ref_ids, s->d_cand_ids, n_ref * sizeof(int), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    const size_t total_tokens = s->h_off[n_ref];
    if (total_tokens > s->max_ref_tokens) {
        snprintf(err, errlen, "refined tokens exceed the workspace");
        return 1;
    }
    const int num_chunks = std::min(num_chunks_opt, n_ref);
    const int chunk_size = (n_ref + num_chunks - 1) / num_chunks;
    std::vector<cudaEvent_t> done(num_chunks), d2h(num_chunks);
    for (int c = 0; c < num_chunks; ++c) {
        CK(cudaEventCreateWithFlags(&done[c], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&d2h[c], cudaEventDisableTiming));
    }
    const size_t lut_smem =
        DOCUMENT_SCORING_LUT_SMEM_FLOATS * sizeof(float) + DOCUMENT_SCORING_LUT_TILE_Q * sizeof(float);
    for (int c = 0; c < num_chunks; ++c) {
        const int c0 = c * chunk_size, c1 = std::min(c0 + chunk_size, n_ref);
        const size_t t0 = s->h_off[c0], t1 = s->h_off[c1];
        if (t1 > t0) {
            one_bit_token_score_kernel<<<(unsigned)((t1 - t0 + 255) / 256), 256, lut_smem, st>>>(
                s->d_lut, s->d_codes, s->d_factor, s->d_cb1, s->d_rpos + t0, s->d_tok_scores + t0, total_tokens,
                t1 - t0);
            CK(cudaGetLastError());
        }
        one_bit_document_score_kernel<<<c1 - c0, 128, 0, st>>>(s->d_tok_scores, s->d_off + c0,
                                                               s->d_doc_scores + c0, total_tokens, c1 - c0);
        CK(cudaGetLastError());
        CK(cudaEventRecord(done[c], st));
        CK(cudaStreamWaitEvent(s->s_d2h, done[c], 0));
        CK(cudaMemcpyAsync(s->h_doc_scores + c0, s->d_doc_scores + c0, (c1 - c0) * sizeof(float),
                           cudaMemcpyDeviceToHost, s->s_d2h));
        CK(cudaEventRecord(d2h[c], s->s_d2h));
    }
    std::priority_queue<std::pair<float, size_t>> heap;
    std::vector<int> seen_list;
    seen_list.reserve(full_bit_target * 2);
    int prev = 0;
    const float* ob = s->h_doc_scores;
    auto desc = [ob](int a, int b) { return ob[a] > ob[b]; };
    std::vector<int32_t> sel_docs;
    std::vector<float> sel_scores;
    for (int c = 0; c < num_chunks; ++c) {
        const int c0 = c * chunk_size, c1 = std::min(c0 + chunk_size, n_ref);
        const int cnt = c1 - c0;
        CK(cudaEventSynchronize(d2h[c]));
        std::iota(s->order.begin() + prev, s->order.begin() + prev + cnt, c0);
        const int merge = prev + cnt;
        const int carry = std::min(full_bit_target, merge);
        std::nth_element(s->order.begin(), s->order.begin() + carry, s->order.begin() + merge, desc);
        const int cum = std::min(full_bit_target * (c + 1) / num_chunks, carry);
        std::nth_element(s->order.begin(), s->order.begin() + cum, s->order.begin() + carry, desc);
        prev = carry;
        std::vector<std::pair<float, int>> fresh;
        fresh.reserve(cum);
        for (int i = 0; i < cum; ++i) {
            const int r = s->order[i];
            if (!s->seen[s->h_ref_ids[r]]) fresh.emplace_back(ob[r], r);
        }
        if (fresh.empty()) continue;
        std::sort(fresh.begin(), fresh.end(), std::greater<>());
        sel_docs.resize(fresh.size());
        sel_scores.resize(fresh.size());
        for (size_t i = 0; i < fresh.size(); ++i) {
            const int d = s->h_ref_ids[fresh[i].second];
            s->seen[d] = 1;
            seen_list.push_back(d);
            sel_docs[i] = d;
        }
        cref_fullbit_doc_scores(s->h_queries, cbex, s->full_codes.data(), s->full_factors.data(),
                                s->doc_ptrs64.data(), sel_docs.data(), (int)sel_docs.size(), (size_t)s->ex_bits,
                                sel_scores.data(), s->threads);
        for (size_t i = 0; i < sel_docs.size(); ++i) heap.emplace(sel_scores[i], (size_t)sel_docs[i]);
    }
    int n = 0;
    for (; n < k && !heap.empty(); ++n) {
        out[n] = (int64_t)heap.top().second;
        heap.pop();
    }
    *n_out = n;
    for (int d : seen_list) s->seen[d] = 0;
    for (int c = 0; c < num_chunks; ++c) {
        cudaEventDestroy(done[c]);
        cudaEventDestroy(d2h[c]);
    }
    return 0;
}
