// Test infrastructure only (never linked into the product): drives the
// reference's own CUDA kernels (kernels.cu, compiled from the reference
// sources by oracle/Makefile) for one query, launching them with the
// reference's grid shapes and in its order:
//
//   precompute_one_bit_lut_kernel          search_impl.cu:92-94
//   mark / count / ExclusiveSum / materialize / partial_score /
//   sum_partial_scores / SortPairsDescending  search_impl.cu:118-262
//   gather lengths / InclusiveScan / gather positions, then per chunk
//   one_bit_token_score + one_bit_document_score  search_impl.cu:264-420
//
// so that the plain-C oracle's restatement of those stages can be pinned
// to the reference's outputs on the same inputs.  The probe lists are an
// input (the reference's CAGRA probe is replaced by the exact probe).
//
// Host arrays in, host arrays out; device memory is allocated per call.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cub/cub.cuh>
#include <vector>

#include "chimera/kernels.cuh"

using namespace Chimera;

namespace {

struct Dev {
    std::vector<void*> ptrs;
    ~Dev() {
        for (void* p : ptrs) cudaFree(p);
    }
    template <typename T>
    T* alloc(size_t n) {
        void* p = nullptr;
        if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) return nullptr;
        ptrs.push_back(p);
        return static_cast<T*>(p);
    }
    template <typename T>
    T* upload(const T* h, size_t n) {
        T* d = alloc<T>(n);
        if (d && n) cudaMemcpy(d, h, n * sizeof(T), cudaMemcpyHostToDevice);
        return d;
    }
};

#define CK(x)                                                                              \
    do {                                                                                   \
        cudaError_t e_ = (x);                                                              \
        if (e_ != cudaSuccess) {                                                           \
            snprintf(err, errlen, "%s: %s", #x, cudaGetErrorString(e_));                  \
            return 1;                                                                      \
        }                                                                                  \
    } while (0)

}  // namespace

// Outputs:
//   lut_out[32 * 512]                        the reference LUT
//   n_candidates                             candidate docs (visited docs)
//   refined_docs[k_refine], refined_partial  sorted prefix of the candidate list
//   n_refined = min(k_refine, n_candidates)
//   onebit[k_refine]                         1-bit document scores of the refined docs
extern "C" int cref_gpu_query_stages(
    const float* rot_queries, const float* cb1, const uint32_t* labels, int nprobe,
    const uint8_t* codes1, const float* factor1, const int32_t* doc_ids, int64_t n_tokens,
    const uint64_t* cluster_pos, int64_t n_clusters, const int32_t* doc_ptrs,
    const uint32_t* tok2pos, int64_t num_docs, int k_refine, int num_chunks_opt, float* lut_out,
    int64_t* n_candidates_out, int32_t* refined_docs, float* refined_partial, int32_t* n_refined_out,
    float* onebit, char* err, int errlen) {
    err[0] = 0;
    if (nprobe <= 0 || nprobe > kCandidateRefinementMaxNprobe || k_refine <= 0 || num_chunks_opt <= 0 ||
        num_docs <= 0 || n_clusters <= 0 || n_tokens <= 0) {
        snprintf(err, errlen, "invalid arguments");
        return 2;
    }
    for (int i = 0; i < Q_DOCLEN * nprobe; ++i)
        if (labels[i] >= (uint64_t)n_clusters) {
            snprintf(err, errlen, "label out of range");
            return 2;
        }
    int max_cluster_size = 0;
    for (int64_t c = 0; c < n_clusters; ++c)
        max_cluster_size = std::max<int>(max_cluster_size, (int)(cluster_pos[c + 1] - cluster_pos[c]));

    Dev d;
    float* d_q = d.upload(rot_queries, (size_t)Q_DOCLEN * PADDED_DIM);
    float* d_cb1 = d.upload(cb1, Q_DOCLEN);
    uint32_t* d_labels = d.upload(labels, (size_t)Q_DOCLEN * nprobe);
    char* d_codes = reinterpret_cast<char*>(d.upload(codes1, (size_t)n_tokens * CODE_BYTES));
    float* d_factor = d.upload(factor1, (size_t)n_tokens);
    int* d_doc_ids = d.upload(doc_ids, (size_t)n_tokens);
    size_t* d_cpos = reinterpret_cast<size_t*>(d.upload(cluster_pos, (size_t)n_clusters + 1));
    int* d_doc_ptrs = d.upload(doc_ptrs, (size_t)num_docs + 1);
    uint32_t* d_tok2pos = d.upload(tok2pos, (size_t)n_tokens);
    float* d_lut = d.alloc<float>(LUT_TOTAL_FLOATS);
    const size_t nb = candidate_bitmap_num_buckets((size_t)num_docs);
    const size_t noff = candidate_bitmap_num_offsets(nb);
    uint32_t* d_bitmap = d.alloc<uint32_t>(nb);
    uint32_t* d_offsets = d.alloc<uint32_t>(noff);
    int* d_cand = d.alloc<int>((size_t)num_docs);
    float* d_pq = d.alloc<float>((size_t)num_docs * Q_DOCLEN);
    float* d_ps = d.alloc<float>((size_t)num_docs);
    int* d_ids = d.alloc<int>((size_t)num_docs);
    float* d_sps = d.alloc<float>((size_t)num_docs);
    int* d_sids = d.alloc<int>((size_t)num_docs);
    if (!d_q || !d_cb1 || !d_labels || !d_codes || !d_factor || !d_doc_ids || !d_cpos || !d_doc_ptrs ||
        !d_tok2pos || !d_lut || !d_bitmap || !d_offsets || !d_cand || !d_pq || !d_ps || !d_ids || !d_sps ||
        !d_sids) {
        snprintf(err, errlen, "device allocation failed");
        return 1;
    }

    precompute_one_bit_lut_kernel<<<Q_DOCLEN, 256>>>(d_q, d_lut);
    CK(cudaGetLastError());
    CK(cudaMemcpy(lut_out, d_lut, sizeof(float) * LUT_TOTAL_FLOATS, cudaMemcpyDeviceToHost));

    CK(cudaMemset(d_bitmap, 0, nb * sizeof(uint32_t)));
    CK(cudaMemset(d_offsets, 0, noff * sizeof(uint32_t)));
    const int tpb = 256;
    const dim3 grid(std::max((max_cluster_size + tpb - 1) / tpb, 16), Q_DOCLEN);
    mark_candidate_documents_kernel<<<grid, tpb>>>(d_labels, d_cpos, d_doc_ids, d_bitmap, (size_t)num_docs,
                                                   nprobe, (size_t)n_clusters);
    CK(cudaGetLastError());
    count_candidate_bitmap_kernel<<<(unsigned)((nb + tpb - 1) / tpb), tpb>>>(d_bitmap, nb, d_offsets);
    CK(cudaGetLastError());
    size_t scan_bytes = 0;
    CK(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, d_offsets, d_offsets, (int)noff));
    size_t sort_bytes = 0;
    CK(cub::DeviceRadixSort::SortPairsDescending(nullptr, sort_bytes, d_ps, d_sps, d_ids, d_sids,
                                                 (int)num_docs, 0, 32));
    void* d_temp = d.alloc<char>(std::max(scan_bytes, sort_bytes));
    if (!d_temp) {
        snprintf(err, errlen, "device allocation failed");
        return 1;
    }
    CK(cub::DeviceScan::ExclusiveSum(d_temp, scan_bytes, d_offsets, d_offsets, (int)noff));
    uint32_t n_cand_u32 = 0;
    CK(cudaMemcpy(&n_cand_u32, d_offsets + noff - 1, sizeof(uint32_t), cudaMemcpyDeviceToHost));
    const int n_cand = (int)n_cand_u32;
    *n_candidates_out = n_cand;
    *n_refined_out = 0;
    if (n_cand == 0) return 0;
    if ((int64_t)n_cand > num_docs) {
        snprintf(err, errlen, "candidate count exceeds num_docs");
        return 1;
    }
    CK(cudaMemset(d_pq, 0, (size_t)n_cand * Q_DOCLEN * sizeof(float)));
    materialize_candidate_documents_kernel<<<(unsigned)((nb + tpb - 1) / tpb), tpb>>>(d_bitmap, nb, d_offsets,
                                                                                      d_cand);
    CK(cudaGetLastError());
    partial_score_kernel<<<grid, tpb>>>(d_lut, d_codes, d_factor, d_cb1, d_labels, d_cpos, d_doc_ids, d_pq,
                                        d_bitmap, d_offsets, n_cand, (size_t)num_docs, nprobe,
                                        (size_t)n_clusters);
    CK(cudaGetLastError());
    const int n_ref = std::min(k_refine, n_cand);
    sum_partial_scores_kernel<<<(n_cand + PARTIAL_SCORE_WARPS_PER_BLOCK - 1) / PARTIAL_SCORE_WARPS_PER_BLOCK,
                                PARTIAL_SCORE_WARPS_PER_BLOCK * 32>>>(d_pq, d_cand, d_ps, d_ids, n_cand);
    CK(cudaGetLastError());
    CK(cub::DeviceRadixSort::SortPairsDescending(d_temp, sort_bytes, d_ps, d_sps, d_ids, d_sids, n_cand, 0,
                                                 32));
    CK(cudaMemcpy(refined_docs, d_sids, sizeof(int) * n_ref, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(refined_partial, d_sps, sizeof(float) * n_ref, cudaMemcpyDeviceToHost));
    *n_refined_out = n_ref;

    // ---- 1-bit document scores of the refined docs -------------------------
    int* d_rdocs = d_sids;  // the sorted prefix is the refined list
    int* d_len = d.alloc<int>(n_ref);
    size_t* d_off = d.alloc<size_t>((size_t)n_ref + 1);
    if (!d_len || !d_off) {
        snprintf(err, errlen, "device allocation failed");
        return 1;
    }
    gather_refined_doc_lengths_kernel<<<(n_ref + 255) / 256, 256>>>(d_rdocs, d_doc_ptrs, d_len, n_ref);
    CK(cudaGetLastError());
    std::vector<int> h_len(n_ref);
    CK(cudaMemcpy(h_len.data(), d_len, sizeof(int) * n_ref, cudaMemcpyDeviceToHost));
    // inclusive prefix of the lengths (the reference scans on the device;
    // an integer prefix sum has one result)
    std::vector<size_t> h_off(n_ref + 1, 0);
    for (int i = 0; i < n_ref; ++i) h_off[i + 1] = h_off[i] + (size_t)h_len[i];
    CK(cudaMemcpy(d_off, h_off.data(), sizeof(size_t) * (n_ref + 1), cudaMemcpyHostToDevice));
    const size_t total_tokens = h_off[n_ref];
    uint32_t* d_rpos = d.alloc<uint32_t>(total_tokens);
    float* d_tok_scores = d.alloc<float>(total_tokens * Q_DOCLEN);
    float* d_doc_scores = d.alloc<float>(n_ref);
    if (!d_rpos || !d_tok_scores || !d_doc_scores) {
        snprintf(err, errlen, "device allocation failed");
        return 1;
    }
    gather_refined_token_positions_kernel<<<n_ref, 256>>>(d_rdocs, d_doc_ptrs, d_tok2pos, d_off, d_rpos, n_ref);
    CK(cudaGetLastError());
    const int num_chunks = std::min(num_chunks_opt, n_ref);
    const int chunk_size = (n_ref + num_chunks - 1) / num_chunks;
    const size_t lut_smem = DOCUMENT_SCORING_LUT_SMEM_FLOATS * sizeof(float) + DOCUMENT_SCORING_LUT_TILE_Q * sizeof(float);
    int score_threads = 128;
    for (int c = 0; c < num_chunks; ++c) {
        const int s = c * chunk_size;
        const int e = std::min(s + chunk_size, n_ref);
        if (e <= s) continue;
        const size_t t0 = h_off[s], t1 = h_off[e];
        if (t1 > t0) {
            one_bit_token_score_kernel<<<(unsigned)((t1 - t0 + 255) / 256), 256, lut_smem>>>(
                d_lut, d_codes, d_factor, d_cb1, d_rpos + t0, d_tok_scores + t0, total_tokens, t1 - t0);
            CK(cudaGetLastError());
        }
        one_bit_document_score_kernel<<<e - s, score_threads>>>(d_tok_scores, d_off + s, d_doc_scores + s,
                                                                total_tokens, e - s);
        CK(cudaGetLastError());
    }
    CK(cudaMemcpy(onebit, d_doc_scores, sizeof(float) * n_ref, cudaMemcpyDeviceToHost));
    CK(cudaDeviceSynchronize());
    return 0;
}
