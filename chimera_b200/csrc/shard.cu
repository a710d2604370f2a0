// Document-sharded search: the kernels between the exchange steps.
//
// Each rank holds the documents [doc_base, doc_base + num_docs) of the
// corpus with local ids.  After the ranks' stage-1 lists are gathered,
// chm_merge_refined rebuilds the refined list the whole corpus would give:
// the top k_refine of the union by (partial score desc, global doc asc),
// which is the reference's stable descending sort of ascending doc ids
// (search_impl.cu:245-261).  A shard's list is the restriction of that order
// to its documents, so the union of the shards' top k_refine holds the
// global top k_refine.  chm_shard_localize turns global ids into this rank's
// local ids (-1 where another shard owns the document), which the refine and
// full-bit kernels skip.
#include <algorithm>

#include "common.cuh"

namespace chm {

constexpr int kMergeThreads = 256;

// key order: partial score desc, global doc asc (scores are >= 0 so the
// float bits order like the values)
__device__ __forceinline__ uint64_t refined_key(float partial, int64_t gdoc) {
    return ((uint64_t)__float_as_uint(partial) << 32) | (uint32_t)(~(uint32_t)gdoc);
}

// One thread per gathered element; its rank in the union is its position in
// its own list plus, for every other list, the number of elements ordered
// before it (binary search: the lists are sorted).  Keys are distinct because
// documents are, so the ranks are a permutation.
__global__ void __launch_bounds__(kMergeThreads) merge_refined_kernel(
    int shards, int nq, int k_refine, const int32_t* __restrict__ docs, const float* __restrict__ partial,
    const int32_t* __restrict__ counts, const int64_t* __restrict__ doc_base, int32_t* __restrict__ out_docs,
    float* __restrict__ out_partial, int32_t* __restrict__ out_counts) {
    const int q = blockIdx.y;
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        int64_t tot = 0;
        for (int s = 0; s < shards; ++s) tot += counts[(size_t)s * nq + q];
        out_counts[q] = (int32_t)(tot < k_refine ? tot : (int64_t)k_refine);
    }
    if (e >= (int64_t)shards * k_refine) return;
    const int s = (int)(e / k_refine), j = (int)(e % k_refine);
    const int cnt = counts[(size_t)s * nq + q];
    if (j >= cnt) return;
    const size_t at = ((size_t)s * nq + q) * k_refine + j;
    const int64_t g = doc_base[s] + docs[at];
    const float p = partial[at];
    const uint64_t key = refined_key(p, g);
    int64_t rank = j;
    for (int o = 0; o < shards && rank < k_refine; ++o) {
        if (o == s) continue;
        const int n = counts[(size_t)o * nq + q];
        const size_t base = ((size_t)o * nq + q) * k_refine;
        int lo = 0, hi = n;  // first position whose key is below ours
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            const uint64_t km = refined_key(partial[base + mid], doc_base[o] + docs[base + mid]);
            if (km > key) lo = mid + 1; else hi = mid;
        }
        rank += lo;
    }
    if (rank < k_refine) {
        out_docs[(size_t)q * k_refine + rank] = (int32_t)g;
        out_partial[(size_t)q * k_refine + rank] = p;
    }
}

__global__ void shard_localize_kernel(int nq, int cap, const int32_t* __restrict__ gdocs,
                                      const int32_t* __restrict__ counts, int64_t doc_base, int64_t num_docs,
                                      int32_t* __restrict__ ldocs) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)nq * cap) return;
    const int q = (int)(i / cap), j = (int)(i % cap);
    int32_t out = -1;
    if (j < counts[q]) {
        const int64_t g = gdocs[i];
        if (g >= doc_base && g < doc_base + num_docs) out = (int32_t)(g - doc_base);
    }
    ldocs[i] = out;
}

chm_status stage1_run(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                      const uint32_t* labels, int32_t nprobe, int32_t k_refine, int32_t* refined_docs,
                      float* refined_partial, int32_t* num_refined, int64_t* num_candidates, void* ws,
                      size_t ws_bytes, cudaStream_t st, bool force_marks, uint32_t* flags_out, int log2_extra);
size_t stage1_bytes(const chm_index* idx, int32_t nq, int32_t nprobe, int extra, int k_refine);

}  // namespace chm

extern "C" chm_status chm_merge_refined(int32_t nq, int32_t shards, int32_t k_refine, const int32_t* docs,
                                        const float* partial, const int32_t* counts, const int64_t* doc_base,
                                        int32_t* out_docs, float* out_partial, int32_t* out_counts,
                                        void* stream) {
    if (nq <= 0) return CHM_OK;
    if (shards <= 0 || k_refine <= 0 || k_refine > CHM_MAX_K_REFINE) return CHM_ERR_INVALID;
    const int64_t n = (int64_t)shards * k_refine;
    dim3 g((unsigned)((n + chm::kMergeThreads - 1) / chm::kMergeThreads), (unsigned)nq);
    chm::merge_refined_kernel<<<g, chm::kMergeThreads, 0, (cudaStream_t)stream>>>(
        shards, nq, k_refine, docs, partial, counts, doc_base, out_docs, out_partial, out_counts);
    return chm::launch_status("merge_refined_kernel");
}

extern "C" chm_status chm_shard_localize(int32_t nq, int32_t cap, const int32_t* global_docs,
                                         const int32_t* counts, int64_t doc_base, int64_t num_docs,
                                         int32_t* local_docs, void* stream) {
    if (nq <= 0) return CHM_OK;
    if (cap <= 0 || doc_base < 0 || num_docs < 0) return CHM_ERR_INVALID;
    const int64_t n = (int64_t)nq * cap;
    chm::shard_localize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        nq, cap, global_docs, counts, doc_base, num_docs, local_docs);
    return chm::launch_status("shard_localize_kernel");
}

extern "C" size_t chm_stage1_ex_workspace_bytes(const chm_index* idx, int32_t nq, int32_t nprobe,
                                                int32_t table_log2_extra) {
    if (!idx || nq <= 0 || nprobe <= 0 || table_log2_extra < 0 || table_log2_extra > 8) return 0;
    // sized for any k_refine (the call's own is not an argument): the
    // dense-bound pass, when it runs (k_refine <= num_docs), needs the same
    // bytes for every k_refine
    const int64_t kr = std::max<int64_t>(1, std::min<int64_t>(CHM_MAX_K_REFINE, idx->num_docs));
    return chm::stage1_bytes(idx, nq, nprobe, table_log2_extra, (int)kr);
}

extern "C" chm_status chm_stage1_ex(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                                    const uint32_t* labels, int32_t nprobe, int32_t k_refine,
                                    int32_t* refined_docs, float* refined_partial, int32_t* num_refined,
                                    uint32_t* flags, int32_t table_log2_extra, void* ws, size_t ws_bytes,
                                    void* stream) {
    if (table_log2_extra < 0 || table_log2_extra > 8) return CHM_ERR_INVALID;
    return chm::stage1_run(idx, nq, lut, cb1, labels, nprobe, k_refine, refined_docs, refined_partial, num_refined,
                           nullptr, ws, ws_bytes, (cudaStream_t)stream, false, flags, table_log2_extra);
}
