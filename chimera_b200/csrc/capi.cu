// C ABI: version / error reporting and the batched end-to-end search.
//
// chm_search runs, per batch of `params->batch` queries, the whole search
// hot path on one stream with no host synchronisation:
//   prepare (rotate, QueryState, LUT) -> exact probe -> stage 1 (scoring,
//   aggregation, top-k_refine) -> 1-bit refinement -> progressive selection
//   -> full-bit MaxSim -> final ordering.
// The reference performs the same stages one query at a time with two host
// round trips and a CPU full-bit stage (search_impl.cu:72-574).
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace chm {

static thread_local char g_err[512] = "";

void set_last_error(const char* where, cudaError_t err) {
    std::snprintf(g_err, sizeof(g_err), "%s: %s", where, cudaGetErrorString(err));
}

void set_last_message(const char* msg) { std::snprintf(g_err, sizeof(g_err), "%s", msg); }

chm_status stage1_run(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                      const uint32_t* labels, int32_t nprobe, int32_t k_refine,
                      int32_t* refined_docs, float* refined_partial, int32_t* num_refined,
                      int64_t* num_candidates, void* ws, size_t ws_bytes, cudaStream_t st,
                      bool force_marks, uint32_t* flags_out, int log2_extra);
size_t stage1_bytes(const chm_index* idx, int32_t nq, int32_t nprobe, int extra, int k_refine);

__global__ void fold_flags_kernel(const uint32_t* __restrict__ flags, int32_t* __restrict__ num_results,
                                  int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && flags[i] != 0) num_results[i] = -(int32_t)flags[i];
}

struct SearchBuffers {
    float* rot;
    float* cb1;
    float* cbex;
    float* lut;
    uint32_t* labels;
    void* probe_ws;
    size_t probe_bytes;
    void* s1_ws;
    size_t s1_bytes;
    void* rt_ws;
    size_t rt_bytes;
    int32_t* refined_docs;
    float* refined_partial;
    float* onebit;
    int32_t* num_refined;
    int32_t* fb_docs;
    float* fb_scores;
    int32_t* num_fb;
    uint32_t* flags;
};

// The tensor-core probe is used when the index carries the bf16 centroids.
static bool use_tc_probe(const chm_index* idx, const chm_search_params* p) {
    return idx->centroids_bf16 != nullptr && idx->centroid_norm_max != nullptr && p->nprobe <= 448;
}

template <typename A>
static void layout(A& a, const chm_index* idx, const chm_search_params* p, SearchBuffers* b) {
    const size_t B = (size_t)p->batch;
    const size_t ntok = B * kQ;
    const size_t probe_bytes = use_tc_probe(idx, p)
                                   ? chm_probe_tc_workspace_bytes((int64_t)ntok, idx->n_clusters, p->nprobe)
                                   : chm_probe_workspace_bytes((int64_t)ntok, idx->n_clusters, p->nprobe);
    const size_t s1_bytes = stage1_bytes(idx, p->batch, p->nprobe, p->table_log2_extra, p->k_refine);
    const size_t rt_bytes = chm_refine_tc_workspace_bytes(idx, p->batch, p->k_refine);
    auto rot = a.template take<float>(ntok * kDim);
    auto cb1 = a.template take<float>(ntok);
    auto cbex = a.template take<float>(ntok);
    auto lut = a.template take<float>(ntok * kLutPerQ);
    auto labels = a.template take<uint32_t>(ntok * p->nprobe);
    auto pws = a.template take<char>(probe_bytes);
    auto sws = a.template take<char>(s1_bytes);
    auto rtws = a.template take<char>(rt_bytes);
    auto rd = a.template take<int32_t>(B * p->k_refine);
    auto rp = a.template take<float>(B * p->k_refine);
    auto ob = a.template take<float>(B * p->k_refine);
    auto nr = a.template take<int32_t>(B);
    auto fd = a.template take<int32_t>(B * p->k_refine);
    auto fs = a.template take<float>(B * p->k_refine);
    auto nf = a.template take<int32_t>(B);
    auto fl = a.template take<uint32_t>(B);
    if (b) {
        *b = SearchBuffers{(float*)rot, (float*)cb1, (float*)cbex, (float*)lut, (uint32_t*)labels,
                           (void*)pws, probe_bytes, (void*)sws, s1_bytes, (void*)rtws, rt_bytes,
                           (int32_t*)rd, (float*)rp,
                           (float*)ob, (int32_t*)nr, (int32_t*)fd, (float*)fs, (int32_t*)nf,
                           (uint32_t*)fl};
    }
}

struct SizerT {
    Sizer s;
    template <typename T>
    void* take(size_t n) {
        s.take<T>(n);
        return nullptr;
    }
};

static chm_status validate(const chm_index* idx, const chm_search_params* p) {
    if (!idx || !p) return CHM_ERR_INVALID;
    if (p->nprobe <= 0 || p->k_refine <= 0 || p->k_full_bit <= 0 || p->num_chunks <= 0 || p->k <= 0 ||
        p->batch <= 0)
        return CHM_ERR_INVALID;
    if (p->k_full_bit > p->k_refine) return CHM_ERR_INVALID;  // chimera_index.cu:100-102
    if (p->nprobe > idx->n_clusters || p->nprobe > CHM_MAX_NPROBE) return CHM_ERR_INVALID;
    if (p->k_refine > CHM_MAX_K_REFINE || p->k > CHM_MAX_K) return CHM_ERR_INVALID;
    if (p->table_log2_extra < 0 || p->table_log2_extra > 8) return CHM_ERR_INVALID;
    return CHM_OK;
}

}  // namespace chm

extern "C" const char* chm_version(void) { return "chimera_b200 0.1 (sm_100a)"; }

extern "C" const char* chm_last_error(void) { return chm::g_err; }

extern "C" size_t chm_search_workspace_bytes(const chm_index* idx, const chm_search_params* p) {
    if (chm::validate(idx, p) != CHM_OK) return 0;
    chm::SizerT s;
    chm::layout(s, idx, p, nullptr);
    return s.s.off;
}

extern "C" chm_status chm_search(const chm_index* idx, const chm_search_params* p,
                                 const float* queries, int64_t num_queries, int64_t* results,
                                 int32_t* num_results, void* ws, size_t ws_bytes, void* stream) {
    CHM_TRY(chm::validate(idx, p));
    if (num_queries < 0) return CHM_ERR_INVALID;
    if (num_queries == 0) return CHM_OK;
    chm::Arena a(ws, ws_bytes);
    chm::SearchBuffers b;
    chm::layout(a, idx, p, &b);
    if (a.overflow) return CHM_ERR_CAPACITY;
    cudaStream_t st = (cudaStream_t)stream;
    const int fb_cap = p->k_refine;
    for (int64_t q0 = 0; q0 < num_queries; q0 += p->batch) {
        const int nq = (int)std::min<int64_t>(p->batch, num_queries - q0);
        const int64_t ntok = (int64_t)nq * chm::kQ;
        CHM_TRY(chm_prepare_queries(idx->flips, idx->dim, idx->ex_bits,
                                    queries + q0 * chm::kQ * idx->dim, ntok, b.rot, b.cb1, b.cbex,
                                    b.lut, st));
        if (chm::use_tc_probe(idx, p))
            CHM_TRY(chm_probe_tc(b.rot, ntok, idx->centroids, idx->centroids_bf16, idx->centroid_norms,
                                 idx->centroid_norm_max, idx->n_clusters, p->nprobe, b.labels, b.probe_ws,
                                 b.probe_bytes, st));
        else
            CHM_TRY(chm_probe(b.rot, ntok, idx->centroids, idx->centroid_norms, idx->n_clusters,
                              p->nprobe, b.labels, b.probe_ws, b.probe_bytes, st));
        CHM_TRY(chm::stage1_run(idx, nq, b.lut, b.cb1, b.labels, p->nprobe, p->k_refine,
                                b.refined_docs, b.refined_partial, b.num_refined, nullptr, b.s1_ws,
                                b.s1_bytes, st, false, b.flags, p->table_log2_extra));
        // the tensor-core filters pay off on batches; a few queries are faster
        // with the plain kernels' single launch (same scores either way)
        if (nq >= 16)
            CHM_TRY(chm_refine_1bit_tc(idx, nq, b.lut, b.cb1, b.rot, b.refined_docs, b.num_refined, p->k_refine,
                                       b.onebit, b.rt_ws, b.rt_bytes, st));
        else
            CHM_TRY(chm_refine_1bit(idx, nq, b.lut, b.cb1, b.refined_docs, b.num_refined, p->k_refine,
                                    b.onebit, st));
        CHM_TRY(chm_select_fullbit(nq, b.refined_docs, b.onebit, b.num_refined, p->k_refine,
                                   p->k_full_bit, p->num_chunks, b.fb_docs, b.num_fb, fb_cap, st));
        if (nq >= 16)
            CHM_TRY(chm_fullbit_score_tc(idx, nq, b.rot, b.cbex, b.fb_docs, b.num_fb, fb_cap, b.fb_scores, b.rt_ws,
                                         b.rt_bytes, st));
        else
            CHM_TRY(chm_fullbit_score(idx, nq, b.rot, b.cbex, b.fb_docs, b.num_fb, fb_cap, b.fb_scores, st));
        CHM_TRY(chm_final_topk(nq, b.fb_docs, b.fb_scores, b.num_fb, fb_cap, p->k, results + q0 * p->k,
                               num_results + q0, st));
        chm::fold_flags_kernel<<<(nq + 255) / 256, 256, 0, st>>>(b.flags, num_results + q0, nq);
        CHM_TRY(chm::launch_status("fold_flags_kernel"));
    }
    return CHM_OK;
}
