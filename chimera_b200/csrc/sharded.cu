// Document-sharded search over NCCL: the exchange protocol of
// include/chimera_b200_sharded.h, with the stage kernels of the C ABI and the
// collectives enqueued on one stream.  Built into lib/libchimera_nccl.so
// (links NCCL and libchimera_b200.so), so the core library has no NCCL
// dependency.
#include <nccl.h>

#include <cstdio>
#include <cstring>

#include "chimera_b200_sharded.h"
#include "common.cuh"

struct chm_comm {
    ncclComm_t nccl;
    int32_t world;
    int32_t rank;
    int32_t device;
};

namespace chm {
namespace {

// NCCL failures are reported through chm_last_error like CUDA ones.
chm_status nccl_status(ncclResult_t r, const char* where) {
    if (r == ncclSuccess) return CHM_OK;
    char msg[256];
    std::snprintf(msg, sizeof(msg), "%s: %s", where, ncclGetErrorString(r));
    set_last_message(msg);
    return CHM_ERR_CUDA;
}

__global__ void fold_shard_flags_kernel(const int32_t* __restrict__ flags, int32_t* __restrict__ num_results, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && flags[i] != 0) num_results[i] = -flags[i];
}

bool use_tc_probe(const chm_index* idx, const chm_search_params* p) {
    return idx->centroids_bf16 != nullptr && idx->centroid_norm_max != nullptr && p->nprobe <= 448;
}

struct ShardBuffers {
    float* rot;
    float* cb1;
    float* cbex;
    float* lut;
    uint32_t* my_labels;   // [per][nprobe]
    uint32_t* labels;      // [world][per][nprobe] (the first 32 B rows are the batch's)
    void* probe_ws;
    size_t probe_bytes;
    void* s1_ws;
    size_t s1_bytes;
    void* rt_ws;
    size_t rt_bytes;
    int32_t* rd;           // [B][kr] local ids
    float* rp;
    int32_t* nr;           // [B]
    int32_t* flags;        // [B]
    int32_t* g_rd;         // [world][B][kr]
    float* g_rp;
    int32_t* g_nr;         // [world][B]
    int64_t* doc_base;     // [world]
    int32_t* mdocs;        // [B][kr] global ids
    float* mpart;
    int32_t* mcount;       // [B]
    int32_t* local;        // [B][kr]
    float* onebit;         // [B][kr]
    int32_t* fd;           // [B][kr] global ids
    int32_t* nf;           // [B]
    int32_t* fb_local;     // [B][kr]
    float* fs;             // [B][kr]
};

template <typename A>
void shard_layout(A& a, const chm_index* idx, const chm_search_params* p, int world, ShardBuffers* b) {
    const size_t B = (size_t)p->batch, kr = (size_t)p->k_refine, rows = B * kQ;
    const size_t per = (rows + world - 1) / world;
    const size_t probe_bytes = use_tc_probe(idx, p)
                                   ? chm_probe_tc_workspace_bytes((int64_t)per, idx->n_clusters, p->nprobe)
                                   : chm_probe_workspace_bytes((int64_t)per, idx->n_clusters, p->nprobe);
    const size_t s1_bytes = chm_stage1_ex_workspace_bytes(idx, p->batch, p->nprobe, p->table_log2_extra);
    const size_t rt_bytes = chm_refine_tc_workspace_bytes(idx, p->batch, p->k_refine);
    ShardBuffers s;
    s.rot = (float*)a.template take<float>(rows * kDim);
    s.cb1 = (float*)a.template take<float>(rows);
    s.cbex = (float*)a.template take<float>(rows);
    s.lut = (float*)a.template take<float>(rows * kLutPerQ);
    s.my_labels = (uint32_t*)a.template take<uint32_t>(per * p->nprobe);
    s.labels = (uint32_t*)a.template take<uint32_t>((size_t)world * per * p->nprobe);
    s.probe_ws = a.template take<char>(probe_bytes);
    s.probe_bytes = probe_bytes;
    s.s1_ws = a.template take<char>(s1_bytes);
    s.s1_bytes = s1_bytes;
    s.rt_ws = a.template take<char>(rt_bytes);
    s.rt_bytes = rt_bytes;
    s.rd = (int32_t*)a.template take<int32_t>(B * kr);
    s.rp = (float*)a.template take<float>(B * kr);
    s.nr = (int32_t*)a.template take<int32_t>(B);
    s.flags = (int32_t*)a.template take<int32_t>(B);
    s.g_rd = (int32_t*)a.template take<int32_t>((size_t)world * B * kr);
    s.g_rp = (float*)a.template take<float>((size_t)world * B * kr);
    s.g_nr = (int32_t*)a.template take<int32_t>((size_t)world * B);
    s.doc_base = (int64_t*)a.template take<int64_t>((size_t)world);
    s.mdocs = (int32_t*)a.template take<int32_t>(B * kr);
    s.mpart = (float*)a.template take<float>(B * kr);
    s.mcount = (int32_t*)a.template take<int32_t>(B);
    s.local = (int32_t*)a.template take<int32_t>(B * kr);
    s.onebit = (float*)a.template take<float>(B * kr);
    s.fd = (int32_t*)a.template take<int32_t>(B * kr);
    s.nf = (int32_t*)a.template take<int32_t>(B);
    s.fb_local = (int32_t*)a.template take<int32_t>(B * kr);
    s.fs = (float*)a.template take<float>(B * kr);
    if (b) *b = s;
}

struct ShardSizer {
    Sizer s;
    template <typename T>
    void* take(size_t n) {
        s.take<T>(n);
        return nullptr;
    }
};

chm_status validate(const chm_index* idx, const chm_search_params* p, const chm_shard* sh, const chm_comm* comm) {
    if (!idx || !p || !sh || !comm || !sh->doc_base) return CHM_ERR_INVALID;
    if (sh->world <= 0 || sh->rank < 0 || sh->rank >= sh->world) return CHM_ERR_INVALID;
    if (comm->world != sh->world || comm->rank != sh->rank) return CHM_ERR_INVALID;
    if (p->nprobe <= 0 || p->k_refine <= 0 || p->k_full_bit <= 0 || p->num_chunks <= 0 || p->k <= 0 ||
        p->batch <= 0 || p->k_full_bit > p->k_refine)
        return CHM_ERR_INVALID;
    if (p->nprobe > idx->n_clusters || p->nprobe > CHM_MAX_NPROBE || p->k_refine > CHM_MAX_K_REFINE ||
        p->k > CHM_MAX_K || p->table_log2_extra < 0 || p->table_log2_extra > 8)
        return CHM_ERR_INVALID;
    if (sh->doc_base[sh->rank + 1] - sh->doc_base[sh->rank] != idx->num_docs) return CHM_ERR_INVALID;
    return CHM_OK;
}

}  // namespace
}  // namespace chm

extern "C" chm_status chm_comm_unique_id(uint8_t id[CHM_COMM_ID_BYTES]) {
    static_assert(sizeof(ncclUniqueId) == CHM_COMM_ID_BYTES, "NCCL unique id size");
    if (!id) return CHM_ERR_INVALID;
    ncclUniqueId u;
    CHM_TRY(chm::nccl_status(ncclGetUniqueId(&u), "ncclGetUniqueId"));
    std::memcpy(id, &u, sizeof(u));
    return CHM_OK;
}

extern "C" chm_status chm_comm_init(const uint8_t id[CHM_COMM_ID_BYTES], int32_t world, int32_t rank, int32_t device,
                                    chm_comm** out) {
    if (!id || !out || world <= 0 || rank < 0 || rank >= world || device < 0) return CHM_ERR_INVALID;
    *out = nullptr;
    CHM_CUDA(cudaSetDevice(device));
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    CHM_TRY(chm::nccl_status(ncclCommInitRank(&c, world, u, rank), "ncclCommInitRank"));
    *out = new chm_comm{c, world, rank, device};
    return CHM_OK;
}

extern "C" chm_status chm_comm_init_all(int32_t ndev, const int32_t* devices, chm_comm** comms) {
    if (ndev <= 0 || !devices || !comms) return CHM_ERR_INVALID;
    ncclComm_t* c = new ncclComm_t[ndev];
    const chm_status s = chm::nccl_status(ncclCommInitAll(c, ndev, devices), "ncclCommInitAll");
    if (s == CHM_OK)
        for (int i = 0; i < ndev; ++i) comms[i] = new chm_comm{c[i], ndev, i, devices[i]};
    delete[] c;
    return s;
}

extern "C" chm_status chm_comm_destroy(chm_comm* comm) {
    if (!comm) return CHM_OK;
    const ncclResult_t r = ncclCommDestroy(comm->nccl);
    delete comm;
    return chm::nccl_status(r, "ncclCommDestroy");
}

extern "C" size_t chm_search_sharded_workspace_bytes(const chm_index* idx, const chm_search_params* p, int32_t world) {
    if (!idx || !p || world <= 0 || p->batch <= 0 || p->k_refine <= 0 || p->nprobe <= 0) return 0;
    chm::ShardSizer s;
    chm::shard_layout(s, idx, p, world, nullptr);
    return s.s.off;
}

extern "C" chm_status chm_search_sharded(const chm_index* idx, const chm_search_params* p, const chm_shard* sh,
                                         chm_comm* comm, const float* queries, int64_t num_queries, int64_t* results,
                                         int32_t* num_results, void* ws, size_t ws_bytes, void* stream,
                                         float* timing) {
    CHM_TRY(chm::validate(idx, p, sh, comm));
    if (num_queries < 0) return CHM_ERR_INVALID;
    if (num_queries == 0) return CHM_OK;
    const int world = sh->world, rank = sh->rank;
    chm::Arena a(ws, ws_bytes);
    chm::ShardBuffers b;
    chm::shard_layout(a, idx, p, world, &b);
    if (a.overflow) return CHM_ERR_CAPACITY;
    cudaStream_t st = (cudaStream_t)stream;
    const int kr = p->k_refine;
    CHM_CUDA(cudaMemcpyAsync(b.doc_base, sh->doc_base, sizeof(int64_t) * world, cudaMemcpyHostToDevice, st));
    cudaEvent_t evs[CHM_SH_STEPS + 1] = {};
    const bool timed = timing != nullptr;
    if (timed)
        for (int i = 0; i <= CHM_SH_STEPS; ++i) CHM_CUDA(cudaEventCreate(&evs[i]));
    chm_status status = CHM_OK;
    auto run = [&]() -> chm_status {
        for (int64_t q0 = 0; q0 < num_queries; q0 += p->batch) {
            const int nq = (int)std::min<int64_t>(p->batch, num_queries - q0);
            const bool last = q0 + p->batch >= num_queries;
            auto mark = [&](int step) -> chm_status {
                if (timed && last) CHM_CUDA(cudaEventRecord(evs[step], st));
                return CHM_OK;
            };
            const int64_t rows = (int64_t)nq * chm::kQ;
            const int64_t per = (rows + world - 1) / world;
            const int64_t lo = std::min<int64_t>((int64_t)rank * per, rows), hi = std::min<int64_t>(lo + per, rows);
            CHM_TRY(mark(CHM_SH_PREPARE));
            CHM_TRY(chm_prepare_queries(idx->flips, idx->dim, idx->ex_bits, queries + q0 * chm::kQ * idx->dim, rows,
                                        b.rot, b.cb1, b.cbex, b.lut, st));
            CHM_TRY(mark(CHM_SH_PROBE));
            // this rank's rows of the probe; rows past the batch stay 0 (valid ids, never read)
            CHM_CUDA(cudaMemsetAsync(b.my_labels, 0, sizeof(uint32_t) * per * p->nprobe, st));
            if (hi > lo) {
                if (chm::use_tc_probe(idx, p))
                    CHM_TRY(chm_probe_tc(b.rot + lo * chm::kDim, hi - lo, idx->centroids, idx->centroids_bf16,
                                         idx->centroid_norms, idx->centroid_norm_max, idx->n_clusters, p->nprobe,
                                         b.my_labels, b.probe_ws, b.probe_bytes, st));
                else
                    CHM_TRY(chm_probe(b.rot + lo * chm::kDim, hi - lo, idx->centroids, idx->centroid_norms,
                                      idx->n_clusters, p->nprobe, b.my_labels, b.probe_ws, b.probe_bytes, st));
            }
            CHM_TRY(mark(CHM_SH_GATHER_LABELS));
            CHM_TRY(chm::nccl_status(ncclAllGather(b.my_labels, b.labels, (size_t)per * p->nprobe, ncclUint32,
                                                   comm->nccl, st),
                                     "ncclAllGather(labels)"));
            CHM_TRY(mark(CHM_SH_STAGE1));
            CHM_TRY(chm_stage1_ex(idx, nq, b.lut, b.cb1, b.labels, p->nprobe, kr, b.rd, b.rp, b.nr,
                                  reinterpret_cast<uint32_t*>(b.flags), p->table_log2_extra, b.s1_ws, b.s1_bytes,
                                  st));
            CHM_TRY(mark(CHM_SH_GATHER_LISTS));
            // the lists are gathered as [world][nq][kr]: each rank's block holds nq rows
            CHM_TRY(chm::nccl_status(ncclGroupStart(), "ncclGroupStart"));
            CHM_TRY(chm::nccl_status(ncclAllGather(b.rd, b.g_rd, (size_t)nq * kr, ncclInt32, comm->nccl, st),
                                     "ncclAllGather(docs)"));
            CHM_TRY(chm::nccl_status(ncclAllGather(b.rp, b.g_rp, (size_t)nq * kr, ncclFloat32, comm->nccl, st),
                                     "ncclAllGather(partial)"));
            CHM_TRY(chm::nccl_status(ncclAllGather(b.nr, b.g_nr, (size_t)nq, ncclInt32, comm->nccl, st),
                                     "ncclAllGather(counts)"));
            CHM_TRY(chm::nccl_status(ncclAllReduce(b.flags, b.flags, (size_t)nq, ncclInt32, ncclMax, comm->nccl, st),
                                     "ncclAllReduce(flags)"));
            CHM_TRY(chm::nccl_status(ncclGroupEnd(), "ncclGroupEnd"));
            CHM_TRY(mark(CHM_SH_MERGE));
            CHM_TRY(chm_merge_refined(nq, world, kr, b.g_rd, b.g_rp, b.g_nr, b.doc_base, b.mdocs, b.mpart, b.mcount,
                                      st));
            CHM_TRY(chm_shard_localize(nq, kr, b.mdocs, b.mcount, sh->doc_base[rank], idx->num_docs, b.local, st));
            CHM_TRY(mark(CHM_SH_REFINE));
            if (nq >= 16)
                CHM_TRY(chm_refine_1bit_tc(idx, nq, b.lut, b.cb1, b.rot, b.local, b.mcount, kr, b.onebit, b.rt_ws,
                                           b.rt_bytes, st));
            else
                CHM_TRY(chm_refine_1bit(idx, nq, b.lut, b.cb1, b.local, b.mcount, kr, b.onebit, st));
            CHM_TRY(mark(CHM_SH_REDUCE_ONEBIT));
            CHM_TRY(chm::nccl_status(
                ncclAllReduce(b.onebit, b.onebit, (size_t)nq * kr, ncclFloat32, ncclMax, comm->nccl, st),
                "ncclAllReduce(1-bit)"));
            CHM_TRY(mark(CHM_SH_SELECT));
            CHM_TRY(chm_select_fullbit(nq, b.mdocs, b.onebit, b.mcount, kr, p->k_full_bit, p->num_chunks, b.fd, b.nf,
                                       kr, st));
            CHM_TRY(chm_shard_localize(nq, kr, b.fd, b.nf, sh->doc_base[rank], idx->num_docs, b.fb_local, st));
            CHM_TRY(mark(CHM_SH_FULLBIT));
            if (nq >= 16)
                CHM_TRY(chm_fullbit_score_tc(idx, nq, b.rot, b.cbex, b.fb_local, b.nf, kr, b.fs, b.rt_ws, b.rt_bytes,
                                             st));
            else
                CHM_TRY(chm_fullbit_score(idx, nq, b.rot, b.cbex, b.fb_local, b.nf, kr, b.fs, st));
            CHM_TRY(mark(CHM_SH_REDUCE_FULLBIT));
            CHM_TRY(chm::nccl_status(ncclAllReduce(b.fs, b.fs, (size_t)nq * kr, ncclFloat32, ncclMax, comm->nccl, st),
                                     "ncclAllReduce(full-bit)"));
            CHM_TRY(mark(CHM_SH_FINAL));
            CHM_TRY(chm_final_topk(nq, b.fd, b.fs, b.nf, kr, p->k, results + q0 * p->k, num_results + q0, st));
            chm::fold_shard_flags_kernel<<<(nq + 255) / 256, 256, 0, st>>>(b.flags, num_results + q0, nq);
            CHM_TRY(chm::launch_status("fold_shard_flags_kernel"));
            if (timed && last) CHM_CUDA(cudaEventRecord(evs[CHM_SH_STEPS], st));
        }
        return CHM_OK;
    };
    status = run();
    if (timed) {
        if (status == CHM_OK) {
            cudaError_t e = cudaEventSynchronize(evs[CHM_SH_STEPS]);
            for (int i = 0; i < CHM_SH_STEPS && e == cudaSuccess; ++i) e = cudaEventElapsedTime(&timing[i], evs[i], evs[i + 1]);
            if (e != cudaSuccess) {
                chm::set_last_error("sharded timing", e);
                status = CHM_ERR_CUDA;
            }
        }
        for (int i = 0; i <= CHM_SH_STEPS; ++i)
            if (evs[i]) cudaEventDestroy(evs[i]);
    }
    return status;
}
