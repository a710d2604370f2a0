// Exact centroid probe and nearest-centroid assignment.
//
// dist(q, c) = ||c||^2 - 2 <q, c>, the dot a sequential fma chain over the
// 128 dims in ascending order (this is the probe's contract; it replaces the
// approximate cuVS CAGRA search of ivf_pg.cpp:37-65).  A register-tiled SIMT
// GEMM gives exactly that chain per output (rank-1 updates in k order).
//
//  probe  : GEMM -> dist matrix [rows x n_clusters] -> one CTA per row does
//           an exact radix select of the nprobe smallest (dist, id) and a
//           bitonic sort, nearest first, ties to the lower id.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "select.cuh"

namespace chm {

constexpr int BM = 64, BN = 128, BK = 16;
constexpr int kGemmThreads = 256;  // 16 x 16 threads, 4 x 8 outputs each

// Loads a BK-wide k-slab of A (rows) and B (cols) into shared memory,
// transposed so the inner loop reads contiguous rows/cols.
// rows_dev (optional): a device count that caps `rows` (row tiles past it
// return at once).
__global__ void __launch_bounds__(kGemmThreads) dist_gemm_kernel(
    const float* __restrict__ A, int64_t rows, const float* __restrict__ B,
    const float* __restrict__ bnorm, int64_t cols, int lda, int kdim, float* __restrict__ dist,
    const uint32_t* __restrict__ rows_dev = nullptr) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t row0 = (int64_t)blockIdx.y * BM;
    if (rows_dev != nullptr) {
        rows = min(rows, (int64_t)*rows_dev);
        if (row0 >= rows) return;
    }
    const int64_t col0 = (int64_t)blockIdx.x * BN;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < kdim; k0 += BK) {
        // A tile: 64 rows x 16 k = 1024 values, 4 per thread
        for (int e = threadIdx.x; e < BM * BK; e += kGemmThreads) {
            const int r = e / BK, kk = e % BK;
            const int64_t gr = row0 + r;
            const int gk = k0 + kk;
            As[kk][r] = (gr < rows && gk < kdim) ? A[gr * lda + gk] : 0.0f;
        }
        for (int e = threadIdx.x; e < BN * BK; e += kGemmThreads) {
            const int c = e / BK, kk = e % BK;
            const int64_t gc = col0 + c;
            const int gk = k0 + kk;
            Bs[kk][c] = (gc < cols && gk < kdim) ? B[gc * lda + gk] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[4], b[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = Bs[kk][tx * 8 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t gr = row0 + ty * 4 + i;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t gc = col0 + tx * 8 + j;
            if (gr < rows && gc < cols) dist[gr * cols + gc] = fsub(bnorm[gc], fmul(2.0f, acc[i][j]));
        }
    }
}

constexpr int kSelThreads = 1024;

__global__ void __launch_bounds__(kSelThreads) row_select_kernel(
    const float* __restrict__ dist, int64_t cols, int k, uint32_t* __restrict__ labels) {
    const int64_t row = blockIdx.x;
    block_select_smallest(dist + row * cols, cols, k, labels + row * k);
}

// Exact top-k of listed rows in batches (the tensor-core probe's and the
// assignment's fallback): the first min(count, max_rows) listed rows are
// gathered, one SIMT GEMM pass computes their exact dists to every centroid
// (each centroid read once for the whole batch), and a CTA per row selects.
__global__ void fallback_gather_kernel(const float* __restrict__ x, const int32_t* __restrict__ list,
                                       const uint32_t* __restrict__ count, int max_rows, float* __restrict__ q) {
    const int i = blockIdx.x;
    const int n = min((int)*count, max_rows);
    const float v = i < n ? x[(int64_t)list[i] * kDim + threadIdx.x] : 0.0f;
    q[(int64_t)i * kDim + threadIdx.x] = v;
}

__global__ void __launch_bounds__(kSelThreads) fallback_select_kernel(const float* __restrict__ dist, int64_t cols,
                                                                      int k, const int32_t* __restrict__ list,
                                                                      const uint32_t* __restrict__ count, int max_rows,
                                                                      uint32_t* __restrict__ labels) {
    const int i = blockIdx.x;
    if (i >= min((int)*count, max_rows)) return;
    block_select_smallest(dist + (int64_t)i * cols, cols, k, labels + (int64_t)list[i] * k);
}

}  // namespace chm

chm_status chm_probe_fallback_batch(const float* x, const int32_t* list, const uint32_t* count, int max_rows,
                                    const float* centroids, const float* cn, int64_t nc, int k, float* q_scratch,
                                    float* dist_scratch, uint32_t* labels, cudaStream_t st) {
    chm::fallback_gather_kernel<<<max_rows, chm::kDim, 0, st>>>(x, list, count, max_rows, q_scratch);
    CHM_TRY(chm::launch_status("fallback_gather_kernel"));
    dim3 g((unsigned)((nc + chm::BN - 1) / chm::BN), (unsigned)((max_rows + chm::BM - 1) / chm::BM));
    chm::dist_gemm_kernel<<<g, chm::kGemmThreads, 0, st>>>(q_scratch, max_rows, centroids, cn, nc, chm::kDim,
                                                           chm::kDim, dist_scratch, count);
    CHM_TRY(chm::launch_status("dist_gemm_kernel"));
    chm::fallback_select_kernel<<<max_rows, chm::kSelThreads, 0, st>>>(dist_scratch, nc, k, list, count, max_rows,
                                                                        labels);
    return chm::launch_status("fallback_select_kernel");
}

namespace chm {

// k-th smallest value per row (the tensor-core probe's filter threshold).
__global__ void __launch_bounds__(kSelThreads) row_kth_kernel(const float* __restrict__ dist, int64_t cols, int k,
                                                              float* __restrict__ kth) {
    __shared__ KthState s;
    const int64_t row = blockIdx.x;
    uint32_t key, need;
    block_kth_key(dist + row * cols, cols, k, s, &key, &need);
    if (threadIdx.x == 0) kth[row] = key_to_float_asc(key);
}

__global__ void row_norms_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* r = x + i * kDim;
    float acc = 0.0f;
    for (int k = 0; k < kDim; ++k) acc = __fmaf_rn(r[k], r[k], acc);
    out[i] = acc;
}

}  // namespace chm

extern "C" size_t chm_probe_workspace_bytes(int64_t nrows, int64_t n_clusters, int32_t nprobe) {
    (void)nprobe;
    chm::Sizer s;
    s.take<float>((size_t)nrows * n_clusters);
    return s.off;
}

extern "C" chm_status chm_probe(const float* rot_queries, int64_t nrows, const float* centroids,
                                const float* centroid_norms, int64_t n_clusters, int32_t nprobe,
                                uint32_t* labels, void* ws, size_t ws_bytes, void* stream) {
    if (nrows <= 0) return CHM_OK;
    if (nprobe <= 0 || nprobe > CHM_MAX_NPROBE || nprobe > n_clusters) return CHM_ERR_INVALID;
    chm::Arena a(ws, ws_bytes);
    float* dist = a.take<float>((size_t)nrows * n_clusters);
    if (a.overflow) return CHM_ERR_CAPACITY;
    cudaStream_t st = (cudaStream_t)stream;
    dim3 g((unsigned)((n_clusters + chm::BN - 1) / chm::BN), (unsigned)((nrows + chm::BM - 1) / chm::BM));
    chm::dist_gemm_kernel<<<g, chm::kGemmThreads, 0, st>>>(rot_queries, nrows, centroids, centroid_norms,
                                                           n_clusters, chm::kDim, chm::kDim, dist);
    CHM_TRY(chm::launch_status("dist_gemm_kernel"));
    chm::row_select_kernel<<<(unsigned)nrows, chm::kSelThreads, 0, st>>>(dist, n_clusters, nprobe, labels);
    return chm::launch_status("row_select_kernel");
}

chm_status chm_row_kth(const float* dist, int64_t rows, int64_t cols, int k, float* kth, uint32_t* labels,
                       void* stream) {
    (void)labels;
    if (rows <= 0) return CHM_OK;
    chm::row_kth_kernel<<<(unsigned)rows, chm::kSelThreads, 0, (cudaStream_t)stream>>>(dist, cols, k, kth);
    return chm::launch_status("row_kth_kernel");
}

extern "C" chm_status chm_row_norms(const float* x, int64_t n, float* out, void* stream) {
    if (n <= 0) return CHM_OK;
    chm::row_norms_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, n, out);
    return chm::launch_status("row_norms_kernel");
}

// x and centroids are [*, 128] rows with the raw dims first and zeros after
// (zero padding leaves every fma chain unchanged).  Rows go through the
// tensor-core top-16 pass with exact re-ranking, in slabs.
size_t chm_tc_assign_workspace_bytes(int64_t rows, int64_t nc);
chm_status chm_tc_assign(const float* x128, int64_t rows, const float* centroids, const __nv_bfloat16* cent_bf16,
                         const float* cn, const float* cnmax, int64_t nc, uint32_t* assign, void* ws,
                         size_t ws_bytes, cudaStream_t st);

namespace chm { constexpr int64_t kAssignSlab = 1 << 20; }

extern "C" size_t chm_build_assign_workspace_bytes(int64_t n, int64_t nc) {
    chm::Sizer s;
    s.take<__nv_bfloat16>((size_t)nc * chm::kDim);
    s.take<float>(4);
    s.take<char>(chm_tc_assign_workspace_bytes(std::min<int64_t>(n, chm::kAssignSlab), nc));
    return s.off;
}

extern "C" chm_status chm_build_assign(const float* x, int64_t n, int32_t dim, const float* centroids,
                                       const float* centroid_norms, int64_t n_clusters,
                                       uint32_t* assign, void* ws, size_t ws_bytes, void* stream) {
    if (n <= 0) return CHM_OK;
    if (dim <= 0 || dim > CHM_PADDED_DIM || n_clusters <= 0) return CHM_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    chm::Arena a(ws, ws_bytes);
    auto* cb = a.take<__nv_bfloat16>((size_t)n_clusters * chm::kDim);
    auto* cnmax = a.take<float>(4);
    const size_t inner = chm_tc_assign_workspace_bytes(std::min<int64_t>(n, chm::kAssignSlab), n_clusters);
    auto* iws = a.take<char>(inner);
    if (a.overflow) return CHM_ERR_CAPACITY;
    CHM_TRY(chm_to_bf16(centroids, n_clusters * chm::kDim, cb, st));
    CHM_TRY(chm_max_value(centroid_norms, n_clusters, cnmax, st));
    for (int64_t r0 = 0; r0 < n; r0 += chm::kAssignSlab) {
        const int64_t rows = std::min<int64_t>(chm::kAssignSlab, n - r0);
        CHM_TRY(chm_tc_assign(x + r0 * chm::kDim, rows, centroids, cb, centroid_norms, cnmax, n_clusters,
                              assign + r0, iws, inner, st));
    }
    return CHM_OK;
}

// ---- probe without allocation ---------------------------------------------
// chm_probe_noalloc runs the same two kernels as chm_probe, with the distance
// matrix in a file-scope device array instead of a caller workspace.  The
// array is fully written by dist_gemm_kernel before row_select_kernel reads
// it, so nothing in it has to start at zero.  One array per device: calls
// that overlap on one device (two streams, two host threads) race on it.
#include <atomic>
#include <cstdio>
#include <mutex>

namespace chm {

void set_last_message(const char* msg);

constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) float g_noalloc_probe_dist[CHM_PROBE_NOALLOC_MAX_ELEMENTS];
static std::atomic<float*> g_noalloc_probe_ptr[kNoAllocMaxDevices];
static std::mutex g_noalloc_probe_mu;

// Device address of the static scratch for the current device, looked up once
// per device with that device current (the first call on the device), then
// cached.  cudaDeviceReset unloads the module, which leaves the cached
// address stale.
static chm_status noalloc_probe_scratch(float** out) {
    int dev = 0;
    CHM_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        set_last_message("chm_probe_noalloc: device ordinal beyond 63");
        return CHM_ERR_UNSUPPORTED;
    }
    float* p = g_noalloc_probe_ptr[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_noalloc_probe_mu);
        p = g_noalloc_probe_ptr[dev].load(std::memory_order_acquire);
        if (!p) {
            void* addr = nullptr;
            CHM_CUDA(cudaGetSymbolAddress(&addr, g_noalloc_probe_dist));
            p = static_cast<float*>(addr);
            g_noalloc_probe_ptr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return CHM_OK;
}

}  // namespace chm

extern "C" chm_status chm_probe_noalloc(const float* rot_queries, int64_t nrows, const float* centroids,
                                        const float* centroid_norms, int64_t n_clusters, int32_t nprobe,
                                        uint32_t* labels, void* stream) {
    if (nrows <= 0) return CHM_OK;
    if (nprobe <= 0 || nprobe > CHM_MAX_NPROBE || nprobe > n_clusters) return CHM_ERR_INVALID;
    if (nrows > (int64_t)CHM_PROBE_NOALLOC_MAX_ELEMENTS / n_clusters) {
        char msg[200];
        std::snprintf(msg, sizeof(msg),
                      "chm_probe_noalloc: nrows * n_clusters = %lld * %lld exceeds the static scratch of %lld "
                      "floats",
                      (long long)nrows, (long long)n_clusters, (long long)CHM_PROBE_NOALLOC_MAX_ELEMENTS);
        chm::set_last_message(msg);
        return CHM_ERR_CAPACITY;
    }
    float* dist = nullptr;
    CHM_TRY(chm::noalloc_probe_scratch(&dist));
    cudaStream_t st = (cudaStream_t)stream;
    dim3 g((unsigned)((n_clusters + chm::BN - 1) / chm::BN), (unsigned)((nrows + chm::BM - 1) / chm::BM));
    chm::dist_gemm_kernel<<<g, chm::kGemmThreads, 0, st>>>(rot_queries, nrows, centroids, centroid_norms,
                                                           n_clusters, chm::kDim, chm::kDim, dist);
    CHM_TRY(chm::launch_status("dist_gemm_kernel"));
    chm::row_select_kernel<<<(unsigned)nrows, chm::kSelThreads, 0, st>>>(dist, n_clusters, nprobe, labels);
    return chm::launch_status("row_select_kernel");
}
