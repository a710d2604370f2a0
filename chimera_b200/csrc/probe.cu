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
//  assign : GEMM with a fused arg-min (packed (key, id) 64-bit atomicMin).
#include <algorithm>

#include "common.cuh"

namespace chm {

constexpr int BM = 64, BN = 128, BK = 16;
constexpr int kGemmThreads = 256;  // 16 x 16 threads, 4 x 8 outputs each

// Loads a BK-wide k-slab of A (rows) and B (cols) into shared memory,
// transposed so the inner loop reads contiguous rows/cols.
template <bool kArgmin>
__global__ void __launch_bounds__(kGemmThreads) dist_gemm_kernel(
    const float* __restrict__ A, int64_t rows, const float* __restrict__ B,
    const float* __restrict__ bnorm, int64_t cols, int lda, int kdim, float* __restrict__ dist,
    unsigned long long* __restrict__ best) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t row0 = (int64_t)blockIdx.y * BM;
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
        unsigned long long mn = ~0ull;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t gc = col0 + tx * 8 + j;
            if (gr < rows && gc < cols) {
                const float d = fsub(bnorm[gc], fmul(2.0f, acc[i][j]));
                if (kArgmin) {
                    const unsigned long long key = ((unsigned long long)float_key_asc(d) << 32) | (uint32_t)gc;
                    mn = key < mn ? key : mn;
                } else {
                    dist[gr * cols + gc] = d;
                }
            }
        }
        if (kArgmin) {
            // the 16 threads sharing a row are 16 consecutive lanes
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, mn, off, 16);
                mn = o < mn ? o : mn;
            }
            if (tx == 0 && gr < rows) atomicMin(best + gr, mn);
        }
    }
}

constexpr int kSelThreads = 1024;

__device__ uint32_t scan_excl(uint32_t v, uint32_t* s_warp, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = s_warp[lane];
        uint32_t z = w;
#pragma unroll
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

// Exact k smallest (dist, id) per row; 8-bit digits over the ordered key,
// then an id-ordered collection (ties keep the lowest ids) and a sort.
__global__ void __launch_bounds__(kSelThreads) row_select_kernel(
    const float* __restrict__ dist, int64_t cols, int k, uint32_t* __restrict__ labels) {
    __shared__ uint32_t s_hist[256];
    __shared__ uint32_t s_warp[33];
    __shared__ uint32_t s_prefix, s_need;
    __shared__ uint64_t s_out[CHM_MAX_NPROBE];
    __shared__ uint32_t s_nl, s_ne;
    const int64_t row = blockIdx.x;
    const float* d = dist + row * cols;
    if (threadIdx.x == 0) { s_prefix = 0; s_need = (uint32_t)k; s_nl = 0; s_ne = 0; }
    uint32_t pmask = 0;
    for (int sh = 24; sh >= 0; sh -= 8) {
        if (threadIdx.x < 256) s_hist[threadIdx.x] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
            const uint32_t key = float_key_asc(d[i]);
            if ((key & pmask) == prefix) atomicAdd(&s_hist[(key >> sh) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // smallest digit whose cumulative count reaches need (lane owns 8 digits)
            uint32_t c = 0;
            for (int j = 0; j < 8; ++j) c += s_hist[threadIdx.x * 8 + j];
            uint32_t x = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
                if ((int)threadIdx.x >= off) x += y;
            }
            const uint32_t before = x - c;
            const uint32_t need = s_need;
            if (before < need && need <= before + c) {
                uint32_t cum = before;
                for (int j = 0; j < 8; ++j) {
                    const uint32_t h = s_hist[threadIdx.x * 8 + j];
                    if (cum + h >= need) {
                        s_prefix = prefix | ((uint32_t)(threadIdx.x * 8 + j) << sh);
                        s_need = need - cum;
                        break;
                    }
                    cum += h;
                }
            }
        }
        pmask |= 255u << sh;
        __syncthreads();
    }
    const uint32_t kth = s_prefix;
    const uint32_t need_eq = s_need;   // equal keys to take, lowest ids first
    // id-ordered pass: every key < kth, and the first need_eq keys == kth
    for (int64_t base = 0; base < cols; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        uint32_t key = 0xFFFFFFFFu;
        if (i < cols) key = float_key_asc(d[i]);
        const uint32_t lt = (i < cols) && key < kth;
        const uint32_t eq = (i < cols) && key == kth;
        uint32_t tl, te;
        const uint32_t rl = scan_excl(lt, s_warp, &tl);
        const uint32_t re = scan_excl(eq, s_warp, &te);
        const uint32_t nl = s_nl, ne = s_ne;
        if (lt) s_out[nl + rl] = ((uint64_t)key << 32) | (uint32_t)i;
        if (eq && ne + re < need_eq) s_out[(uint32_t)k - need_eq + ne + re] = ((uint64_t)key << 32) | (uint32_t)i;
        __syncthreads();
        if (threadIdx.x == 0) { s_nl = nl + tl; s_ne = ne + te; }
        __syncthreads();
    }
    int n = 1;
    while (n < k) n <<= 1;
    for (int i = k + threadIdx.x; i < n; i += blockDim.x) s_out[i] = ~0ull;
    __syncthreads();
    // ascending bitonic sort
    for (int kk = 2; kk <= n; kk <<= 1) {
        for (int j = kk >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const uint64_t x = s_out[i], y = s_out[l];
                    const bool asc = (i & kk) == 0;
                    if (asc ? (x > y) : (x < y)) { s_out[i] = y; s_out[l] = x; }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < k; i += blockDim.x) labels[row * k + i] = (uint32_t)s_out[i];
}

__global__ void row_norms_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* r = x + i * kDim;
    float acc = 0.0f;
    for (int k = 0; k < kDim; ++k) acc = __fmaf_rn(r[k], r[k], acc);
    out[i] = acc;
}

__global__ void unpack_argmin_kernel(const unsigned long long* __restrict__ best, int64_t n,
                                     uint32_t* __restrict__ assign) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) assign[i] = (uint32_t)best[i];
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
    chm::dist_gemm_kernel<false><<<g, chm::kGemmThreads, 0, st>>>(
        rot_queries, nrows, centroids, centroid_norms, n_clusters, chm::kDim, chm::kDim, dist, nullptr);
    CHM_TRY(chm::launch_status("dist_gemm_kernel"));
    chm::row_select_kernel<<<(unsigned)nrows, chm::kSelThreads, 0, st>>>(dist, n_clusters, nprobe, labels);
    return chm::launch_status("row_select_kernel");
}

extern "C" chm_status chm_row_norms(const float* x, int64_t n, float* out, void* stream) {
    if (n <= 0) return CHM_OK;
    chm::row_norms_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, n, out);
    return chm::launch_status("row_norms_kernel");
}

// x and centroids are [*, 128] rows with the raw dims first and zeros after
// (zero padding leaves every fma chain unchanged).
namespace chm { constexpr int64_t kAssignSlab = 1 << 20; }

extern "C" size_t chm_build_assign_workspace_bytes(int64_t n) {
    chm::Sizer s;
    s.take<unsigned long long>((size_t)std::min<int64_t>(n, chm::kAssignSlab));
    return s.off;
}

extern "C" chm_status chm_build_assign(const float* x, int64_t n, int32_t dim, const float* centroids,
                                       const float* centroid_norms, int64_t n_clusters,
                                       uint32_t* assign, void* ws, size_t ws_bytes, void* stream) {
    if (n <= 0) return CHM_OK;
    if (dim <= 0 || dim > CHM_PADDED_DIM || n_clusters <= 0) return CHM_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    chm::Arena a(ws, ws_bytes);
    unsigned long long* best = a.take<unsigned long long>((size_t)std::min<int64_t>(n, chm::kAssignSlab));
    if (a.overflow) return CHM_ERR_CAPACITY;
    for (int64_t r0 = 0; r0 < n; r0 += chm::kAssignSlab) {
        const int64_t rows = std::min<int64_t>(chm::kAssignSlab, n - r0);
        CHM_CUDA(cudaMemsetAsync(best, 0xFF, sizeof(unsigned long long) * rows, st));
        dim3 g((unsigned)((n_clusters + chm::BN - 1) / chm::BN), (unsigned)((rows + chm::BM - 1) / chm::BM));
        chm::dist_gemm_kernel<true><<<g, chm::kGemmThreads, 0, st>>>(
            x + r0 * chm::kDim, rows, centroids, centroid_norms, n_clusters, chm::kDim, chm::kDim, nullptr, best);
        CHM_TRY(chm::launch_status("dist_gemm_kernel<argmin>"));
        chm::unpack_argmin_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(best, rows, assign + r0);
        CHM_TRY(chm::launch_status("unpack_argmin_kernel"));
    }
    return CHM_OK;
}
