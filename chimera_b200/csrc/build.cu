// Index build on the GPU: FhtKac rotation + RaBitQ encoding of every token
// embedding, one warp per vector (replaces the OpenMP loop of
// encode_embeddings, build_index.cu:258-303, and quantization.cpp:47-193).
//
// The encoder's floating-point steps follow the reference build exactly:
// Eigen packet reductions for the dots and the norm (see rotate.cuh), and
// best_rescale_factor's event sweep in double precision, where the pop order
// of the reference's min-priority-queue of (t, dim) events is reproduced by a
// warp arg-min over the pending event of every dimension.
#include <cmath>

#include "codes.cuh"
#include "common.cuh"
#include "rotate.cuh"

namespace chm {

__constant__ float kTightStart[9] = {0.f, 0.15f, 0.20f, 0.52f, 0.59f, 0.71f, 0.75f, 0.77f, 0.81f};

__device__ __forceinline__ void warp_argmin(double& t, int& id) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const double ot = __shfl_xor_sync(0xffffffffu, t, off);
        const int oid = __shfl_xor_sync(0xffffffffu, id, off);
        if (ot < t || (ot == t && oid < id)) { t = ot; id = oid; }
    }
}

// best_rescale_factor (quantization.cpp:62-119) for the vector whose |o|/||o||
// values lane l holds at slots k (dim 32k + l).
__device__ double best_rescale_warp(const float (&oa)[4], int lane, int ex_bits, float* s_oa) {
    const double kEps = 1e-5;
    float mx = fmaxf(fmaxf(oa[0], oa[1]), fmaxf(oa[2], oa[3]));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const double max_o = (double)mx;
    const int top = (1 << ex_bits) - 1;
    const double t_end = __ddiv_rn((double)(top + 10), max_o);
    const double t_start = __dmul_rn(t_end, (double)kTightStart[ex_bits]);
    int cur[4];
    long long den_part = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        cur[k] = (int)__fma_rn(t_start, (double)oa[k], kEps);
        den_part += (long long)cur[k] * cur[k] + cur[k];
        s_oa[32 * k + lane] = oa[k];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) den_part += __shfl_xor_sync(0xffffffffu, den_part, off);
    // integer-valued, so exact in any order
    double sqr_den = 128.0 * 0.25 + (double)den_part;
    // numerator: sequential over dims 0..127 (order matters)
    double num = 0.0;
    for (int i = 0; i < kDim; ++i) {
        const int c = __shfl_sync(0xffffffffu, cur[i >> 5], i & 31);
        num = __fma_rn((double)c + 0.5, (double)s_oa[i], num);
    }
    double next[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        next[k] = oa[k] > 0.0f ? __ddiv_rn((double)(cur[k] + 1), (double)oa[k]) : INFINITY;
    double max_ip = 0.0, t = 0.0;
    for (;;) {
        double bt = next[0];
        int bid = lane;
#pragma unroll
        for (int k = 1; k < 4; ++k)
            if (next[k] < bt) { bt = next[k]; bid = 32 * k + lane; }
        warp_argmin(bt, bid);
        if (bt == INFINITY) break;
        const int k = bid >> 5;
        int upd = 0;
        if (lane == (bid & 31)) {
            // owner advances its dimension and schedules the next event
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                if (kk == k) {
                    upd = ++cur[kk];
                    double tn = INFINITY;
                    if (upd < top) {
                        const double cand = __ddiv_rn((double)(upd + 1), (double)oa[kk]);
                        if (cand < t_end) tn = cand;
                    }
                    next[kk] = tn;
                }
            }
        }
        upd = __shfl_sync(0xffffffffu, upd, bid & 31);
        sqr_den = __dadd_rn(sqr_den, (double)(2 * upd));
        num = __dadd_rn(num, (double)s_oa[bid]);
        const double ip = __ddiv_rn(num, __dsqrt_rn(sqr_den));
        if (ip > max_ip) { max_ip = ip; t = bt; }
    }
    return t;
}

__global__ void __launch_bounds__(128) encode_kernel(
    const uint8_t* __restrict__ flips, const float* __restrict__ x, int64_t n, int dim, int trunc,
    float fac, int ex_bits, uint8_t* __restrict__ codes1, float* __restrict__ f1,
    uint8_t* __restrict__ full, float* __restrict__ ff, float* __restrict__ rot_out) {
    __shared__ uint8_t s_flips[64];
    __shared__ float s_oa[4][kDim];
    __shared__ uint8_t s_raw[4][kDim];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 64) s_flips[threadIdx.x] = flips[threadIdx.x];
    __syncthreads();
    const int64_t row = (int64_t)blockIdx.x * 4 + warp;
    if (row >= n) return;
    float v[4];
    const float* src = x + row * dim;
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = (32 * k + lane < dim) ? src[32 * k + lane] : 0.0f;
    rotate_warp(v, lane, s_flips, trunc, fac);
    if (rot_out) {
#pragma unroll
        for (int k = 0; k < 4; ++k) rot_out[row * kDim + 32 * k + lane] = v[k];
    }
    // encode_one_bit (quantization.cpp:47-60)
    float xu[4];
    uint32_t words[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool bit = v[k] > 0.0f;
        words[k] = __ballot_sync(0xffffffffu, bit);
        xu[k] = fadd(bit ? 1.0f : 0.0f, -0.5f);
    }
    const float ip1 = eigen_dot_warp(xu, v);
    if (lane < 4) reinterpret_cast<uint32_t*>(codes1 + row * 16)[lane] = words[lane];
    if (lane == 0) f1[row] = __fdiv_rn(1.0f, ip1);
    // quantize_ex (quantization.cpp:121-146): |o / ||o|| |
    const float nrm = __fsqrt_rn(eigen_dot_warp(v, v));
    float oa[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) oa[k] = fabsf(__fdiv_rn(v[k], nrm));
    const double t = best_rescale_warp(oa, lane, ex_bits, s_oa[warp]);
    const int top = (1 << ex_bits) - 1;
    const float cb = -((float)(1 << ex_bits) - 0.5f);
    float xf[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int c = (int)__fma_rn(t, (double)oa[k], 1e-5);
        if (c >= (1 << ex_bits)) c = top;
        if (v[k] < 0.0f) c = (~c) & top;
        const int tot = c + ((v[k] >= 0.0f ? 1 : 0) << ex_bits);
        s_raw[warp][32 * k + lane] = (uint8_t)tot;
        xf[k] = fadd((float)tot, cb);
    }
    const float ipf = eigen_dot_warp(xf, v);
    if (lane == 0) ff[row] = __fdiv_rn(1.0f, ipf);
    __syncwarp();
    const int w = 1 + ex_bits;
    const int bytes = kDim * w / 8;
    uint8_t* dst = full + row * bytes;
    for (int b = lane; b < bytes; b += 32) dst[b] = packed_byte(s_raw[warp], b, w);
}

}  // namespace chm

extern "C" chm_status chm_build_encode(const uint8_t* flips, const float* x, int64_t n, int32_t dim,
                                       int32_t ex_bits, uint8_t* codes1, float* f1, uint8_t* full,
                                       float* ff, float* rot, void* stream) {
    if (n <= 0) return CHM_OK;
    if (dim < 64 || dim > CHM_PADDED_DIM || ex_bits < 1 || ex_bits > 7) return CHM_ERR_INVALID;
    int l = 0;
    while ((2 << l) <= dim) ++l;
    const int trunc = 1 << l;
    const float fac = 1.0F / std::sqrt(static_cast<float>(trunc));
    const int64_t blocks = (n + 3) / 4;
    chm::encode_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(
        flips, x, n, dim, trunc, fac, ex_bits, codes1, f1, full, ff, rot);
    return chm::launch_status("encode_kernel");
}

namespace chm {

// Token-order copy of the cluster-ordered 1-bit arrays: four lanes per token,
// each moving one 4-byte word of the code, so a warp reads eight 16-byte codes
// and writes 128 contiguous bytes.
__global__ void __launch_bounds__(256) token_order_1bit_kernel(const uint32_t* __restrict__ codes1,
                                                               const float* __restrict__ factor1,
                                                               const uint32_t* __restrict__ tok2pos, int64_t n,
                                                               uint32_t* __restrict__ codes_tok,
                                                               float* __restrict__ factor_tok) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t tok = i >> 2;
    const int w = (int)(i & 3);
    if (tok >= n) return;
    const uint32_t pos = __ldg(tok2pos + tok);
    codes_tok[tok * 4 + w] = __ldg(codes1 + (size_t)pos * 4 + w);
    if (w == 0) factor_tok[tok] = __ldg(factor1 + pos);
}

}  // namespace chm

extern "C" chm_status chm_token_order_1bit(const uint8_t* codes1, const float* factor1, const uint32_t* tok2pos,
                                           int64_t n, uint8_t* codes_tok, float* factor_tok, void* stream) {
    if (n < 0 || (n > 0 && (!codes1 || !factor1 || !tok2pos || !codes_tok || !factor_tok))) return CHM_ERR_INVALID;
    if (n == 0) return CHM_OK;
    const int64_t threads = n * 4;
    chm::token_order_1bit_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint32_t*>(codes1), factor1, tok2pos, n, reinterpret_cast<uint32_t*>(codes_tok),
        factor_tok);
    return chm::launch_status("token_order_1bit_kernel");
}

namespace chm {

// tok_cluster[t]: the last cluster c with cluster_pos[c] <= tok2pos[t]
// (empty lists share their start with the next list, so the last such c is
// the one whose list holds the position).
__global__ void __launch_bounds__(256) token_clusters_kernel(const int64_t* __restrict__ cluster_pos,
                                                             int64_t n_clusters, const uint32_t* __restrict__ tok2pos,
                                                             int64_t n, uint32_t* __restrict__ tok_cluster) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    const int64_t pos = __ldg(tok2pos + t);
    int64_t lo = 0, hi = n_clusters;  // invariant: cluster_pos[lo] <= pos < cluster_pos[hi]
    while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (__ldg(cluster_pos + mid) <= pos) lo = mid; else hi = mid;
    }
    tok_cluster[t] = (uint32_t)lo;
}

}  // namespace chm

extern "C" chm_status chm_token_clusters(const int64_t* cluster_pos, int64_t n_clusters, const uint32_t* tok2pos,
                                         int64_t n, uint32_t* tok_cluster, void* stream) {
    if (n < 0 || n_clusters <= 0 || n_clusters > 0xFFFFFFFFll) return CHM_ERR_INVALID;
    if (n == 0) return CHM_OK;
    chm::token_clusters_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        cluster_pos, n_clusters, tok2pos, n, tok_cluster);
    return chm::launch_status("token_clusters_kernel");
}

// ---- IVF lists and the cluster-ordered 1-bit arrays ----------------------
// IVF_PG::build_from_assignments (ivf_pg.cpp:110-126): a stable counting sort
// of the tokens by cluster, and reorder_by_cluster (build_index.cu:328-363):
// the 1-bit codes, factors and owning docs in that order plus each token's
// position.  On the GPU: per-cluster counts -> an exclusive scan -> a scatter
// by atomic slot -> a sort of each list's token ids (restores the stable,
// ascending order) -> a gather.
namespace chm {

constexpr int kScanPer = 4;                       // elements per thread
constexpr int kScanBlock = 1024 * kScanPer;       // elements per scan block
constexpr int kListSmall = 4096;                  // lists sorted by a 256-thread CTA
constexpr int kListBig = 32768;                   // lists sorted by a 1024-thread CTA (128 KB; a power of
                                                  // two: the bitonic sort pads to one)

__global__ void cluster_count_kernel(const uint32_t* __restrict__ assign, int64_t n, int64_t nc,
                                     uint32_t* __restrict__ counts, uint32_t* __restrict__ bad) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t c = assign[t];
        if ((int64_t)c < nc) atomicAdd(counts + c, 1u);
        else atomicOr(bad, 1u);
    }
}

// Exclusive scan of a 1024-thread block's values, one per thread.
__device__ uint64_t scan_block_excl(uint64_t v, uint64_t* s_warp, uint64_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint64_t y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const uint64_t w = s_warp[lane];
        uint64_t z = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, z, off);
            if (lane >= off) z += y;
        }
        s_warp[lane] = z - w;
        if (lane == 31) s_warp[32] = z;
    }
    __syncthreads();
    const uint64_t r = s_warp[warp] + x - v;
    *total = s_warp[32];
    __syncthreads();
    return r;
}

// Pass 1: each block's exclusive prefix of its kScanBlock counts, and the block's sum.
__global__ void __launch_bounds__(1024) scan_blocks_kernel(const uint32_t* __restrict__ counts, int64_t nc,
                                                           int64_t* __restrict__ pos, uint64_t* __restrict__ sums) {
    __shared__ uint64_t s_warp[33];
    const int64_t base = (int64_t)blockIdx.x * kScanBlock + (int64_t)threadIdx.x * kScanPer;
    uint64_t v[kScanPer], run = 0;
#pragma unroll
    for (int j = 0; j < kScanPer; ++j) {
        v[j] = base + j < nc ? counts[base + j] : 0;
        run += v[j];
    }
    uint64_t total;
    uint64_t off = scan_block_excl(run, s_warp, &total);
#pragma unroll
    for (int j = 0; j < kScanPer; ++j) {
        if (base + j < nc) pos[base + j] = (int64_t)off;
        off += v[j];
    }
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Pass 2 (one block): the blocks' exclusive offsets (at most kScanBlock blocks).
__global__ void __launch_bounds__(1024) scan_sums_kernel(uint64_t* __restrict__ sums, int nblocks,
                                                         int64_t* __restrict__ pos_end) {
    __shared__ uint64_t s_warp[33];
    const int base = threadIdx.x * kScanPer;
    uint64_t v[kScanPer], run = 0;
#pragma unroll
    for (int j = 0; j < kScanPer; ++j) {
        v[j] = base + j < nblocks ? sums[base + j] : 0;
        run += v[j];
    }
    uint64_t total;
    uint64_t off = scan_block_excl(run, s_warp, &total);
#pragma unroll
    for (int j = 0; j < kScanPer; ++j) {
        if (base + j < nblocks) sums[base + j] = off;
        off += v[j];
    }
    if (threadIdx.x == 0) *pos_end = (int64_t)total;
}

// Pass 3: add each block's offset.
__global__ void __launch_bounds__(1024) scan_add_kernel(int64_t* __restrict__ pos, int64_t nc,
                                                        const uint64_t* __restrict__ sums) {
    const int64_t base = (int64_t)blockIdx.x * kScanBlock + (int64_t)threadIdx.x * kScanPer;
    const int64_t add = (int64_t)sums[blockIdx.x];
#pragma unroll
    for (int j = 0; j < kScanPer; ++j)
        if (base + j < nc) pos[base + j] += add;
}

__global__ void cluster_scatter_kernel(const uint32_t* __restrict__ assign, int64_t n, int64_t nc,
                                       const int64_t* __restrict__ cluster_pos, uint32_t* __restrict__ fill,
                                       uint32_t* __restrict__ inv) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t c = assign[t];
        if ((int64_t)c >= nc) continue;  // counted as bad; its token gets no position
        const uint32_t slot = atomicAdd(fill + c, 1u);
        inv[cluster_pos[c] + slot] = (uint32_t)t;
    }
}

// Ascending bitonic sort of n (power of two) keys in shared memory.
__device__ void sort_asc_u32(uint32_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const uint32_t x = a[i], y = a[l];
                    const bool asc = (i & k) == 0;
                    if (asc ? (x > y) : (x < y)) {
                        a[i] = y;
                        a[l] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Sorts list c's token ids in place (cap: shared-memory keys).
__device__ void sort_list(uint32_t* __restrict__ inv, int64_t start, int len, uint32_t* s) {
    int n = 1;
    while (n < len) n <<= 1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s[i] = i < len ? inv[start + i] : 0xFFFFFFFFu;
    __syncthreads();
    sort_asc_u32(s, n);
    for (int i = threadIdx.x; i < len; i += blockDim.x) inv[start + i] = s[i];
    __syncthreads();
}

// CTAs stride over the clusters; lists longer than kListSmall are queued for
// the big-list kernel.
__global__ void __launch_bounds__(256) cluster_sort_small_kernel(uint32_t* __restrict__ inv,
                                                                 const int64_t* __restrict__ cluster_pos, int64_t nc,
                                                                 uint32_t* __restrict__ big,
                                                                 uint32_t* __restrict__ n_big) {
    __shared__ uint32_t s[kListSmall];
    for (int64_t c = blockIdx.x; c < nc; c += gridDim.x) {
        const int64_t start = cluster_pos[c];
        const int64_t len = cluster_pos[c + 1] - start;
        if (len <= 1) continue;
        if (len > kListSmall) {
            if (threadIdx.x == 0) big[atomicAdd(n_big, 1u)] = (uint32_t)c;
            continue;
        }
        sort_list(inv, start, (int)len, s);
    }
}

__global__ void __launch_bounds__(1024) cluster_sort_big_kernel(uint32_t* __restrict__ inv,
                                                                const int64_t* __restrict__ cluster_pos,
                                                                const uint32_t* __restrict__ big,
                                                                const uint32_t* __restrict__ n_big,
                                                                uint32_t* __restrict__ bad) {
    extern __shared__ uint32_t s_big[];
    const uint32_t nb = *n_big;
    for (uint32_t i = blockIdx.x; i < nb; i += gridDim.x) {
        const uint32_t c = big[i];
        const int64_t start = cluster_pos[c];
        const int64_t len = cluster_pos[c + 1] - start;
        if (len > kListBig) {
            if (threadIdx.x == 0) atomicOr(bad, 2u);
            continue;
        }
        sort_list(inv, start, (int)len, s_big);
    }
}

// Each document's id over its tokens.
__global__ void token_docs_kernel(const int64_t* __restrict__ doc_ptrs, int64_t num_docs, int32_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    for (int64_t d = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; d < num_docs;
         d += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        for (int64_t t = doc_ptrs[d] + lane; t < doc_ptrs[d + 1]; t += 32) out[t] = (int32_t)d;
    }
}

// position -> token: the token's position, and the cluster-ordered code,
// factor and owning doc.  Only the positions the lists hold (*pos_end, n
// unless an assignment was out of range) are read.
__global__ void cluster_gather_kernel(const uint32_t* __restrict__ inv, int64_t n, const int64_t* __restrict__ pos_end,
                                      const uint4* __restrict__ codes_tok, const float* __restrict__ f_tok,
                                      const int32_t* __restrict__ tok_doc, uint4* __restrict__ codes1,
                                      float* __restrict__ factor1, int32_t* __restrict__ doc_ids,
                                      uint32_t* __restrict__ tok2pos) {
    const int64_t m = min(n, *pos_end);
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < m; p += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t t = inv[p];
        if ((int64_t)t >= n) continue;
        tok2pos[t] = (uint32_t)p;
        codes1[p] = codes_tok[t];
        factor1[p] = f_tok[t];
        doc_ids[p] = tok_doc[t];
    }
}

struct OrderWork {
    uint32_t* counts;  // [nc]
    uint32_t* fill;    // [nc]
    uint64_t* sums;    // [kScanBlock]
    uint32_t* big;     // [nc]
    uint32_t* n_big;
    uint32_t* bad;
    int32_t* tok_doc;  // [n]
};

template <typename A>
void order_layout(A& a, int64_t n, int64_t nc, OrderWork* w) {
    auto counts = a.template take<uint32_t>((size_t)nc);
    auto fill = a.template take<uint32_t>((size_t)nc);
    auto sums = a.template take<uint64_t>((size_t)kScanBlock);
    auto big = a.template take<uint32_t>((size_t)nc);
    auto n_big = a.template take<uint32_t>(2);
    auto tok_doc = a.template take<int32_t>((size_t)n);
    if (w)
        *w = OrderWork{(uint32_t*)counts, (uint32_t*)fill, (uint64_t*)sums, (uint32_t*)big, (uint32_t*)n_big,
                       (uint32_t*)n_big + 1, (int32_t*)tok_doc};
}

struct OrderSizer {
    Sizer s;
    template <typename T>
    void* take(size_t n) {
        s.take<T>(n);
        return nullptr;
    }
};

}  // namespace chm

extern "C" size_t chm_build_cluster_order_workspace_bytes(int64_t n, int64_t n_clusters) {
    if (n <= 0 || n_clusters <= 0) return 0;
    chm::OrderSizer s;
    chm::order_layout(s, n, n_clusters, nullptr);
    return s.s.off;
}

extern "C" chm_status chm_build_cluster_order(const uint32_t* assign, int64_t n, int64_t n_clusters,
                                              const int64_t* doc_ptrs, int64_t num_docs, const uint8_t* codes_tok,
                                              const float* factor_tok, int64_t* cluster_pos, uint32_t* inv,
                                              uint8_t* codes1, float* factor1, int32_t* doc_ids, uint32_t* tok2pos,
                                              uint32_t* status, void* ws, size_t ws_bytes, void* stream) {
    if (n <= 0 || n > 0xFFFFFFFFll || n_clusters <= 0 || num_docs <= 0 ||
        n_clusters > (int64_t)chm::kScanBlock * chm::kScanBlock)
        return CHM_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    chm::Arena a(ws, ws_bytes);
    chm::OrderWork w;
    chm::order_layout(a, n, n_clusters, &w);
    if (a.overflow) return CHM_ERR_CAPACITY;
    CHM_CUDA(cudaMemsetAsync(w.counts, 0, sizeof(uint32_t) * n_clusters, st));
    CHM_CUDA(cudaMemsetAsync(w.fill, 0, sizeof(uint32_t) * n_clusters, st));
    CHM_CUDA(cudaMemsetAsync(w.n_big, 0, sizeof(uint32_t) * 2, st));
    const int grid = 148 * 16;
    chm::cluster_count_kernel<<<grid, 256, 0, st>>>(assign, n, n_clusters, w.counts, w.bad);
    CHM_TRY(chm::launch_status("cluster_count_kernel"));
    const int nblocks = (int)((n_clusters + chm::kScanBlock - 1) / chm::kScanBlock);
    chm::scan_blocks_kernel<<<nblocks, 1024, 0, st>>>(w.counts, n_clusters, cluster_pos, w.sums);
    CHM_TRY(chm::launch_status("scan_blocks_kernel"));
    chm::scan_sums_kernel<<<1, 1024, 0, st>>>(w.sums, nblocks, cluster_pos + n_clusters);
    CHM_TRY(chm::launch_status("scan_sums_kernel"));
    chm::scan_add_kernel<<<nblocks, 1024, 0, st>>>(cluster_pos, n_clusters, w.sums);
    CHM_TRY(chm::launch_status("scan_add_kernel"));
    chm::cluster_scatter_kernel<<<grid, 256, 0, st>>>(assign, n, n_clusters, cluster_pos, w.fill, inv);
    CHM_TRY(chm::launch_status("cluster_scatter_kernel"));
    chm::cluster_sort_small_kernel<<<(unsigned)std::min<int64_t>(n_clusters, 148 * 8), 256, 0, st>>>(
        inv, cluster_pos, n_clusters, w.big, w.n_big);
    CHM_TRY(chm::launch_status("cluster_sort_small_kernel"));
    const size_t big_smem = sizeof(uint32_t) * chm::kListBig;
    CHM_CUDA(cudaFuncSetAttribute(chm::cluster_sort_big_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)big_smem));
    chm::cluster_sort_big_kernel<<<148, 1024, big_smem, st>>>(inv, cluster_pos, w.big, w.n_big, w.bad);
    CHM_TRY(chm::launch_status("cluster_sort_big_kernel"));
    chm::token_docs_kernel<<<grid, 256, 0, st>>>(doc_ptrs, num_docs, w.tok_doc);
    CHM_TRY(chm::launch_status("token_docs_kernel"));
    chm::cluster_gather_kernel<<<grid, 256, 0, st>>>(inv, n, cluster_pos + n_clusters,
                                                     reinterpret_cast<const uint4*>(codes_tok), factor_tok,
                                                     w.tok_doc, reinterpret_cast<uint4*>(codes1), factor1, doc_ids,
                                                     tok2pos);
    CHM_TRY(chm::launch_status("cluster_gather_kernel"));
    if (status) CHM_CUDA(cudaMemcpyAsync(status, w.bad, sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
    return CHM_OK;
}
