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
