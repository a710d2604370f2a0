// Query preparation: FhtKac rotation of every query token, QueryState sums
// and the 1-bit lookup table (one warp per query token).
#include <cmath>

#include "common.cuh"
#include "rotate.cuh"

namespace chm {

__global__ void __launch_bounds__(128) prepare_queries_kernel(
    const uint8_t* __restrict__ flips, int dim, int trunc, float fac, float cbex_mul,
    const float* __restrict__ raw, int64_t ntok, float* __restrict__ rot,
    float* __restrict__ cb1, float* __restrict__ cbex, float* __restrict__ lut) {
    __shared__ float s_q[4][kDim];
    __shared__ uint8_t s_flips[64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 64) s_flips[threadIdx.x] = flips[threadIdx.x];
    __syncthreads();
    const int64_t tok = (int64_t)blockIdx.x * 4 + warp;
    if (tok >= ntok) return;
    const float* src = raw + tok * dim;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = 32 * k + lane;
        v[k] = i < dim ? src[i] : 0.0f;
    }
    rotate_warp(v, lane, s_flips, trunc, fac);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        s_q[warp][32 * k + lane] = v[k];
        rot[tok * kDim + 32 * k + lane] = v[k];
    }
    __syncwarp();
    if (lane == 0) {
        // QueryState (chimera_index_internal.cuh:58-64): std::accumulate from 0.0f
        float sumq = 0.0f;
        for (int i = 0; i < kDim; ++i) sumq = fadd(sumq, s_q[warp][i]);
        cb1[tok] = __fdiv_rn(fmul(sumq, 1.0f), 2.0f);
        cbex[tok] = __fdiv_rn(fmul(sumq, cbex_mul), 2.0f);
    }
    if (lut != nullptr) {
        // precompute_one_bit_lut_kernel (kernels.cu:412-427)
        float* out = lut + tok * kLutPerQ;
#pragma unroll 4
        for (int j = 0; j < 16; ++j) {
            const int idx = lane + 32 * j;
            const int chunk = idx >> 4, e = idx & 15;
            float s = 0.0f;
#pragma unroll
            for (int b = 0; b < 4; ++b)
                if ((e >> b) & 1) s = fadd(s, s_q[warp][chunk * 4 + b]);
            out[idx] = s;
        }
    }
}

int floor_log2(int x) {
    int l = 0;
    while ((2 << l) <= x) ++l;
    return l;
}

}  // namespace chm

extern "C" chm_status chm_prepare_queries(const uint8_t* flips, int32_t dim, int32_t ex_bits,
                                          const float* raw, int64_t ntok, float* rot, float* cb1,
                                          float* cbex, float* lut, void* stream) {
    if (dim < 64 || dim > CHM_PADDED_DIM || ex_bits < 1 || ex_bits > 7 || ntok < 0)
        return CHM_ERR_INVALID;
    if (ntok == 0) return CHM_OK;
    const int trunc = 1 << chm::floor_log2(dim);
    const float fac = 1.0F / std::sqrt(static_cast<float>(trunc));
    const float cbex_mul = static_cast<float>((1 << (ex_bits + 1)) - 1);
    const int64_t blocks = (ntok + 3) / 4;
    chm::prepare_queries_kernel<<<(unsigned)blocks, 128, 0, (cudaStream_t)stream>>>(
        flips, dim, trunc, fac, cbex_mul, raw, ntok, rot, cb1, cbex, lut);
    return chm::launch_status("prepare_queries_kernel");
}
