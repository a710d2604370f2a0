// Block-wide exact selection over a row of fp32 distances (blockDim 1024):
// radix select on the order-preserving 32-bit key, then an id-ordered pass
// so ties keep the lowest ids, then a bitonic sort of (key, id).
#pragma once
#include "common.cuh"

namespace chm {

__device__ inline uint32_t blk_scan_excl(uint32_t v, uint32_t* s_warp, uint32_t* total) {
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
        const uint32_t w = (lane < (int)(blockDim.x >> 5)) ? s_warp[lane] : 0;
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

struct KthState {
    uint32_t hist[256];
    uint32_t warp[33];
    uint32_t prefix, need;
};

// The k-th smallest of the 32-bit keys key_at(0..cols) and how many keys
// equal to it are needed to complete the k smallest (blockDim >= 256).
template <typename KeyAt>
__device__ inline void block_kth_key_of(KeyAt key_at, int64_t cols, int k, KthState& s, uint32_t* kth,
                                        uint32_t* need_eq) {
    if (threadIdx.x == 0) { s.prefix = 0; s.need = (uint32_t)k; }
    uint32_t pmask = 0;
    for (int sh = 24; sh >= 0; sh -= 8) {
        if (threadIdx.x < 256) s.hist[threadIdx.x] = 0;
        __syncthreads();
        const uint32_t prefix = s.prefix;
        for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
            const uint32_t key = key_at(i);
            if ((key & pmask) == prefix) atomicAdd(&s.hist[(key >> sh) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            uint32_t c = 0;
            for (int j = 0; j < 8; ++j) c += s.hist[threadIdx.x * 8 + j];
            uint32_t x = c;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
                if ((int)threadIdx.x >= off) x += y;
            }
            const uint32_t before = x - c;
            const uint32_t need = s.need;
            if (before < need && need <= before + c) {
                uint32_t cum = before;
                for (int j = 0; j < 8; ++j) {
                    const uint32_t h = s.hist[threadIdx.x * 8 + j];
                    if (cum + h >= need) {
                        s.prefix = prefix | ((uint32_t)(threadIdx.x * 8 + j) << sh);
                        s.need = need - cum;
                        break;
                    }
                    cum += h;
                }
            }
        }
        pmask |= 255u << sh;
        __syncthreads();
    }
    *kth = s.prefix;
    *need_eq = s.need;
    __syncthreads();
}

// Key of the k-th smallest value and how many values equal to it are needed
// to complete the k smallest (key order == float order).
__device__ inline void block_kth_key(const float* d, int64_t cols, int k, KthState& s, uint32_t* kth,
                                     uint32_t* need_eq) {
    block_kth_key_of([d](int64_t i) { return float_key_asc(d[i]); }, cols, k, s, kth, need_eq);
}

// The k (<= CHM_MAX_NPROBE) smallest (value, id) of d[0..cols), nearest
// first, ties to the lower id, written to out[0..k).
__device__ inline void block_select_smallest(const float* d, int64_t cols, int k, uint32_t* out) {
    __shared__ KthState s;
    __shared__ uint64_t s_out[CHM_MAX_NPROBE];
    __shared__ uint32_t s_nl, s_ne;
    uint32_t kth, need_eq;
    block_kth_key(d, cols, k, s, &kth, &need_eq);
    if (threadIdx.x == 0) { s_nl = 0; s_ne = 0; }
    __syncthreads();
    for (int64_t base = 0; base < cols; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        uint32_t key = 0xFFFFFFFFu;
        if (i < cols) key = float_key_asc(d[i]);
        const uint32_t lt = (i < cols) && key < kth;
        const uint32_t eq = (i < cols) && key == kth;
        uint32_t tl, te;
        const uint32_t rl = blk_scan_excl(lt, s.warp, &tl);
        const uint32_t re = blk_scan_excl(eq, s.warp, &te);
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
    for (int i = threadIdx.x; i < k; i += blockDim.x) out[i] = (uint32_t)s_out[i];
    __syncthreads();
}

}  // namespace chm
