// Warp-level FhtKac rotation and Eigen-order reductions.
//
// Register layout ("strided"): lane l holds v[k] = x[32*k + l], k = 0..3.
// With this layout
//  * FHT strides 1..16 are lane exchanges (xor 1..16) and strides 32, 64
//    are register exchanges;
//  * word k of a 1-bit code (dims 32k..32k+31) is __ballot_sync(v[k] > 0);
//  * Eigen 3.4's AVX-512 dot product of two 128-vectors (two 16-lane packet
//    accumulators over alternating packets, then predux) is a per-lane chain
//    x*y, fma, fma, fma over slots 0..3 followed by a shuffle-down tree
//    16, 8, 4, 2, 1.
#pragma once
#include "common.cuh"

namespace chm {

// Butterfly (a, b) -> (a + b, a - b) between lanes l and l ^ m: the lower
// lane keeps a + b, the upper lane a - b (FFHT helper_float_*, fht_avx.cpp).
__device__ __forceinline__ float bfly_lane(float x, int lane, int m) {
    const float p = __shfl_xor_sync(0xffffffffu, x, m);
    return (lane & m) ? fsub(p, x) : fadd(x, p);
}

// In-place FHT of `n` (64 or 128) consecutive elements starting at slot
// `s0`, ascending strides 1, 2, 4, ... n/2 (FFHT stage order).
__device__ __forceinline__ void fht_warp(float (&v)[4], int lane, int n, int s0) {
    const int slots = n / 32;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (k >= s0 && k < s0 + slots) v[k] = bfly_lane(v[k], lane, m);
    }
    // stride 32 (slot pairs (0,1), (2,3)) then, for n == 128, stride 64.
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
        if (k >= s0 && k < s0 + slots) {
            const float a = v[k], b = v[k + 1];
            v[k] = fadd(a, b);
            v[k + 1] = fsub(a, b);
        }
    }
    if (n == 128) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float a = v[k], b = v[k + 2];
            v[k] = fadd(a, b);
            v[k + 2] = fsub(a, b);
        }
    }
}

// FhtKacRotator::rotate (rotator.hpp:281-334) for one vector held in the
// strided layout; padded_dim is 128, `trunc` = 2^floor(log2(dim)), `fac` =
// 1.0f / std::sqrt((float)trunc) computed by the host.
__device__ __forceinline__ void rotate_warp(float (&v)[4], int lane, const uint8_t* flips,
                                            int trunc, float fac) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        // flip_sign: element i flips when bit i % 8 of byte 16r + i / 8 is set
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint8_t byte = flips[16 * r + 4 * k + (lane >> 3)];
            if ((byte >> (lane & 7)) & 1) v[k] = -v[k];
        }
        if (trunc == 128) {
            fht_warp(v, lane, 128, 0);
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = fmul(v[k], fac);
        } else {
            const int s0 = (r & 1) ? 2 : 0;  // rounds 1 and 3 act on the upper 64
            fht_warp(v, lane, 64, s0);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (k >= s0 && k < s0 + 2) v[k] = fmul(v[k], fac);
            // kacs_walk(128): x[i] +- x[i + 64]
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const float a = v[k], b = v[k + 2];
                v[k] = fadd(a, b);
                v[k + 2] = fsub(a, b);
            }
        }
    }
    if (trunc != 128) {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = fmul(v[k], 0.25f);
    }
}

// Eigen 3.4 dot of two 128-vectors in the strided layout (Redux.h:227-282
// with Packet16f, products fused into the accumulating adds).  Result valid
// in every lane.
__device__ __forceinline__ float eigen_dot_warp(const float (&a)[4], const float (&b)[4]) {
    float x = fmul(a[0], b[0]);
    x = __fmaf_rn(a[1], b[1], x);
    x = __fmaf_rn(a[2], b[2], x);
    x = __fmaf_rn(a[3], b[3], x);
    // predux: lane L of packet_res0 (+) lane L of packet_res1, then 8, 4,
    // (0+2)+(1+3).  Lane l < 16 is packet_res0[l], lane 16 + l packet_res1[l].
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off));
    return __shfl_sync(0xffffffffu, x, 0);
}

}  // namespace chm
