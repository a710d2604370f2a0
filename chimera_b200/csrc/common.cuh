// Shared device helpers for the chimera_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "chimera_b200.h"

namespace chm {

constexpr int kDim = CHM_PADDED_DIM;
constexpr int kQ = CHM_QLEN;
constexpr int kLutPerQ = 512;  // 32 chunks x 16 entries (config.cuh:16-20)

// Thread-local record of the last CUDA error, surfaced by chm_last_error().
void set_last_error(const char* where, cudaError_t err);
void set_last_message(const char* msg);

inline chm_status launch_status(const char* where) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error(where, e);
        return CHM_ERR_CUDA;
    }
    return CHM_OK;
}

#define CHM_TRY(expr)                          \
    do {                                       \
        chm_status _s = (expr);                \
        if (_s != CHM_OK) return _s;           \
    } while (0)

#define CHM_CUDA(expr)                                   \
    do {                                                 \
        cudaError_t _e = (expr);                         \
        if (_e != cudaSuccess) {                         \
            ::chm::set_last_error(#expr, _e);            \
            return CHM_ERR_CUDA;                         \
        }                                                \
    } while (0)

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace.
struct Arena {
    char* base;
    size_t cap;
    size_t off = 0;
    bool overflow = false;
    Arena(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
    template <typename T>
    T* take(size_t count) {
        size_t o = align_up(off, 256);
        size_t bytes = align_up(count * sizeof(T), 256);
        off = o + bytes;
        if (base == nullptr || off > cap) {
            overflow = true;
            return nullptr;
        }
        return reinterpret_cast<T*>(base + o);
    }
};

// Counting pass with the same layout as Arena (base == nullptr).
struct Sizer {
    size_t off = 0;
    template <typename T>
    void take(size_t count) {
        off = align_up(off, 256) + align_up(count * sizeof(T), 256);
    }
};

// ---- exact fp32 arithmetic (no contraction) -------------------------------
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }

// 1-bit LUT inner product in the reference order: chunk c (0..31) is nibble
// (c & 1) of code byte c/2 (kernels.cu:361-373).  `lut` points at one query
// token's 512 floats in shared memory.
__device__ __forceinline__ float lut_ip(const float* lut, uint4 code) {
    float ip = 0.0f;
    const uint32_t w[4] = {code.x, code.y, code.z, code.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int n = 0; n < 8; ++n) ip = fadd(ip, lut[(q * 8 + n) * 16 + ((w[q] >> (n * 4)) & 0xF)]);
    }
    return ip;
}

// Sum of 16 AVX-512 lanes in _mm512_reduce_add_ps order: upper 8 + lower 8,
// then upper 4 + lower 4, then (0 + 2) + (1 + 3).
__device__ __forceinline__ float reduce16_avx512(const float (&s)[16]) {
    float t3[8], t6[4];
#pragma unroll
    for (int i = 0; i < 8; ++i) t3[i] = fadd(s[8 + i], s[i]);
#pragma unroll
    for (int i = 0; i < 4; ++i) t6[i] = fadd(t3[4 + i], t3[i]);
    return fadd(fadd(t6[0], t6[2]), fadd(t6[1], t6[3]));
}

// Ordered-key transform: ascending uint order == ascending float order.
__device__ __forceinline__ uint32_t float_key_asc(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_to_float_asc(uint32_t k) {
    uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(b);
}

}  // namespace chm
