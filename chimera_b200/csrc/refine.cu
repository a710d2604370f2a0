// Refinement: segmented 1-bit MaxSim of the refined docs, the reference's
// progressive chunked selection of docs to full-bit score, the
// (1+ex_bits)-bit MaxSim itself (moved from the reference's AVX-512 host
// loop onto the GPU with the same arithmetic order), and the final ordering.
#include "codes.cuh"
#include "common.cuh"

namespace chm {

constexpr int kRefineWarps = 8;

// The 1-bit arrays refinement reads: the token-order copies when the index
// has them (a document is one contiguous span, tok2pos passed as NULL), else
// the cluster-ordered arrays gathered through tok2pos.
struct OneBitView {
    const uint32_t* tok2pos;
    const uint8_t* codes;
    const float* factors;
};
inline OneBitView one_bit_view(const chm_index* idx) {
    if (idx->codes1_tok && idx->factor1_tok) return OneBitView{nullptr, idx->codes1_tok, idx->factor1_tok};
    return OneBitView{idx->tok2pos, idx->codes1, idx->factor1};
}

// One warp per refined document; all 32 query-token LUTs in shared memory.
// Replaces gather_refined_doc_lengths/positions, one_bit_token_score and
// one_bit_document_score (kernels.cu:430-617) without materialising the
// [32 x tokens] score matrix.
// Modes (for the tensor-core refinement in refine_tc.cu):
//   kRefineAll     every refined doc;
//   kRefineFlagged every refined doc of the queries whose `status` is set
//                  (a tensor-core launch gave up on a bounded wait).
enum RefineMode { kRefineAll = 0, kRefineFlagged = 1 };

template <int kMode>
__global__ void __launch_bounds__(kRefineWarps * 32) refine_1bit_kernel(
    const int64_t* __restrict__ doc_ptrs, const uint32_t* __restrict__ tok2pos,
    const uint8_t* __restrict__ codes1, const float* __restrict__ factor1,
    const float* __restrict__ lut, const float* __restrict__ cb1,
    const int32_t* __restrict__ refined_docs, const int32_t* __restrict__ num_refined, int k_refine,
    float* __restrict__ scores, const uint32_t* __restrict__ status) {
    extern __shared__ float s_lut[];  // [32][512]
    __shared__ float s_cb1[kQ];
    const int q = blockIdx.y;
    if (kMode == kRefineFlagged && status[q] == 0u) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = num_refined[q];
    if ((int)blockIdx.x * kRefineWarps >= R) return;
    const float4* src = reinterpret_cast<const float4*>(lut + (size_t)q * kQ * kLutPerQ);
    for (int i = threadIdx.x; i < kQ * kLutPerQ / 4; i += blockDim.x)
        reinterpret_cast<float4*>(s_lut)[i] = src[i];
    if (threadIdx.x < kQ) s_cb1[threadIdx.x] = cb1[q * kQ + threadIdx.x];
    __syncthreads();
    // warps stride over the query's docs (one pass for the full grid of kRefineAll)
    for (int i = blockIdx.x * kRefineWarps + warp; i < R; i += gridDim.x * kRefineWarps) {
        const int r = i;
        const int64_t doc = refined_docs[(size_t)q * k_refine + r];
        if (doc < 0) {  // a slot another document shard owns
            if (lane == 0) scores[(size_t)q * k_refine + r] = -INFINITY;
            continue;
        }
        const int64_t t0 = doc_ptrs[doc], t1 = doc_ptrs[doc + 1];
        float m[kQ];
#pragma unroll
        for (int t = 0; t < kQ; ++t) m[t] = -FLT_MAX;
        for (int64_t tok = t0 + lane; tok < t1; tok += 32) {
            const size_t pos = tok2pos ? (size_t)tok2pos[tok] : (size_t)tok;
            const uint4 code = __ldg(reinterpret_cast<const uint4*>(codes1) + pos);
            const float f = __ldg(factor1 + pos);
#pragma unroll
            for (int t = 0; t < kQ; ++t) {
                const float ip = lut_ip(s_lut + t * kLutPerQ, code);
                m[t] = fmaxf(m[t], fmul(fsub(ip, s_cb1[t]), f));
            }
        }
        float mine = 0.0f;
#pragma unroll
        for (int t = 0; t < kQ; ++t) {
            float x = m[t];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
            if (lane == t) mine = x;
        }
        // one_bit_document_score_kernel's 128-thread tree (kernels.cu:557-570):
        // 0.0f + max, two zero strides, then 16, 8, 4, 2, 1.
        float x = fadd(fadd(fadd(0.0f, mine), 0.0f), 0.0f);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off));
        if (lane == 0) scores[(size_t)q * k_refine + r] = x;
    }
}

// The refined docs longer than one tensor-core tile (positions in `list`
// [nq][k_refine], list_count [nq]): one CTA per doc, its warps striding over
// the doc's tokens, the per-query-token maxima merged across warps (max is
// exact in any order), then refine_1bit_kernel's tree.  CTAs stride over the
// listed docs; each stages the query's LUTs once.
__global__ void __launch_bounds__(kRefineWarps * 32) refine_1bit_long_kernel(
    const int64_t* __restrict__ doc_ptrs, const uint32_t* __restrict__ tok2pos,
    const uint8_t* __restrict__ codes1, const float* __restrict__ factor1,
    const float* __restrict__ lut, const float* __restrict__ cb1,
    const int32_t* __restrict__ refined_docs, int k_refine, float* __restrict__ scores,
    const int32_t* __restrict__ list, const int32_t* __restrict__ list_count) {
    extern __shared__ float s_lut[];  // [32][512]
    __shared__ float s_cb1[kQ];
    __shared__ float s_m[kRefineWarps][kQ];
    const int q = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int F = list_count[q];
    if ((int)blockIdx.x >= F) return;
    const float4* src = reinterpret_cast<const float4*>(lut + (size_t)q * kQ * kLutPerQ);
    for (int i = threadIdx.x; i < kQ * kLutPerQ / 4; i += blockDim.x)
        reinterpret_cast<float4*>(s_lut)[i] = src[i];
    if (threadIdx.x < kQ) s_cb1[threadIdx.x] = cb1[q * kQ + threadIdx.x];
    __syncthreads();
    for (int li = blockIdx.x; li < F; li += gridDim.x) {
        const int r = list[(size_t)q * k_refine + li];
        const int64_t doc = refined_docs[(size_t)q * k_refine + r];
        if (doc < 0) {  // uniform across the CTA
            if (threadIdx.x == 0) scores[(size_t)q * k_refine + r] = -INFINITY;
            continue;
        }
        const int64_t t0 = doc_ptrs[doc], t1 = doc_ptrs[doc + 1];
        float m[kQ];
#pragma unroll
        for (int t = 0; t < kQ; ++t) m[t] = -FLT_MAX;
        for (int64_t tok = t0 + threadIdx.x; tok < t1; tok += blockDim.x) {
            const size_t pos = tok2pos ? (size_t)tok2pos[tok] : (size_t)tok;
            const uint4 code = __ldg(reinterpret_cast<const uint4*>(codes1) + pos);
            const float f = __ldg(factor1 + pos);
#pragma unroll
            for (int t = 0; t < kQ; ++t) {
                const float ip = lut_ip(s_lut + t * kLutPerQ, code);
                m[t] = fmaxf(m[t], fmul(fsub(ip, s_cb1[t]), f));
            }
        }
        float mine = 0.0f;
#pragma unroll
        for (int t = 0; t < kQ; ++t) {
            float x = m[t];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
            if (lane == t) mine = x;
        }
        s_m[warp][lane] = mine;
        __syncthreads();
        if (warp == 0) {
            float v = s_m[0][lane];
#pragma unroll
            for (int w = 1; w < kRefineWarps; ++w) v = fmaxf(v, s_m[w][lane]);
            float x = fadd(fadd(fadd(0.0f, v), 0.0f), 0.0f);
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off));
            if (lane == 0) scores[(size_t)q * k_refine + r] = x;
        }
        __syncthreads();  // s_m is reused by the next doc
    }
}

__device__ uint32_t excl_scan_1024(uint32_t v, uint32_t* s_warp, uint32_t* total) {
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

__device__ void sort_desc_u64(uint64_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const uint64_t x = a[i], y = a[l];
                    const bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) { a[i] = y; a[l] = x; }
                }
            }
            __syncthreads();
        }
    }
}

// search_impl.cu:341-494.  After chunk c the reference has full-bit scored
// the top min(T*(c+1)/nch, min(T, end_c)) docs (by 1-bit score) of the
// refined prefix [0, end_c); the union over chunks is what gets scored.
// Ties in the 1-bit score resolve to the lower refined index.
__global__ void __launch_bounds__(1024) select_fullbit_kernel(
    const int32_t* __restrict__ refined_docs, const float* __restrict__ onebit,
    const int32_t* __restrict__ num_refined, int k_refine, int k_full_bit, int num_chunks,
    int32_t* __restrict__ fb_docs, int32_t* __restrict__ num_fb, int fb_cap) {
    extern __shared__ uint64_t s_keys[];   // [sort_n]
    __shared__ uint8_t s_chosen[CHM_MAX_K_REFINE];
    __shared__ uint32_t s_warp[33];
    const int q = blockIdx.x;
    const int R = num_refined[q];
    int sort_n = 1;
    while (sort_n < R) sort_n <<= 1;
    for (int i = threadIdx.x; i < sort_n; i += blockDim.x) {
        if (i < R) {
            const float s = onebit[(size_t)q * k_refine + i];
            s_keys[i] = ((uint64_t)float_key_asc(s) << 32) | (uint32_t)(~(uint32_t)i);
            s_chosen[i] = 0;
        } else {
            s_keys[i] = 0;
        }
    }
    __syncthreads();
    if (R == 0) {
        if (threadIdx.x == 0) num_fb[q] = 0;
        return;
    }
    sort_desc_u64(s_keys, sort_n);
    const int T = min(k_full_bit, R);
    const int nch = min(num_chunks, R);
    const int cs = (R + nch - 1) / nch;
    const int per = (R + blockDim.x - 1) / blockDim.x;  // sorted entries per thread
    for (int c = 0; c < nch; ++c) {
        const int end = min((c + 1) * cs, R);
        const int carry = min(T, end);
        const int cum = min(T * (c + 1) / nch, carry);
        uint32_t cnt = 0;
        const int i0 = threadIdx.x * per, i1 = min(R, i0 + per);
        for (int i = i0; i < i1; ++i) cnt += ((int)(~(uint32_t)s_keys[i]) < end);
        uint32_t tot;
        uint32_t rank = excl_scan_1024(cnt, s_warp, &tot);
        for (int i = i0; i < i1 && (int)rank < cum; ++i) {
            const int idx = (int)(~(uint32_t)s_keys[i]);
            if (idx < end) { s_chosen[idx] = 1; ++rank; }
        }
        __syncthreads();
    }
    // compact chosen refined indices in ascending order
    const int i0 = threadIdx.x * per, i1 = min(R, i0 + per);
    uint32_t cnt = 0;
    for (int i = i0; i < i1; ++i) cnt += s_chosen[i];
    uint32_t tot;
    uint32_t at = excl_scan_1024(cnt, s_warp, &tot);
    for (int i = i0; i < i1; ++i)
        if (s_chosen[i] && (int)at < fb_cap) fb_docs[(size_t)q * fb_cap + at++] = refined_docs[(size_t)q * k_refine + i];
    if (threadIdx.x == 0) num_fb[q] = min((int)tot, fb_cap);
}

// (1+ex_bits)-bit MaxSim, one warp per selected doc, lane t = query token t
// with its 128 rotated query values held in registers.  For every token the
// warp decodes the packed code once into shared memory; each lane then forms
// the 16 AVX-512 lane accumulators of gemv_batch8_avx512
// (space.hpp:806-851), s[l] = fma(decoded[16b + l], q[16b + l], s[l]) over
// b = 0..7, reduces them in _mm512_reduce_add_ps order (8+8, 4+4, (0+2)+(1+3)),
// and keeps max((ip - cbex) * factor) (search_impl.cu:538-566).  The doc
// score adds the two 16-lane halves of the maxima and reduces them the same
// way (:569-572).
constexpr int kFbWarps = 4;
constexpr int kFbChunkTokens = 32;   // tokens staged in shared memory at a time

__global__ void __launch_bounds__(kFbWarps * 32) fullbit_kernel(
    const int64_t* __restrict__ doc_ptrs, const uint8_t* __restrict__ full_codes,
    const float* __restrict__ full_factors, int w, const float* __restrict__ rot,
    const float* __restrict__ cbex, const int32_t* __restrict__ fb_docs,
    const int32_t* __restrict__ num_fb, int fb_cap, float* __restrict__ scores) {
    // per warp: up to 32 tokens' packed codes (<= 128 B each) and factors,
    // plus one decoded token (128 floats)
    __shared__ __align__(16) uint8_t s_code[kFbWarps][kFbChunkTokens * 128];
    __shared__ float s_fac[kFbWarps][kFbChunkTokens];
    __shared__ __align__(16) float s_dec[kFbWarps][kDim];
    const int q = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int F = num_fb[q];
    // warps stride over the query's docs (the grid may be smaller than F / kFbWarps)
    for (int li = blockIdx.x * kFbWarps + warp; li < F; li += gridDim.x * kFbWarps) {
        const int i = li;
        float qr[kDim];
        const float4* qsrc = reinterpret_cast<const float4*>(rot + ((size_t)q * kQ + lane) * kDim);
#pragma unroll
        for (int j = 0; j < kDim / 4; ++j) {
            const float4 v = qsrc[j];
            qr[4 * j] = v.x; qr[4 * j + 1] = v.y; qr[4 * j + 2] = v.z; qr[4 * j + 3] = v.w;
        }
        const float cb = cbex[q * kQ + lane];
        const int64_t doc = fb_docs[(size_t)q * fb_cap + i];
        if (doc < 0) {  // a slot another document shard owns
            if (lane == 0) scores[(size_t)q * fb_cap + i] = -INFINITY;
            continue;
        }
        const int bytes = kDim * w / 8;       // 16 * w, a multiple of 16
        const int64_t t0 = doc_ptrs[doc], t1 = doc_ptrs[doc + 1];
        float m = -INFINITY;
        for (int64_t c0 = t0; c0 < t1; c0 += kFbChunkTokens) {
            const int nt = (int)min((int64_t)kFbChunkTokens, t1 - c0);
            // one coalesced burst: the chunk's codes are contiguous in token order
            const uint4* src = reinterpret_cast<const uint4*>(full_codes + (size_t)c0 * bytes);
            uint4* dst = reinterpret_cast<uint4*>(s_code[warp]);
            for (int v = lane; v < nt * bytes / 16; v += 32) dst[v] = __ldg(src + v);
            if (lane < nt) s_fac[warp][lane] = __ldg(full_factors + c0 + lane);
            __syncwarp();
            for (int t = 0; t < nt; ++t) {
                const uint8_t* code = s_code[warp] + t * bytes;
#pragma unroll
                for (int k = 0; k < 4; ++k) s_dec[warp][32 * k + lane] = (float)code_at(code, 32 * k + lane, w);
                __syncwarp();
                float s[16];
#pragma unroll
                for (int l = 0; l < 16; ++l) s[l] = 0.0f;
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const float4* dv = reinterpret_cast<const float4*>(&s_dec[warp][16 * b]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float4 d4 = dv[j];
                        s[4 * j + 0] = __fmaf_rn(d4.x, qr[16 * b + 4 * j + 0], s[4 * j + 0]);
                        s[4 * j + 1] = __fmaf_rn(d4.y, qr[16 * b + 4 * j + 1], s[4 * j + 1]);
                        s[4 * j + 2] = __fmaf_rn(d4.z, qr[16 * b + 4 * j + 2], s[4 * j + 2]);
                        s[4 * j + 3] = __fmaf_rn(d4.w, qr[16 * b + 4 * j + 3], s[4 * j + 3]);
                    }
                }
                const float ip = reduce16_avx512(s);
                m = fmaxf(m, fmul(fsub(ip, cb), s_fac[warp][t]));
                __syncwarp();
            }
        }
        // sum = max[0:16] + max[16:32] lane-wise, then the 16-lane reduction
        float x = fadd(m, __shfl_down_sync(0xffffffffu, m, 16));
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off, 16));
        if (lane == 0) scores[(size_t)q * fb_cap + i] = x;
        __syncwarp();  // s_code / s_dec are reused by the warp's next doc
    }
}

// The full-bit docs longer than one tensor-core tile (positions in `list`
// [nq][fb_cap], list_count [nq]): one CTA per doc, each warp taking every
// kFbWarps-th chunk of kFbChunkTokens tokens with fullbit_kernel's
// arithmetic, the per-query-token maxima merged across warps (exact in any
// order), then fullbit_kernel's reduction.  CTAs stride over the listed docs.
__global__ void __launch_bounds__(kFbWarps * 32) fullbit_long_kernel(
    const int64_t* __restrict__ doc_ptrs, const uint8_t* __restrict__ full_codes,
    const float* __restrict__ full_factors, int w, const float* __restrict__ rot,
    const float* __restrict__ cbex, const int32_t* __restrict__ fb_docs, int fb_cap, float* __restrict__ scores,
    const int32_t* __restrict__ list, const int32_t* __restrict__ list_count) {
    __shared__ __align__(16) uint8_t s_code[kFbWarps][kFbChunkTokens * 128];
    __shared__ float s_fac[kFbWarps][kFbChunkTokens];
    __shared__ __align__(16) float s_dec[kFbWarps][kDim];
    __shared__ float s_m[kFbWarps][kQ];
    const int q = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int F = list_count[q];
    if ((int)blockIdx.x >= F) return;
    float qr[kDim];
    const float4* qsrc = reinterpret_cast<const float4*>(rot + ((size_t)q * kQ + lane) * kDim);
#pragma unroll
    for (int j = 0; j < kDim / 4; ++j) {
        const float4 v = qsrc[j];
        qr[4 * j] = v.x; qr[4 * j + 1] = v.y; qr[4 * j + 2] = v.z; qr[4 * j + 3] = v.w;
    }
    const float cb = cbex[q * kQ + lane];
    const int bytes = kDim * w / 8;  // 16 * w, a multiple of 16
    for (int li = blockIdx.x; li < F; li += gridDim.x) {
        const int i = list[(size_t)q * fb_cap + li];
        const int64_t doc = fb_docs[(size_t)q * fb_cap + i];
        if (doc < 0) {  // uniform across the CTA
            if (threadIdx.x == 0) scores[(size_t)q * fb_cap + i] = -INFINITY;
            continue;
        }
        const int64_t t0 = doc_ptrs[doc], t1 = doc_ptrs[doc + 1];
        float m = -INFINITY;
        for (int64_t c0 = t0 + (int64_t)warp * kFbChunkTokens; c0 < t1; c0 += kFbWarps * kFbChunkTokens) {
            const int nt = (int)min((int64_t)kFbChunkTokens, t1 - c0);
            const uint4* src = reinterpret_cast<const uint4*>(full_codes + (size_t)c0 * bytes);
            uint4* dst = reinterpret_cast<uint4*>(s_code[warp]);
            for (int v = lane; v < nt * bytes / 16; v += 32) dst[v] = __ldg(src + v);
            if (lane < nt) s_fac[warp][lane] = __ldg(full_factors + c0 + lane);
            __syncwarp();
            for (int t = 0; t < nt; ++t) {
                const uint8_t* code = s_code[warp] + t * bytes;
#pragma unroll
                for (int k = 0; k < 4; ++k) s_dec[warp][32 * k + lane] = (float)code_at(code, 32 * k + lane, w);
                __syncwarp();
                float s[16];
#pragma unroll
                for (int l = 0; l < 16; ++l) s[l] = 0.0f;
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const float4* dv = reinterpret_cast<const float4*>(&s_dec[warp][16 * b]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float4 d4 = dv[j];
                        s[4 * j + 0] = __fmaf_rn(d4.x, qr[16 * b + 4 * j + 0], s[4 * j + 0]);
                        s[4 * j + 1] = __fmaf_rn(d4.y, qr[16 * b + 4 * j + 1], s[4 * j + 1]);
                        s[4 * j + 2] = __fmaf_rn(d4.z, qr[16 * b + 4 * j + 2], s[4 * j + 2]);
                        s[4 * j + 3] = __fmaf_rn(d4.w, qr[16 * b + 4 * j + 3], s[4 * j + 3]);
                    }
                }
                const float ip = reduce16_avx512(s);
                m = fmaxf(m, fmul(fsub(ip, cb), s_fac[warp][t]));
                __syncwarp();
            }
        }
        s_m[warp][lane] = m;
        __syncthreads();
        if (warp == 0) {
            float v = s_m[0][lane];
#pragma unroll
            for (int ww = 1; ww < kFbWarps; ++ww) v = fmaxf(v, s_m[ww][lane]);
            // sum = max[0:16] + max[16:32] lane-wise, then the 16-lane reduction
            float x = fadd(v, __shfl_down_sync(0xffffffffu, v, 16));
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off, 16));
            if (lane == 0) scores[(size_t)q * fb_cap + i] = x;
        }
        __syncthreads();  // s_m is reused by the next doc
    }
}

// std::priority_queue<std::pair<float, size_t>> pop order: score desc, doc
// desc (search_impl.cu:409, 496-500).
__global__ void __launch_bounds__(1024) final_topk_kernel(
    const int32_t* __restrict__ fb_docs, const float* __restrict__ fb_scores,
    const int32_t* __restrict__ num_fb, int fb_cap, int k, int64_t* __restrict__ results,
    int32_t* __restrict__ num_results) {
    extern __shared__ uint64_t s_keys[];
    const int q = blockIdx.x;
    const int F = num_fb[q];
    int sort_n = 1;
    while (sort_n < F) sort_n <<= 1;
    for (int i = threadIdx.x; i < sort_n; i += blockDim.x) {
        if (i < F) {
            const float s = fb_scores[(size_t)q * fb_cap + i];
            s_keys[i] = ((uint64_t)float_key_asc(s) << 32) | (uint32_t)fb_docs[(size_t)q * fb_cap + i];
        } else {
            s_keys[i] = 0;
        }
    }
    __syncthreads();
    sort_desc_u64(s_keys, sort_n);
    const int nk = min(k, F);
    for (int i = threadIdx.x; i < k; i += blockDim.x)
        results[(size_t)q * k + i] = i < nk ? (int64_t)(uint32_t)s_keys[i] : -1;
    if (threadIdx.x == 0) num_results[q] = nk;
}

// Merge of per-shard top-k lists gathered across GPUs (same ordering rule).
__global__ void __launch_bounds__(1024) merge_topk_kernel(
    int shards, int k, const float* __restrict__ scores, const int64_t* __restrict__ docs,
    const int32_t* __restrict__ counts, int64_t* __restrict__ results,
    float* __restrict__ result_scores, int32_t* __restrict__ num_results) {
    extern __shared__ uint64_t s_keys[];
    const int q = blockIdx.x;
    const int n = shards * k;
    int sort_n = 1;
    while (sort_n < n) sort_n <<= 1;
    for (int i = threadIdx.x; i < sort_n; i += blockDim.x) {
        uint64_t key = 0;
        if (i < n) {
            const int s = i / k, j = i % k;
            const size_t at = ((size_t)s * gridDim.x + q) * k + j;
            if (j < counts[(size_t)s * gridDim.x + q])
                key = ((uint64_t)float_key_asc(scores[at]) << 32) | (uint32_t)docs[at];
        }
        s_keys[i] = key;
    }
    __syncthreads();
    sort_desc_u64(s_keys, sort_n);
    __shared__ int s_n;
    if (threadIdx.x == 0) {
        int c = 0;
        while (c < k && c < n && s_keys[c] != 0) ++c;
        s_n = c;
        num_results[q] = c;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const bool ok = i < s_n;
        results[(size_t)q * k + i] = ok ? (int64_t)(uint32_t)s_keys[i] : -1;
        if (result_scores) result_scores[(size_t)q * k + i] = ok ? key_to_float_asc((uint32_t)(s_keys[i] >> 32)) : -INFINITY;
    }
}

static size_t pow2_bytes(int n) {
    int s = 1;
    while (s < n) s <<= 1;
    return sizeof(uint64_t) * (size_t)s;
}

// Always raise the dynamic limit: static + dynamic shared memory together
// may pass the 48 KB default even when the dynamic part alone does not.
template <typename K>
static chm_status set_smem(K kernel, size_t bytes) {
    CHM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return CHM_OK;
}

}  // namespace chm

extern "C" chm_status chm_refine_1bit(const chm_index* idx, int32_t nq, const float* lut,
                                      const float* cb1, const int32_t* refined_docs,
                                      const int32_t* num_refined, int32_t k_refine, float* scores,
                                      void* stream) {
    if (nq <= 0) return CHM_OK;
    const size_t smem = sizeof(float) * chm::kQ * chm::kLutPerQ;
    CHM_TRY(chm::set_smem(chm::refine_1bit_kernel<chm::kRefineAll>, smem));
    dim3 g((k_refine + chm::kRefineWarps - 1) / chm::kRefineWarps, nq);
    const chm::OneBitView v = chm::one_bit_view(idx);
    chm::refine_1bit_kernel<chm::kRefineAll><<<g, chm::kRefineWarps * 32, smem, (cudaStream_t)stream>>>(
        idx->doc_ptrs, v.tok2pos, v.codes, v.factors, lut, cb1, refined_docs, num_refined, k_refine, scores,
        nullptr);
    return chm::launch_status("refine_1bit_kernel");
}

// SIMT passes that complete the tensor-core refinement: the listed long docs,
// then every doc of the queries whose tensor-core launch reported a failure.
chm_status chm_refine_1bit_complete(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                                    const int32_t* refined_docs, const int32_t* num_refined, int32_t k_refine,
                                    float* scores, const int32_t* list, const int32_t* list_count,
                                    const uint32_t* status, cudaStream_t st) {
    const size_t smem = sizeof(float) * chm::kQ * chm::kLutPerQ;
    const chm::OneBitView v = chm::one_bit_view(idx);
    // a few long docs per query, a CTA each
    CHM_TRY(chm::set_smem(chm::refine_1bit_long_kernel, smem));
    chm::refine_1bit_long_kernel<<<dim3(16, nq), chm::kRefineWarps * 32, smem, st>>>(
        idx->doc_ptrs, v.tok2pos, v.codes, v.factors, lut, cb1, refined_docs, k_refine, scores, list, list_count);
    CHM_TRY(chm::launch_status("refine_1bit_long_kernel"));
    // (rarely) every doc of a flagged query: a small grid whose warps stride over them
    CHM_TRY(chm::set_smem(chm::refine_1bit_kernel<chm::kRefineFlagged>, smem));
    chm::refine_1bit_kernel<chm::kRefineFlagged><<<dim3(4, nq), chm::kRefineWarps * 32, smem, st>>>(
        idx->doc_ptrs, v.tok2pos, v.codes, v.factors, lut, cb1, refined_docs, num_refined, k_refine, scores,
        status);
    return chm::launch_status("refine_1bit_flagged");
}

extern "C" chm_status chm_select_fullbit(int32_t nq, const int32_t* refined_docs,
                                         const float* onebit, const int32_t* num_refined,
                                         int32_t k_refine, int32_t k_full_bit, int32_t num_chunks,
                                         int32_t* fb_docs, int32_t* num_fb, int32_t fb_cap,
                                         void* stream) {
    if (nq <= 0) return CHM_OK;
    if (k_refine > CHM_MAX_K_REFINE || k_full_bit <= 0 || num_chunks <= 0) return CHM_ERR_INVALID;
    const size_t smem = chm::pow2_bytes(k_refine);
    CHM_TRY(chm::set_smem(chm::select_fullbit_kernel, smem));
    chm::select_fullbit_kernel<<<nq, 1024, smem, (cudaStream_t)stream>>>(
        refined_docs, onebit, num_refined, k_refine, k_full_bit, num_chunks, fb_docs, num_fb, fb_cap);
    return chm::launch_status("select_fullbit_kernel");
}

extern "C" chm_status chm_fullbit_score(const chm_index* idx, int32_t nq, const float* rot,
                                        const float* cbex, const int32_t* fb_docs,
                                        const int32_t* num_fb, int32_t fb_cap, float* scores,
                                        void* stream) {
    if (nq <= 0) return CHM_OK;
    dim3 g((fb_cap + chm::kFbWarps - 1) / chm::kFbWarps, nq);
    chm::fullbit_kernel<<<g, chm::kFbWarps * 32, 0, (cudaStream_t)stream>>>(
        idx->doc_ptrs, idx->full_codes, idx->full_factors, 1 + idx->ex_bits, rot, cbex, fb_docs,
        num_fb, fb_cap, scores);
    return chm::launch_status("fullbit_kernel");
}

// chm_fullbit_score over a small grid: for rescoring a few flagged queries
chm_status chm_fullbit_flagged(const chm_index* idx, int32_t nq, const float* rot, const float* cbex,
                               const int32_t* fb_docs, const int32_t* counts, int32_t fb_cap, float* scores,
                               cudaStream_t st) {
    chm::fullbit_kernel<<<dim3(2, nq), chm::kFbWarps * 32, 0, st>>>(
        idx->doc_ptrs, idx->full_codes, idx->full_factors, 1 + idx->ex_bits, rot, cbex, fb_docs, counts, fb_cap,
        scores);
    return chm::launch_status("fullbit_flagged");
}

chm_status chm_fullbit_listed(const chm_index* idx, int32_t nq, const float* rot, const float* cbex,
                              const int32_t* fb_docs, const int32_t* num_fb, int32_t fb_cap, float* scores,
                              const int32_t* list, const int32_t* list_count, cudaStream_t st) {
    // a few long docs per query, a CTA each
    chm::fullbit_long_kernel<<<dim3(16, nq), chm::kFbWarps * 32, 0, st>>>(
        idx->doc_ptrs, idx->full_codes, idx->full_factors, 1 + idx->ex_bits, rot, cbex, fb_docs, fb_cap, scores, list,
        list_count);
    return chm::launch_status("fullbit_listed");
}

extern "C" chm_status chm_final_topk(int32_t nq, const int32_t* fb_docs, const float* fb_scores,
                                     const int32_t* num_fb, int32_t fb_cap, int32_t k,
                                     int64_t* results, int32_t* num_results, void* stream) {
    if (nq <= 0) return CHM_OK;
    if (fb_cap > CHM_MAX_K_REFINE || k <= 0) return CHM_ERR_INVALID;
    const size_t smem = chm::pow2_bytes(fb_cap);
    CHM_TRY(chm::set_smem(chm::final_topk_kernel, smem));
    chm::final_topk_kernel<<<nq, 1024, smem, (cudaStream_t)stream>>>(fb_docs, fb_scores, num_fb, fb_cap,
                                                                     k, results, num_results);
    return chm::launch_status("final_topk_kernel");
}

extern "C" chm_status chm_merge_topk(int32_t nq, int32_t shards, int32_t k, const float* scores,
                                     const int64_t* docs, const int32_t* counts, int64_t* results,
                                     float* result_scores, int32_t* num_results, void* stream) {
    if (nq <= 0) return CHM_OK;
    if (shards <= 0 || k <= 0 || (int64_t)shards * k > 16384) return CHM_ERR_INVALID;
    const size_t smem = chm::pow2_bytes(shards * k);
    CHM_TRY(chm::set_smem(chm::merge_topk_kernel, smem));
    chm::merge_topk_kernel<<<nq, 1024, smem, (cudaStream_t)stream>>>(shards, k, scores, docs, counts,
                                                                     results, result_scores, num_results);
    return chm::launch_status("merge_topk_kernel");
}
