// Stage 1, dense-bound path: the same refined list as the hash-table path
// (stage1.cu) and as the reference's mark -> partial_score -> sum -> sort
// pipeline (kernels.cu:117-400, search_impl.cu:118-262), with far less
// memory traffic and aggregation work.
//
// The partial score of a doc is P(doc) = tree-sum over query tokens t of
// m(doc, t), m = max(0, max dist over the doc's visits for t) (kernels.cu:
// 376-397, 192-198).  The sum of all its positive visits,
// S(doc) = sum dist > 0, is an upper bound: P <= S in real arithmetic, and
// with fp32 rounding (any summation order for S, the 5-level tree for P)
//     P_fp32 <= S_fp32 * (1 + eps),  eps = (32 * max_doc_len + 8) * 2^-24 * 1.25
// because a token sits in one cluster, so a doc has at most 32 * doclen
// positive visits.  The score pass sums upper bounds of the dists instead of
// the dists: the 8-bit LUT entry for byte b is the sum of the reference's two
// 4-bit entries (chunks 2b, 2b + 1), and both ip sums are sums of the same
// <= 128 query components along trees of height <= 35 (reference) and <= 12
// (here), so |ip' - ip| <= 47 u sum|q| (u = 2^-24); the subtraction of cb1,
// the product with the factor and the final fma add <= 6 u (sum|q| + |cb1|)
// per unit |factor| for both paths together.  m = |factor| * M_t with
// M_t = 2^-24 (100 sum|q| + 16 |cb1|) covers all of it with room.
//
//  score   : CTA per (query token t, split, query); each warp streams whole
//            probed lists (no per-visit search), scores each code with an
//            8-bit LUT (16 lookups instead of the reference's 32) and posts
//            dist' + m > 0 into S[q][doc] with a fire-and-forget float
//            reduction (runs of one doc inside a warp are summed first: the
//            lists are in doc order).  m bounds |dist' - dist| (below), so
//            every term is at least the reference's dist and S stays an
//            upper bound.
//  hist / pivot / compact : per query, the 12-bit bucket that holds the
//            K'-th largest S (K' = k_refine + slack) and the keys
//            (S << 32 | ~doc) at or above it.
//  select  : per query, the K' + 1 largest keys: K' candidates and the
//            boundary (the largest S left out).
//  exact   : per candidate doc, P exactly as the reference computes it: its
//            tokens (token order) whose cluster query token t probed, the
//            LUT dist in the reference order, max per t, the tree.
//  final   : per query, the candidates by (P desc, doc asc); when
//            boundary * (1 + eps) < the k_refine-th P, no doc left out can
//            reach the refined list, which is then exactly the reference's.
//            An unproven boundary gets a second round with K' = 12,288 (or
//            every doc); what is still unproven -- and queries with fewer than
//            k_refine positive docs, whose zero-score fill needs the
//            visited-doc bitmap -- is flagged for the hash-table path.
#include "common.cuh"

namespace chm {

constexpr int kBsWarps = 8;            // score CTA
constexpr int kBxWarps = 32;           // exact CTA
constexpr int kMapSlots = 8192;        // probed-cluster map per query (>= 2 x 32 x max nprobe / 8)
constexpr uint64_t kMapEmpty = ~0ull;
constexpr int kBPreThreads = 256;
constexpr int kBUnroll = 8;             // loads in flight per thread in the scans over S
constexpr int64_t kBPreCap = 65536;    // compacted keys per query (more: fallback)
constexpr uint32_t kBNoPivot = 0xFFFFFFFFu;
constexpr int kBMaxCand = 12288;       // K' bound (sort buffer 16384 keys)

__device__ __forceinline__ bool b_inactive(const uint32_t* active, int q) { return active != nullptr && active[q] == 0u; }

// LUT sum in the reference order (chunk c = 0..31 is nibble c & 1 of code
// byte c / 2, kernels.cu:361-373).  The nibbles' byte offsets are formed four
// at a time (a shift and a mask per code word) and picked out with one byte
// permute per lookup.  lut: one query token's 512 floats in shared memory.
__device__ __forceinline__ float lut_ip_prmt(const float* lut, uint4 code) {
    const uint32_t w[4] = {code.x, code.y, code.z, code.w};
    const char* base = reinterpret_cast<const char*>(lut);
    float ip = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t lo = (w[q] << 2) & 0x3C3C3C3Cu;  // byte i: 4 x (low nibble of byte i)
        const uint32_t hi = (w[q] >> 2) & 0x3C3C3C3Cu;  // byte i: 4 x (high nibble of byte i)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = q * 8 + 2 * i;
            ip = fadd(ip, *reinterpret_cast<const float*>(base + c * 64 + __byte_perm(lo, 0, 0x4440 + i)));
            ip = fadd(ip, *reinterpret_cast<const float*>(base + (c + 1) * 64 + __byte_perm(hi, 0, 0x4440 + i)));
        }
    }
    return ip;
}

struct BoundCtx {
    const int64_t* cluster_pos;
    const uint8_t* codes1;
    const float* factor1;
    const int32_t* doc_ids;
    int64_t n_clusters;
    int64_t num_docs;
    const float* lut;        // [nq][32][512]
    const float* cb1;        // [nq][32]
    const uint32_t* labels;  // [nq][32][nprobe]
    int nprobe;
    float* S;                // [nq][num_docs], zero on entry
};

// Posts this lane's dist (when valid and positive) into S[doc].  Lanes hold
// consecutive elements of one list, so equal docs are adjacent lanes: when a
// warp has such a run, a segmented scan sums it and the run's last lane posts.
__device__ __forceinline__ void post_dist(float* S, int doc, float d, bool valid, int lane) {
    const bool pos = valid && d > 0.0f;
    const int nd = __shfl_down_sync(0xffffffffu, doc, 1);
    const int npos = __shfl_down_sync(0xffffffffu, pos ? 1 : 0, 1);
    const bool run_next = lane < 31 && pos && npos && nd == doc;
    if (__any_sync(0xffffffffu, run_next)) {
        float s = pos ? d : 0.0f;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, s, off);
            const int pd = __shfl_up_sync(0xffffffffu, doc, off);
            if (lane >= off && pd == doc) s += y;
        }
        const bool last = !(lane < 31 && nd == doc);
        if (valid && last && s > 0.0f) atomicAdd(S + doc, s);
    } else if (pos) {
        atomicAdd(S + doc, d);
    }
}

// 8-bit LUT sum of a 1-bit code: byte b of the code indexes entry b of
// `lut8` ([16][256], shared memory); two interleaved chains of 8 adds.
__device__ __forceinline__ float lut8_ip(const float* lut8, uint4 code) {
    const uint32_t w[4] = {code.x, code.y, code.z, code.w};
    float a = 0.0f, b = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float v = lut8[(q * 4 + i) * 256 + __byte_perm(w[q], 0, 0x4440 + i)];
            if (q < 2) a = fadd(a, v); else b = fadd(b, v);
        }
    }
    return fadd(a, b);
}

__global__ void __launch_bounds__(kBsWarps * 32) bound_score_kernel(BoundCtx c, int splits) {
    __shared__ float s_lut[kLutPerQ];
    __shared__ float s_lut8[16 * 256];
    __shared__ float s_mt;
    __shared__ int s_next;
    const int t = blockIdx.x / splits, split = blockIdx.x % splits;
    const int q = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float4* src = reinterpret_cast<const float4*>(c.lut + ((size_t)q * kQ + t) * kLutPerQ);
    for (int i = threadIdx.x; i < kLutPerQ / 4; i += blockDim.x) reinterpret_cast<float4*>(s_lut)[i] = src[i];
    if (threadIdx.x == 0) s_next = kBsWarps;
    __syncthreads();
    const float cb1 = c.cb1[q * kQ + t];
    // byte b's entries: chunk 2b is its low nibble, chunk 2b + 1 its high one
    for (int i = threadIdx.x; i < 16 * 256; i += blockDim.x) {
        const int b = i >> 8, e = i & 255;
        s_lut8[i] = fadd(s_lut[(2 * b) * 16 + (e & 15)], s_lut[(2 * b + 1) * 16 + (e >> 4)]);
    }
    if (warp == 0) {
        // sum |q_d|: the single-bit entries are the components themselves
        float a = 0.0f;
#pragma unroll
        for (int bit = 0; bit < 4; ++bit) a += fabsf(s_lut[lane * 16 + (1 << bit)]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        if (lane == 0) s_mt = (100.0f * a + 16.0f * fabsf(cb1)) * 0x1p-24f;
    }
    __syncthreads();
    const float mt = s_mt;
    const uint32_t* labels = c.labels + ((size_t)q * kQ + t) * c.nprobe;
    float* S = c.S + (size_t)q * c.num_docs;
    // warps take this split's lists (p = split + k * splits) in turn
    for (int k = warp;;) {
        const int p = split + k * splits;
        if (p >= c.nprobe) break;
        const uint32_t label = labels[p];
        if ((int64_t)label < c.n_clusters) {
            const int64_t st = c.cluster_pos[label];
            const int len = (int)(c.cluster_pos[label + 1] - st);
            const uint4* codes = reinterpret_cast<const uint4*>(c.codes1) + st;
            const float* fac = c.factor1 + st;
            const int32_t* docs = c.doc_ids + st;
            for (int b = 0; b < len; b += 64) {
                // two elements per lane in flight
                const int e0 = b + lane, e1 = b + 32 + lane;
                const bool v0 = e0 < len, v1 = e1 < len;
                uint4 k0 = make_uint4(0, 0, 0, 0), k1 = make_uint4(0, 0, 0, 0);
                float f0 = 0.0f, f1 = 0.0f;
                int d0 = -1, d1 = -1;
                if (v0) { k0 = __ldg(codes + e0); f0 = __ldg(fac + e0); d0 = __ldg(docs + e0); }
                if (v1) { k1 = __ldg(codes + e1); f1 = __ldg(fac + e1); d1 = __ldg(docs + e1); }
                // dist' + |f| M_t >= the reference's dist
                const float dist0 = __fmaf_ru(fabsf(f0), mt, fmul(fsub(lut8_ip(s_lut8, k0), cb1), f0));
                post_dist(S, d0, dist0, v0 && d0 >= 0 && (int64_t)d0 < c.num_docs, lane);
                if (b + 32 < len) {
                    const float dist1 = __fmaf_ru(fabsf(f1), mt, fmul(fsub(lut8_ip(s_lut8, k1), cb1), f1));
                    post_dist(S, d1, dist1, v1 && d1 >= 0 && (int64_t)d1 < c.num_docs, lane);
                }
            }
        }
        int nx = 0;
        if (lane == 0) nx = atomicAdd(&s_next, 1);
        k = __shfl_sync(0xffffffffu, nx, 0);
    }
}

// Histogram of the top 12 bits of the positive S values of (query, slice),
// and the number of positive docs per query.
__global__ void __launch_bounds__(kBPreThreads) bound_hist_kernel(const float* __restrict__ S, int64_t M,
                                                                  uint32_t* __restrict__ hist,
                                                                  uint32_t* __restrict__ npos) {
    __shared__ uint32_t h[4096];
    __shared__ uint32_t s_cnt;
    const int q = blockIdx.y;
    for (int i = threadIdx.x; i < 4096; i += blockDim.x) h[i] = 0;
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    const int64_t per = (M + gridDim.x - 1) / gridDim.x;
    const int64_t i0 = blockIdx.x * per, i1 = min(M, i0 + per);
    const float* qs = S + (size_t)q * M;
    uint32_t cnt = 0;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += kBUnroll * (int64_t)blockDim.x) {
        float v[kBUnroll];
#pragma unroll
        for (int u = 0; u < kBUnroll; ++u) {
            const int64_t j = i + u * (int64_t)blockDim.x;
            v[u] = j < i1 ? qs[j] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kBUnroll; ++u)
            if (v[u] > 0.0f) {
                atomicAdd(&h[__float_as_uint(v[u]) >> 20], 1u);
                ++cnt;
            }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
    if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(&s_cnt, cnt);
    __syncthreads();
    uint32_t* out = hist + ((size_t)q * gridDim.x + blockIdx.x) * 4096;
    for (int i = threadIdx.x; i < 4096; i += blockDim.x) out[i] = h[i];
    if (threadIdx.x == 0 && s_cnt) atomicAdd(npos + q, s_cnt);
}

// Exclusive scan over one value per thread (blockDim 1024), in thread order.
__device__ uint32_t b_scan_excl(uint32_t v, uint32_t* s_warp, uint32_t* total) {
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

// Per query: the highest bucket d whose keys at or above it number at least
// `want` (kBNoPivot when the positive docs number at most `want`).
__global__ void __launch_bounds__(1024) bound_pivot_kernel(const uint32_t* __restrict__ hist, int slices,
                                                           const uint32_t* __restrict__ npos, int want,
                                                           uint32_t* __restrict__ pivot, uint32_t* __restrict__ ccnt,
                                                           const uint32_t* __restrict__ active) {
    __shared__ uint32_t s_warp[33];
    const int q = blockIdx.x;
    if (b_inactive(active, q)) return;
    if (threadIdx.x == 0) {
        pivot[q] = kBNoPivot;
        ccnt[q] = 0;
    }
    if ((int64_t)npos[q] <= want) return;
    const int top = 4095 - 4 * threadIdx.x;
    uint32_t cnt[4] = {0, 0, 0, 0};
    for (int sl = 0; sl < slices; ++sl) {
        const uint32_t* hs = hist + ((size_t)q * slices + sl) * 4096;
#pragma unroll
        for (int j = 0; j < 4; ++j) cnt[j] += hs[top - j];
    }
    const uint32_t mine = cnt[0] + cnt[1] + cnt[2] + cnt[3];
    uint32_t total;
    const uint32_t before = b_scan_excl(mine, s_warp, &total);
    if ((int64_t)before < want && (int64_t)(before + mine) >= want) {
        uint32_t cum = before;
        for (int j = 0; j < 4; ++j) {
            cum += cnt[j];
            if ((int64_t)cum >= want) {
                pivot[q] = (uint32_t)(top - j);
                break;
            }
        }
    }
}

// Appends each query's keys (S << 32 | ~doc) in buckets >= pivot (every
// positive key without a pivot).
__global__ void __launch_bounds__(kBPreThreads) bound_compact_kernel(const float* __restrict__ S, int64_t M,
                                                                     const uint32_t* __restrict__ pivot,
                                                                     uint64_t* __restrict__ ckeys,
                                                                     uint32_t* __restrict__ ccnt,
                                                                     const uint32_t* __restrict__ active) {
    // Kept keys gather in shared memory (warp-aggregated shared atomics) and
    // go out in coalesced runs, one global atomic per run: a global atomic
    // per warp step, whose result the warp waits for, serialised the scan.
    constexpr int kStage = 2 * kBUnroll * kBPreThreads;  // one step adds at most kBUnroll * kBPreThreads keys
    __shared__ uint64_t s_buf[kStage];
    __shared__ uint32_t s_n, s_base;
    const int q = blockIdx.y;
    if (b_inactive(active, q)) return;
    const uint32_t d = pivot[q] == kBNoPivot ? 0u : pivot[q];
    const int64_t per = (M + gridDim.x - 1) / gridDim.x;
    const int64_t i0 = blockIdx.x * per, i1 = min(M, i0 + per);
    const float* qs = S + (size_t)q * M;
    uint64_t* out = ckeys + (size_t)q * kBPreCap;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    auto flush = [&]() {
        const uint32_t n = s_n;
        if (threadIdx.x == 0) s_base = n ? atomicAdd(ccnt + q, n) : 0u;
        __syncthreads();
        const uint32_t base = s_base;
        for (uint32_t j = threadIdx.x; j < n; j += blockDim.x)
            if (base + j < (uint32_t)kBPreCap) out[base + j] = s_buf[j];
        __syncthreads();
        if (threadIdx.x == 0) s_n = 0;
        __syncthreads();
    };
    for (int64_t b = i0; b < i1; b += kBUnroll * (int64_t)blockDim.x) {
        float v[kBUnroll];
#pragma unroll
        for (int u = 0; u < kBUnroll; ++u) {
            const int64_t i = b + u * (int64_t)blockDim.x + threadIdx.x;
            v[u] = i < i1 ? qs[i] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kBUnroll; ++u) {
            const int64_t i = b + u * (int64_t)blockDim.x + threadIdx.x;
            const uint32_t bits = __float_as_uint(v[u]);
            const bool keep = v[u] > 0.0f && (bits >> 20) >= d;
            const uint32_t m = __ballot_sync(0xffffffffu, keep);
            if (m) {
                uint32_t base = 0;
                if (lane == 0) base = atomicAdd(&s_n, (uint32_t)__popc(m));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (keep) s_buf[base + __popc(m & ((1u << lane) - 1))] = ((uint64_t)bits << 32) | (uint32_t)(~(uint32_t)i);
            }
        }
        __syncthreads();
        if (s_n > (uint32_t)(kStage - kBUnroll * kBPreThreads)) flush();  // room for the next step
    }
    flush();
}

// Bitonic sort, descending, of n (power of two) 64-bit keys in shared memory.
__device__ void b_sort_desc(uint64_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const uint64_t x = a[i], y = a[l];
                    const bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[l] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Per query: the K'+1 largest compacted keys (radix select on 12-bit digits,
// then a sort): the first K' docs are the candidates; the boundary is the
// largest S left out -- the (K'+1)-th key, or, when the compacted keys are
// exactly the top K', the lower edge of the pivot bucket (every key left
// below it is smaller).  need_fb: compaction overflow.
__global__ void __launch_bounds__(1024) bound_select_kernel(const uint64_t* __restrict__ ckeys,
                                                            const uint32_t* __restrict__ ccnt,
                                                            const uint32_t* __restrict__ pivot, int kc,
                                                            int32_t* __restrict__ cand, int32_t* __restrict__ n_cand,
                                                            float* __restrict__ boundary,
                                                            uint32_t* __restrict__ need_fb,
                                                            const uint32_t* __restrict__ active) {
    extern __shared__ uint64_t s_keys[];  // [sort_n]
    __shared__ uint32_t s_hist[4096];
    __shared__ uint32_t s_warp[33];
    __shared__ uint32_t s_cnt;
    __shared__ uint64_t s_prefix, s_pmask;
    __shared__ int s_need, s_done;
    const int q = blockIdx.x;
    if (b_inactive(active, q)) return;
    const uint32_t cc = ccnt[q];
    if (cc > (uint32_t)kBPreCap) {
        if (threadIdx.x == 0) {
            need_fb[q] = 1u;
            n_cand[q] = 0;
        }
        return;
    }
    const uint64_t* qk = ckeys + (size_t)q * kBPreCap;
    const int n = (int)cc;
    const int want = min(kc + 1, n);
    if (threadIdx.x == 0) { s_cnt = 0; s_prefix = 0; s_pmask = 0; s_need = want; s_done = 0; }
    __syncthreads();
    if (n <= want) {
        for (int i = threadIdx.x; i < n; i += blockDim.x) s_keys[i] = qk[i];
        if (threadIdx.x == 0) s_cnt = (uint32_t)n;
        __syncthreads();
    } else {
        const int shifts[6] = {52, 40, 28, 16, 4, 0};
        const int widths[6] = {12, 12, 12, 12, 12, 4};
        for (int lv = 0; lv < 6; ++lv) {
            if (s_done) break;
            const int sh = shifts[lv];
            const uint32_t dmask = (1u << widths[lv]) - 1;
            for (int i = threadIdx.x; i < 4096; i += blockDim.x) s_hist[i] = 0;
            __syncthreads();
            const uint64_t prefix = s_prefix, pmask = s_pmask;
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const uint64_t k = qk[i];
                if ((k & pmask) == prefix) atomicAdd(&s_hist[(k >> sh) & dmask], 1u);
            }
            __syncthreads();
            const int top = 4095 - 4 * threadIdx.x;
            uint32_t mine = 0;
            for (int j = 0; j < 4; ++j) mine += s_hist[top - j];
            uint32_t total;
            const uint32_t before = b_scan_excl(mine, s_warp, &total);
            const int need = s_need;
            if ((int)before < need && need <= (int)(before + mine)) {
                uint32_t cum = before;
                for (int j = 0; j < 4; ++j) {
                    const uint32_t h = s_hist[top - j];
                    if ((int)(cum + h) >= need) {
                        const uint32_t dg = (uint32_t)(top - j);
                        s_prefix = prefix | ((uint64_t)dg << sh);
                        s_pmask = pmask | ((uint64_t)dmask << sh);
                        s_need = need - (int)cum;
                        if ((int)h == need - (int)cum) s_done = 1;
                        break;
                    }
                    cum += h;
                }
            }
            __syncthreads();
        }
        const uint64_t prefix = s_prefix, pmask = s_pmask;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint64_t k = qk[i];
            if ((k & pmask) >= prefix) {
                const uint32_t at = atomicAdd(&s_cnt, 1u);
                if (at < (uint32_t)want) s_keys[at] = k;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) s_cnt = (uint32_t)want;  // keys are distinct: exactly `want` pass
        __syncthreads();
    }
    const int cnt = (int)s_cnt;
    int sort_n = 1;
    while (sort_n < cnt) sort_n <<= 1;
    for (int i = cnt + threadIdx.x; i < sort_n; i += blockDim.x) s_keys[i] = 0;
    __syncthreads();
    b_sort_desc(s_keys, sort_n);
    const int nc = min(cnt, kc);
    for (int i = threadIdx.x; i < nc; i += blockDim.x) cand[(size_t)q * kc + i] = (int32_t)(~(uint32_t)s_keys[i]);
    if (threadIdx.x == 0) {
        n_cand[q] = nc;
        float b = 0.0f;
        if (cnt > kc) b = __uint_as_float((uint32_t)(s_keys[kc] >> 32));
        else if (pivot[q] != kBNoPivot) b = __uint_as_float(pivot[q] << 20);
        boundary[q] = b;
    }
}

struct ExactCtx {
    const int64_t* doc_ptrs;
    const uint8_t* codes_tok;
    const float* factor_tok;
    const uint32_t* tok_cluster;
    int64_t n_clusters;
    const float* lut;        // [nq][32][512]
    const float* cb1;        // [nq][32]
    const uint32_t* labels;  // [nq][32][nprobe]
    int nprobe;
    const int32_t* cand;     // [nq][kc]
    const int32_t* n_cand;   // [nq]
    int kc;
    uint64_t* keys;          // [nq][kc] (P << 32 | ~doc)
    const uint32_t* active;  // [nq] nonzero: run this query (NULL: all)
};

__device__ __forceinline__ uint32_t map_hash(uint32_t c) { return (c * 0x9E3779B1u) >> 19; }  // 13 bits

// Exact partial scores of the candidates: one warp per doc, its tokens in
// token order; a token contributes to query token t when its cluster is one
// of t's probed lists (the probed-cluster map: cluster -> mask of t).
__global__ void __launch_bounds__(kBxWarps * 32, 1) bound_exact_kernel(ExactCtx c) {
    extern __shared__ uint8_t smem[];
    float* s_lut = reinterpret_cast<float*>(smem);                                   // [32][512]
    uint64_t* s_map = reinterpret_cast<uint64_t*>(smem + kQ * kLutPerQ * 4);         // [kMapSlots]
    uint32_t* s_m = reinterpret_cast<uint32_t*>(s_map + kMapSlots);                 // [warps][32]
    float* s_cb1 = reinterpret_cast<float*>(s_m + kBxWarps * 32);                    // [32]
    const int q = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (b_inactive(c.active, q)) return;
    const int n = c.n_cand[q];
    if ((int)blockIdx.x * kBxWarps >= n) return;
    const float4* src = reinterpret_cast<const float4*>(c.lut + (size_t)q * kQ * kLutPerQ);
    for (int i = threadIdx.x; i < kQ * kLutPerQ / 4; i += blockDim.x) reinterpret_cast<float4*>(s_lut)[i] = src[i];
    for (int i = threadIdx.x; i < kMapSlots; i += blockDim.x) s_map[i] = kMapEmpty;
    if (threadIdx.x < kQ) s_cb1[threadIdx.x] = c.cb1[q * kQ + threadIdx.x];
    __syncthreads();
    const uint32_t* lab = c.labels + (size_t)q * kQ * c.nprobe;
    for (int i = threadIdx.x; i < kQ * c.nprobe; i += blockDim.x) {
        const uint32_t cl = lab[i];
        if ((int64_t)cl >= c.n_clusters) continue;
        const uint32_t tbit = 1u << (i / c.nprobe);
        uint32_t h = map_hash(cl);
        for (int probe = 0; probe < kMapSlots; ++probe, h = (h + 1) & (kMapSlots - 1)) {
            unsigned long long cur = s_map[h];
            if (cur == kMapEmpty) {
                cur = atomicCAS(reinterpret_cast<unsigned long long*>(&s_map[h]), kMapEmpty,
                                ((uint64_t)cl << 32) | tbit);
                if (cur == kMapEmpty) break;
            }
            if ((uint32_t)(cur >> 32) == cl) {
                atomicOr(reinterpret_cast<unsigned long long*>(&s_map[h]), (unsigned long long)tbit);
                break;
            }
        }
    }
    __syncthreads();
    const uint4* codes = reinterpret_cast<const uint4*>(c.codes_tok);
    uint32_t* m = s_m + warp * 32;
    auto map_mask = [&](uint32_t cl) {
        uint32_t h = map_hash(cl);
        for (int probe = 0; probe < kMapSlots; ++probe, h = (h + 1) & (kMapSlots - 1)) {
            const uint64_t e = s_map[h];
            if (e == kMapEmpty) return 0u;
            if ((uint32_t)(e >> 32) == cl) return (uint32_t)e;
        }
        return 0u;
    };
    auto post = [&](uint32_t mask, uint4 code, float f) {
        for (; mask; mask &= mask - 1) {
            const int t = __ffs(mask) - 1;
            const float dist = fmul(fsub(lut_ip_prmt(s_lut + t * kLutPerQ, code), s_cb1[t]), f);
            if (dist > 0.0f) atomicMax(m + t, __float_as_uint(dist));
        }
    };
    // the next doc's token range is loaded while the current one is scored
    int i = blockIdx.x * kBxWarps + warp;
    int32_t doc = i < n ? c.cand[(size_t)q * c.kc + i] : 0;
    int64_t t0 = i < n ? c.doc_ptrs[doc] : 0, t1 = i < n ? c.doc_ptrs[doc + 1] : 0;
    for (; i < n; i += gridDim.x * kBxWarps) {
        const int inext = i + gridDim.x * kBxWarps;
        int32_t dnext = 0;
        int64_t n0 = 0, n1 = 0;
        if (inext < n) {
            dnext = c.cand[(size_t)q * c.kc + inext];
            n0 = c.doc_ptrs[dnext];
            n1 = c.doc_ptrs[dnext + 1];
        }
        m[lane] = 0u;
        __syncwarp();
        // 64 tokens per step, two per lane: clusters, codes and factors all in
        // flight before the map lookups
        for (int64_t base = t0; base < t1; base += 64) {
            const int64_t ta = base + lane, tb = base + 32 + lane;
            const bool va = ta < t1, vb = tb < t1;
            uint32_t ca = 0xFFFFFFFFu, cb = 0xFFFFFFFFu;
            uint4 ka = make_uint4(0, 0, 0, 0), kb = make_uint4(0, 0, 0, 0);
            float fa = 0.0f, fb = 0.0f;
            if (va) { ca = __ldg(c.tok_cluster + ta); ka = __ldg(codes + ta); fa = __ldg(c.factor_tok + ta); }
            if (vb) { cb = __ldg(c.tok_cluster + tb); kb = __ldg(codes + tb); fb = __ldg(c.factor_tok + tb); }
            const uint32_t ma = va && (int64_t)ca < c.n_clusters ? map_mask(ca) : 0u;
            const uint32_t mb = vb && (int64_t)cb < c.n_clusters ? map_mask(cb) : 0u;
            post(ma, ka, fa);
            post(mb, kb, fb);
        }
        __syncwarp();
        // sum_partial_scores_kernel's tree over the 32 per-token maxima (kernels.cu:192-198)
        float x = __uint_as_float(m[lane]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off));
        if (lane == 0) c.keys[(size_t)q * c.kc + i] = ((uint64_t)__float_as_uint(x) << 32) | (uint32_t)(~(uint32_t)doc);
        __syncwarp();
        doc = dnext;
        t0 = n0;
        t1 = n1;
    }
}

// Per query: the candidates by (P desc, doc asc); the refined list when the
// boundary proves that no doc left out can reach it, else need_fb (and
// retry[q] = 1 when a larger candidate set could still prove it).
__global__ void __launch_bounds__(1024) bound_final_kernel(const uint64_t* __restrict__ keys,
                                                           const int32_t* __restrict__ n_cand, int kc,
                                                           const uint32_t* __restrict__ npos,
                                                           const float* __restrict__ boundary, double eps,
                                                           int k_refine, int32_t* __restrict__ refined_docs,
                                                           float* __restrict__ refined_partial,
                                                           int32_t* __restrict__ num_refined,
                                                           uint32_t* __restrict__ need_fb,
                                                           const uint32_t* __restrict__ active,
                                                           uint32_t* __restrict__ retry) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int s_ok;
    const int q = blockIdx.x;
    if (b_inactive(active, q)) return;
    // round 1: a compaction overflow (flagged by the select kernel) stands
    if (active == nullptr && need_fb[q]) return;
    // fewer positive docs than k_refine: the zero-score fill needs the visited
    // docs (the hash-table path's bitmap)
    const int n = n_cand[q];
    if ((int64_t)npos[q] < k_refine || n < k_refine) {  // n < k_refine: a round-2 overflow
        if (threadIdx.x == 0) need_fb[q] = 1u;
        return;
    }
    int sort_n = 1;
    while (sort_n < n) sort_n <<= 1;
    for (int i = threadIdx.x; i < sort_n; i += blockDim.x) s_keys[i] = i < n ? keys[(size_t)q * kc + i] : 0ull;
    __syncthreads();
    b_sort_desc(s_keys, sort_n);
    if (threadIdx.x == 0) {
        const float tau = __uint_as_float((uint32_t)(s_keys[k_refine - 1] >> 32));
        const float b = boundary[q];
        s_ok = (b == 0.0f || (double)b * (1.0 + eps) < (double)tau) ? 1 : 0;
        if (!s_ok) {
            need_fb[q] = 1u;
            if (retry) retry[q] = 1u;
        } else {
            need_fb[q] = 0u;  // round 2 starts from a flagged query
            num_refined[q] = k_refine;
        }
    }
    __syncthreads();
    if (!s_ok) return;
    for (int i = threadIdx.x; i < k_refine; i += blockDim.x) {
        const uint64_t k = s_keys[i];
        refined_docs[(size_t)q * k_refine + i] = (int32_t)(~(uint32_t)k);
        refined_partial[(size_t)q * k_refine + i] = __uint_as_float((uint32_t)(k >> 32));
    }
}

// ---- host side -------------------------------------------------------------
// The probed-cluster map holds 32 x nprobe clusters at most half full.
constexpr int kBMaxNprobe = kMapSlots / (2 * kQ);

// k_refine above the doc count leaves every query with fewer positive docs
// than k_refine (the hash-table path's zero-score fill), so the pass is skipped.
bool bound_enabled(const chm_index* idx, int nprobe, int k_refine) {
    return idx->tok_cluster && idx->codes1_tok && idx->factor1_tok && idx->max_doc_len > 0 &&
           idx->num_docs > 0 && nprobe > 0 && nprobe <= kBMaxNprobe && k_refine > 0 &&
           k_refine <= CHM_MAX_K_REFINE && (int64_t)k_refine <= idx->num_docs;
}

int bound_kc(const chm_index* idx, int k_refine) {
    int64_t kc = (int64_t)k_refine + std::max(k_refine / 2, 64);
    kc = std::min<int64_t>(kc, kBMaxCand);
    kc = std::min<int64_t>(kc, idx->num_docs);
    return (int)std::max<int64_t>(kc, k_refine);
}
// The second round's candidate count.
int bound_kc2(const chm_index* idx) { return (int)std::min<int64_t>(kBMaxCand, idx->num_docs); }

constexpr int kBPreSlots = 640;
int bound_slices(int nq) { return std::max(1, std::min(64, kBPreSlots / std::max(1, nq))); }

struct BoundWork {
    float* S;
    uint32_t* hist;
    uint32_t* npos;
    uint32_t* pivot;
    uint32_t* ccnt;
    uint64_t* ckeys;
    int32_t* cand;
    int32_t* n_cand;
    float* boundary;
    uint64_t* keys;
    uint32_t* retry;
};

template <typename A>
void bound_layout(A& a, const chm_index* idx, int nq, int k_refine, BoundWork* w) {
    // room for either round's candidates
    const int kc = std::max(bound_kc(idx, k_refine), bound_kc2(idx));
    auto S = a.template take<float>((size_t)nq * idx->num_docs);
    auto hist = a.template take<uint32_t>((size_t)std::max(nq, kBPreSlots) * 4096);
    auto npos = a.template take<uint32_t>((size_t)nq);
    auto pivot = a.template take<uint32_t>((size_t)nq);
    auto ccnt = a.template take<uint32_t>((size_t)nq);
    auto ckeys = a.template take<uint64_t>((size_t)nq * kBPreCap);
    auto cand = a.template take<int32_t>((size_t)nq * kc);
    auto n_cand = a.template take<int32_t>((size_t)nq);
    auto boundary = a.template take<float>((size_t)nq);
    auto keys = a.template take<uint64_t>((size_t)nq * kc);
    auto retry = a.template take<uint32_t>((size_t)nq);
    if (w)
        *w = BoundWork{(float*)S, (uint32_t*)hist, (uint32_t*)npos, (uint32_t*)pivot, (uint32_t*)ccnt,
                       (uint64_t*)ckeys, (int32_t*)cand, (int32_t*)n_cand, (float*)boundary, (uint64_t*)keys,
                       (uint32_t*)retry};
}

struct BoundSizer {
    Sizer s;
    template <typename T>
    void* take(size_t n) {
        s.take<T>(n);
        return nullptr;
    }
};

size_t bound_bytes(const chm_index* idx, int nq, int nprobe, int k_refine) {
    if (!bound_enabled(idx, nprobe, k_refine)) return 0;
    BoundSizer s;
    bound_layout(s, idx, nq, k_refine, nullptr);
    return s.s.off;
}

// SMs of the current device (148 on B200 when none is visible).
static int bound_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                   cudaSuccess || sms <= 0) {
        (void)cudaGetLastError();
        return 148;
    }
    return sms;
}

// The dense-bound pass over `nq` queries.  need_fb[q] = 1 marks the queries
// the hash-table path must redo; the others have their refined list written.
chm_status bound_run(const chm_index* idx, int nq, const float* lut, const float* cb1, const uint32_t* labels,
                     int nprobe, int k_refine, int32_t* refined_docs, float* refined_partial, int32_t* num_refined,
                     uint32_t* need_fb, void* ws, size_t ws_bytes, cudaStream_t st) {
    Arena a(ws, ws_bytes);
    BoundWork w;
    bound_layout(a, idx, nq, k_refine, &w);
    if (a.overflow) return CHM_ERR_CAPACITY;
    const int kc = bound_kc(idx, k_refine);
    const int64_t M = idx->num_docs;
    CHM_CUDA(cudaMemsetAsync(w.S, 0, sizeof(float) * (size_t)nq * M, st));
    CHM_CUDA(cudaMemsetAsync(w.npos, 0, sizeof(uint32_t) * nq, st));
    CHM_CUDA(cudaMemsetAsync(need_fb, 0, sizeof(uint32_t) * nq, st));
    BoundCtx c{idx->cluster_pos, idx->codes1, idx->factor1, idx->doc_ids, idx->n_clusters, M, lut, cb1,
               labels, nprobe, w.S};
    // about eight resident waves of score CTAs over the batch
    int splits = (int)std::max<int64_t>(1, std::min<int64_t>(8, (int64_t)148 * 8 * 8 / std::max(1, kQ * nq)));
    splits = std::min(splits, std::max(1, nprobe / kBsWarps));
    bound_score_kernel<<<dim3((unsigned)(kQ * splits), (unsigned)nq), kBsWarps * 32, 0, st>>>(c, splits);
    CHM_TRY(launch_status("bound_score_kernel"));
    const int slices = bound_slices(nq);
    bound_hist_kernel<<<dim3((unsigned)slices, (unsigned)nq), kBPreThreads, 0, st>>>(w.S, M, w.hist, w.npos);
    CHM_TRY(launch_status("bound_hist_kernel"));
    CHM_CUDA(cudaMemsetAsync(w.retry, 0, sizeof(uint32_t) * nq, st));
    const double eps = ((double)idx->max_doc_len * kQ + 8.0) * 0x1p-24 * 1.25;
    const int kc2 = bound_kc2(idx);
    // round 1 over every query with K' = kc; round 2 over the queries whose
    // boundary round 1 could not prove, with K' = kc2
    for (int round = 0; round < 2; ++round) {
        const int k = round == 0 ? kc : kc2;
        const uint32_t* active = round == 0 ? nullptr : w.retry;
        if (round == 1 && kc2 <= kc) break;
        bound_pivot_kernel<<<nq, 1024, 0, st>>>(w.hist, slices, w.npos, k, w.pivot, w.ccnt, active);
        CHM_TRY(launch_status("bound_pivot_kernel"));
        bound_compact_kernel<<<dim3((unsigned)slices, (unsigned)nq), kBPreThreads, 0, st>>>(w.S, M, w.pivot,
                                                                                           w.ckeys, w.ccnt, active);
        CHM_TRY(launch_status("bound_compact_kernel"));
        int sort_cap = 1;
        while (sort_cap < k + 1) sort_cap <<= 1;
        const size_t sel_smem = sizeof(uint64_t) * sort_cap;
        CHM_CUDA(cudaFuncSetAttribute(bound_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sel_smem));
        bound_select_kernel<<<nq, 1024, sel_smem, st>>>(w.ckeys, w.ccnt, w.pivot, k, w.cand, w.n_cand, w.boundary,
                                                        need_fb, active);
        CHM_TRY(launch_status("bound_select_kernel"));
        ExactCtx x{idx->doc_ptrs, idx->codes1_tok, idx->factor1_tok, idx->tok_cluster, idx->n_clusters, lut, cb1,
                   labels, nprobe, w.cand, w.n_cand, k, w.keys, active};
        const size_t ex_smem = (size_t)kQ * kLutPerQ * 4 + (size_t)kMapSlots * 8 + kBxWarps * 32 * 4 + kQ * 4;
        CHM_CUDA(cudaFuncSetAttribute(bound_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)ex_smem));
        // One resident CTA per SM.  The CTAs per query (gx) minimise the
        // waves times a CTA's time, setup (the LUTs and the cluster map, about
        // 0.4% of one query's work) plus 1/gx of the query's candidates: at 128
        // queries gx = 8 fills 6.9 waves of 148 (gx = 3 left 40% of the SMs idle
        // in its third wave).
        const int sms = bound_sms();
        const int gmax = (int)std::max<int64_t>(1, std::min<int64_t>(1024, (k + kBxWarps - 1) / kBxWarps));
        int gx = 1;
        double best = 1e300;
        for (int g = 1; g <= gmax; ++g) {
            const double waves = (double)(((int64_t)nq * g + sms - 1) / sms);
            const double cost = waves * (0.004 + 1.0 / g);
            if (cost < best - 1e-9) {
                best = cost;
                gx = g;
            }
        }
        bound_exact_kernel<<<dim3((unsigned)gx, (unsigned)nq), kBxWarps * 32, ex_smem, st>>>(x);
        CHM_TRY(launch_status("bound_exact_kernel"));
        int fsort = 1;
        while (fsort < k) fsort <<= 1;
        const size_t fin_smem = sizeof(uint64_t) * fsort;
        CHM_CUDA(cudaFuncSetAttribute(bound_final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)fin_smem));
        bound_final_kernel<<<nq, 1024, fin_smem, st>>>(w.keys, w.n_cand, k, w.npos, w.boundary, eps, k_refine,
                                                       refined_docs, refined_partial, num_refined, need_fb, active,
                                                       round == 0 ? w.retry : nullptr);
        CHM_TRY(launch_status("bound_final_kernel"));
    }
    return CHM_OK;
}

}  // namespace chm
