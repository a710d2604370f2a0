// Tensor-core (tcgen05 / TMEM / TMA) distance GEMM for the centroid probe
// and the build-time assignment, with exact fp32 re-ranking.
//
// Contract (same as the SIMT path in probe.cu): dist(q, c) = ||c||^2 - 2<q, c>
// with <q, c> a sequential fp32 fma chain; top-k by (dist, id).  The bf16
// tensor-core pass only proposes candidates:
//   1. threshold : tensor-core dists to a prefix of the centroids, exact
//                  radix select of a small order statistic per row -> tau_row,
//                  chosen so that about 4 K' centroids pass the filter below
//                  (fewer than K' + 1: the row takes the exact path);
//   2. filter    : tensor-core dists to every centroid, rows keep the
//                  (dist, id) pairs with dist <= tau_row (per-split buffers);
//   3. re-rank   : the K' best survivors get exact fp32 dists; the row is
//                  accepted only when its k-th exact dist is below the
//                  smallest approximate dist left out minus the bf16 error
//                  bound E, which proves no excluded centroid can enter.
//                  Rows that fail (or overflow a buffer) are recomputed
//                  exactly over all centroids.
// The assignment keeps the 16 best approximate centroids per row and
// epilogue group in registers instead of a threshold, with the same
// certificate over the 32 candidates.
//
// GEMM kernel: one CTA = 128 query rows x a range of 128-centroid tiles.
// One warp issues TMA loads (A once, B through a 4-stage ring), one
// owns TMEM and issues tcgen05.mma (M=128, N=128, K=16 x 8) into one TMEM
// accumulator per epilogue group, and the epilogue groups (four warps each,
// warps 0 .. 4 G - 1, so that warp % 4 is the TMEM lane quarter) drain the
// accumulators in turn with tcgen05.ld.  Every TMA load goes to the issuing
// CTA alone (no cluster-wide delivery).
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "select.cuh"
#include "sm100.cuh"

namespace chm {

constexpr int kTM = 128, kTN = 128, kK = 128;
constexpr int kBoxBytes = 128 * 64 * 2;             // one 128 x 64 bf16 TMA box
constexpr int kTileBytes = 2 * kBoxBytes;           // 128 x 128 bf16
constexpr int kTopA = 16;                           // assignment candidates per row
constexpr int kFallbackRows = 16;                   // rows recomputed exactly at a time, past the batch
constexpr int kFallbackBatch = 64;                  // probe rows recomputed exactly in one GEMM pass
constexpr int kMaxSplits = 296;                     // centroid-range splits per row tile
constexpr uint32_t kIdesc = sm100::idesc_bf16_f32(kTM, kTN);

enum TcMode { kStore = 0, kFilter = 1, kTop16 = 2 };

struct TcArgs {
    int64_t rows, cols;
    const float* cn;          // exact ||c||^2
    int tiles_per_split;
    int splits;
    float* dist;              // kStore: [rows x ld]
    int64_t ld;
    const float* tau;         // kFilter: per-row threshold
    uint64_t* surv;           // kFilter: [rows][splits][cap]
    int32_t* surv_cnt;        // kFilter: [rows][splits]
    int cap;
    uint64_t* top;            // kTop16: [rows][splits][2 epilogue groups][16]
    uint32_t* err;
};

// Epilogue groups per mode: the filter and store passes drain with three
// groups (12 epilogue warps, three TMEM accumulators of 128 columns), so that
// three warps per scheduler hide the TMEM-load and shared-load latency; the
// top-16 pass keeps two (its 16 running keys per row need the registers).
// Warps are spread over the four schedulers round-robin, and each scheduler
// holds a quarter of the register file (16,384 registers): with 14 warps
// (at most 4 per scheduler) a thread may use 128.
template <int MODE>
struct TcCfg {
    static constexpr int kGroups = MODE == kTop16 ? 2 : 3;
    static constexpr int kEpiWarps = 4 * kGroups;
    static constexpr int kTmaWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1;
    static constexpr int kThreads = (kEpiWarps + 2) * 32;
    static constexpr int kStages = 4;
    static constexpr uint32_t kTmemCols = kGroups <= 2 ? 256u : 512u;  // a power of two >= kGroups * 128
    static constexpr int kMaxRegs = (16384 / ((kEpiWarps + 2 + 3) / 4 * 32)) / 8 * 8;
};

template <int MODE>
struct TcSmem {
    using C = TcCfg<MODE>;
    alignas(1024) uint8_t a[kTileBytes];
    alignas(1024) uint8_t b[C::kStages][kTileBytes];
    uint64_t full[C::kStages], empty[C::kStages], acc_full[C::kGroups], acc_empty[C::kGroups], a_full, mma_done;
    uint32_t tmem_base;
    alignas(16) float cn[C::kEpiWarps][kTN];  // per epilogue warp: ||c||^2 of its current tile
    float pass[C::kEpiWarps][32][33];         // per lane: 32 values of a group with set mask bits
    int rowcnt[kTM];                          // filter: survivors appended per row (all groups)
};

__device__ __forceinline__ uint64_t dist_key(float d, uint32_t col) {
    return ((uint64_t)float_key_asc(d) << 32) | col;
}

// this lane's 4 norms of tile `tile` (columns 4 lane .. 4 lane + 3); +inf past the end
__device__ __forceinline__ float4 tile_norms4(const float* __restrict__ cn, int64_t cols, int tile, int lane) {
    const int64_t c = (int64_t)tile * kTN + 4 * lane;
    float4 v;
    v.x = c + 0 < cols ? __ldg(cn + c + 0) : INFINITY;
    v.y = c + 1 < cols ? __ldg(cn + c + 1) : INFINITY;
    v.z = c + 2 < cols ? __ldg(cn + c + 2) : INFINITY;
    v.w = c + 3 < cols ? __ldg(cn + c + 3) : INFINITY;
    return v;
}

template <int MODE>
__global__ void __maxnreg__(TcCfg<MODE>::kMaxRegs) tc_dist_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                         const __grid_constant__ CUtensorMap tmB,
                                                                         TcArgs p) {
    using C = TcCfg<MODE>;
    constexpr int NG = C::kGroups, NS = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    TcSmem<MODE>& s =
        *reinterpret_cast<TcSmem<MODE>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.y * kTM;
    const int n_tiles_total = (int)((p.cols + kTN - 1) / kTN);
    const int t_begin = blockIdx.x * p.tiles_per_split;
    const int t_end = min(n_tiles_total, t_begin + p.tiles_per_split);
    const int n_tiles = max(0, t_end - t_begin);

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            sm100::mbar_init(&s.full[i], 1);
            sm100::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < NG; ++i) {
            sm100::mbar_init(&s.acc_full[i], 1);
            sm100::mbar_init(&s.acc_empty[i], 128);
        }
        sm100::mbar_init(&s.a_full, 1);
        sm100::mbar_init(&s.mma_done, 1);
        sm100::fence_mbar_init();
    }
    if (warp == C::kMmaWarp) {
        sm100::tmem_alloc(&s.tmem_base, C::kTmemCols);
        sm100::tmem_relinquish();
    }
    if (threadIdx.x < kTM) s.rowcnt[threadIdx.x] = 0;
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = s.tmem_base;
    bool failed = false;

    if (warp == C::kTmaWarp) {
        if (lane == 0) {
            // ---- TMA producer ----
            sm100::prefetch_tmap(&tmA);
            sm100::prefetch_tmap(&tmB);
            sm100::mbar_expect_tx(&s.a_full, kTileBytes);
            sm100::tma_load_2d(s.a, &tmA, 0, (int)row0, &s.a_full);
            sm100::tma_load_2d(s.a + kBoxBytes, &tmA, 64, (int)row0, &s.a_full);
            for (int it = 0; it < n_tiles; ++it) {
                const int st = it % NS;
                const uint32_t round = it / NS;
                if (!sm100::mbar_wait(&s.empty[st], (round & 1) ^ 1)) { failed = true; break; }
                const int n0 = (t_begin + it) * kTN;
                sm100::mbar_expect_tx(&s.full[st], kTileBytes);
                sm100::tma_load_2d(s.b[st], &tmB, 0, n0, &s.full[st]);
                sm100::tma_load_2d(s.b[st] + kBoxBytes, &tmB, 64, n0, &s.full[st]);
            }
            // drain: every issued load has landed before the CTA may exit
            const int issued = failed ? 0 : n_tiles;
            for (int it = max(0, issued - NS); it < issued; ++it)
                if (!sm100::mbar_wait(&s.full[it % NS], (it / NS) & 1)) failed = true;
            if (!sm100::mbar_wait(&s.a_full, 0)) failed = true;
        }
    } else if (warp == C::kMmaWarp) {
        if (lane == 0) {
            // ---- MMA issuer: tile `it` into accumulator it % NG ----
            bool ok = sm100::mbar_wait(&s.a_full, 0);
            const uint32_t a_base = sm100::smem_addr(s.a);
            for (int it = 0; ok && it < n_tiles; ++it) {
                const int st = it % NS;
                const int buf = it % NG;
                if (!sm100::mbar_wait(&s.acc_empty[buf], ((it / NG) & 1) ^ 1)) { ok = false; break; }
                if (!sm100::mbar_wait(&s.full[st], (it / NS) & 1)) { ok = false; break; }
                sm100::tc_fence_after();
                const uint32_t b_base = sm100::smem_addr(s.b[st]);
                const uint32_t d_tmem = tmem + buf * kTN;
#pragma unroll
                for (int kk = 0; kk < kK / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                    sm100::mma_bf16(d_tmem, sm100::smem_desc_sw128(a_base + off),
                                    sm100::smem_desc_sw128(b_base + off), kIdesc, kk > 0 ? 1u : 0u);
                }
                sm100::mma_commit(&s.empty[st]);
                sm100::mma_commit(&s.acc_full[buf]);
            }
            failed = !ok;
            // all issued MMAs complete before TMEM is released
            sm100::mma_commit(&s.mma_done);
            if (!sm100::mbar_wait(&s.mma_done, 0)) failed = true;
        }
    } else {
        // ---- epilogue: TMEM -> registers -> filter / store / top-16 ----
        // group g drains the tiles it = g, g + NG, ... from accumulator g, so
        // the groups run side by side (top-16: each group keeps its own 16)
        const int g = warp >> 2;
        const int q4 = warp & 3;        // TMEM lane quarter: warp % 4
        const int rl = q4 * 32 + lane;  // row within the tile
        const int64_t row = row0 + rl;
        const bool vrow = row < p.rows;
        float tau = -INFINITY;
        if (MODE == kFilter && vrow) tau = p.tau[row];
        uint64_t best[kTopA];
        if (MODE == kTop16) {
#pragma unroll
            for (int j = 0; j < kTopA; ++j) best[j] = ~0ull;
        }
        float thr = INFINITY;  // kTop16: float of best[15]
        float* row_vals = s.pass[warp][lane];
        float* cnw = s.cn[warp];
        // this lane's share of the warp's next tile norms, loaded one tile ahead
        float4 cn_next = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
        if (g < n_tiles) cn_next = tile_norms4(p.cn, p.cols, t_begin + g, lane);
        for (int it = g; it < n_tiles; it += NG) {
            const int buf = it % NG;
            const int64_t n0 = (int64_t)(t_begin + it) * kTN;
            // stage this tile's norms in the warp's own buffer (warp-synchronous)
            __syncwarp();
            *reinterpret_cast<float4*>(cnw + 4 * lane) = cn_next;
            __syncwarp();
            if (it + NG < n_tiles) cn_next = tile_norms4(p.cn, p.cols, t_begin + it + NG, lane);
            if (failed) continue;
            // warp-uniform wait: the tcgen05.ld below needs every lane
            const bool ok = __all_sync(0xffffffffu, sm100::mbar_wait(&s.acc_full[buf], (it / NG) & 1));
            if (!ok) { failed = true; continue; }
            sm100::tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(q4 * 32) << 16) + buf * kTN;
            // two halves of 64 columns (one TMEM-load wait each) keep 64
            // accumulators in registers at a time
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                uint32_t r2[2][32];
                sm100::tmem_ld32_async(tbase + h * 64, r2[0]);
                sm100::tmem_ld32_async(tbase + h * 64 + 32, r2[1]);
                sm100::tmem_wait_ld();
                if (h == 1) {
                    // the accumulator is in registers: hand TMEM back to the MMA warp
                    sm100::tc_fence_before();
                    sm100::mbar_arrive(&s.acc_empty[buf]);
                }
                if (!vrow) continue;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int c = 2 * h + cc;
                    const uint32_t* r = r2[cc];
                    const float* cnb = cnw + c * 32;
                    if (MODE == kStore) {
                        float* out = p.dist + row * p.ld + n0 + c * 32;
                        if (n0 + c * 32 + 32 <= p.cols && (p.ld & 3) == 0) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4) {
                                float4 o;
                                o.x = __fmaf_rn(-2.0f, __uint_as_float(r[j + 0]), cnb[j + 0]);
                                o.y = __fmaf_rn(-2.0f, __uint_as_float(r[j + 1]), cnb[j + 1]);
                                o.z = __fmaf_rn(-2.0f, __uint_as_float(r[j + 2]), cnb[j + 2]);
                                o.w = __fmaf_rn(-2.0f, __uint_as_float(r[j + 3]), cnb[j + 3]);
                                *reinterpret_cast<float4*>(out + j) = o;
                            }
                        } else {
                            for (int j = 0; j < 32; ++j)
                                if (n0 + c * 32 + j < p.cols) out[j] = __fmaf_rn(-2.0f, __uint_as_float(r[j]), cnb[j]);
                        }
                    } else {
                        // Column j can enter when d <= tau (filter) or d <= the
                        // current 16th best (top-16).  d = cn - 2 v is exact in
                        // one fma because 2 v is exact.  Out-of-range columns
                        // carry +inf norms and never pass.  Most groups of 32
                        // have no such column: the fast pass takes their minimum
                        // in four independent chains (norms four at a time), and
                        // only a passing group builds its mask.
                        const float lim = (MODE == kFilter) ? tau : thr;
                        const float4* cn4 = reinterpret_cast<const float4*>(cnb);
                        float m0 = INFINITY, m1 = INFINITY, m2 = INFINITY, m3 = INFINITY;
#pragma unroll
                        for (int j4 = 0; j4 < 8; ++j4) {
                            const float4 n4 = cn4[j4];
                            m0 = fminf(m0, __fmaf_rn(-2.0f, __uint_as_float(r[4 * j4 + 0]), n4.x));
                            m1 = fminf(m1, __fmaf_rn(-2.0f, __uint_as_float(r[4 * j4 + 1]), n4.y));
                            m2 = fminf(m2, __fmaf_rn(-2.0f, __uint_as_float(r[4 * j4 + 2]), n4.z));
                            m3 = fminf(m3, __fmaf_rn(-2.0f, __uint_as_float(r[4 * j4 + 3]), n4.w));
                        }
                        uint32_t mask = 0;
                        if (fminf(fminf(m0, m1), fminf(m2, m3)) <= lim) {
                            uint32_t mk[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                const float d = __fmaf_rn(-2.0f, __uint_as_float(r[j]), cnb[j]);
                                mk[j & 3] |= (d <= lim ? 1u : 0u) << j;
                            }
                            mask = (mk[0] | mk[1]) | (mk[2] | mk[3]);
                        }
                        if (mask) {
                            // rare: copy the 32 values to this lane's shared row and
                            // walk the set bits with a runtime index (keeps the hot
                            // loop small and r[] in registers)
#pragma unroll
                            for (int j = 0; j < 32; ++j) row_vals[j] = __uint_as_float(r[j]);
                            while (mask) {
                                const int j = __ffs(mask) - 1;
                                mask &= mask - 1;
                                const float d = __fmaf_rn(-2.0f, row_vals[j], cnb[j]);
                                const uint32_t col = (uint32_t)(n0 + c * 32 + j);
                                if (MODE == kFilter) {
                                    const int at = atomicAdd(&s.rowcnt[rl], 1);  // shared by all groups
                                    if (at < p.cap)
                                        p.surv[((size_t)row * p.splits + blockIdx.x) * p.cap + at] = dist_key(d, col);
                                } else {
                                    const uint64_t key = dist_key(d, col);
                                    if (key < best[kTopA - 1]) {
                                        best[kTopA - 1] = key;
#pragma unroll
                                        for (int q = kTopA - 1; q > 0; --q) {
                                            if (best[q] < best[q - 1]) {
                                                const uint64_t t = best[q];
                                                best[q] = best[q - 1];
                                                best[q - 1] = t;
                                            }
                                        }
                                        if (best[kTopA - 1] != ~0ull)
                                            thr = key_to_float_asc((uint32_t)(best[kTopA - 1] >> 32));
                                    }
                                }
                            }
                        }
                    }
                }
            }
        }
        if (MODE == kTop16 && vrow) {
#pragma unroll
            for (int j = 0; j < kTopA; ++j)
                p.top[(((size_t)row * p.splits + blockIdx.x) * 2 + g) * kTopA + j] = best[j];
        }
    }
    if (failed) atomicOr(p.err, 1u);
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    // filter: every group has appended; the first group's threads publish the counts
    if (MODE == kFilter && warp < 4) {
        const int rl = warp * 32 + lane;
        if (row0 + rl < p.rows) p.surv_cnt[(size_t)(row0 + rl) * p.splits + blockIdx.x] = s.rowcnt[rl];
    }
    if (warp == C::kMmaWarp) sm100::tmem_dealloc(tmem, C::kTmemCols);
}

// ---- helpers ---------------------------------------------------------------
__global__ void to_bf16_kernel(const float* __restrict__ x, int64_t n, __nv_bfloat16* __restrict__ y) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}

// Bound on |approx - exact| for dist = ||c||^2 - 2<q,c> with bf16 operands
// (relative rounding 2^-9 on each operand, fp32 accumulation) against the
// sequential fp32 chain: 2 * (2^-8 + 2^-16 + accumulation slack) * ||q|| *
// max||c|| plus fp32 slack on the subtraction.
__device__ __forceinline__ float err_bound(float qnorm, float cnmax) {
    const float cmax = sqrtf(cnmax);
    return 2.0f * (0.00390625f + 0.0000153f + 0.00025f) * 1.05f * cmax * qnorm +
           4e-6f * (cnmax + 2.0f * cmax * qnorm) + 1e-6f;
}

// Exact (sequential fma) dist of row q to centroid c.  Both rows are read
// 16 bytes at a time when both are 16-byte aligned (the fma order is the same).
__device__ __forceinline__ float exact_dist(const float* q, const float* c, float cn) {
    float acc = 0.0f;
    if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(c)) & 15u) == 0) {
        const float4* q4 = reinterpret_cast<const float4*>(q);
        const float4* c4 = reinterpret_cast<const float4*>(c);
#pragma unroll 8
        for (int k4 = 0; k4 < kDim / 4; ++k4) {
            const float4 qv = q4[k4];
            const float4 cv = __ldg(c4 + k4);
            acc = __fmaf_rn(qv.x, cv.x, acc);
            acc = __fmaf_rn(qv.y, cv.y, acc);
            acc = __fmaf_rn(qv.z, cv.z, acc);
            acc = __fmaf_rn(qv.w, cv.w, acc);
        }
    } else {
#pragma unroll 8
        for (int k = 0; k < kDim; ++k) acc = __fmaf_rn(q[k], c[k], acc);
    }
    return fsub(cn, fmul(2.0f, acc));
}

__device__ void bitonic_asc(uint64_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const uint64_t x = a[i], y = a[l];
                    const bool asc = (i & k) == 0;
                    if (asc ? (x > y) : (x < y)) { a[i] = y; a[l] = x; }
                }
            }
            __syncthreads();
        }
}

constexpr int kRerankThreads = 256;
constexpr int kSurvMax = 4096;  // survivors a row can hold in the re-rank sort

// Probe re-rank: one CTA per row (see the file comment for the certificate).
__global__ void __launch_bounds__(kRerankThreads) probe_rerank_kernel(
    const float* __restrict__ q_rows, const float* __restrict__ centroids, const float* __restrict__ cn,
    const uint64_t* __restrict__ surv, const int32_t* __restrict__ surv_cnt, int splits, int cap,
    const float* __restrict__ tau, int kc, int nprobe, const float* __restrict__ cnmax,
    uint32_t* __restrict__ labels, int32_t* __restrict__ fallback_list, uint32_t* __restrict__ fallback_cnt) {
    __shared__ uint64_t s_keys[kSurvMax];
    __shared__ uint64_t s_ex[512];
    __shared__ alignas(16) float s_q[kDim];
    __shared__ int s_total, s_bad;
    const int64_t row = blockIdx.x;
    // fallback_cnt[1] is the tensor-core kernels' error flag: a launch that
    // gave up on a bounded wait left tiles unscored, so every row of the call
    // takes the exact path instead
    if (fallback_cnt[1] != 0u) {
        if (threadIdx.x == 0) fallback_list[atomicAdd(fallback_cnt, 1u)] = (int32_t)row;
        return;
    }
    if (threadIdx.x == 0) { s_total = 0; s_bad = 0; }
    if (threadIdx.x < kDim) s_q[threadIdx.x] = q_rows[row * kDim + threadIdx.x];
    __syncthreads();
    // gather survivors of every split: offsets by one thread, then a flat copy
    __shared__ int s_off[kMaxSplits + 1];
    if (threadIdx.x == 0) {
        int acc = 0;
        s_off[0] = 0;
        for (int sp = 0; sp < splits; ++sp) {
            const int c = surv_cnt[(size_t)row * splits + sp];
            if (c > cap) s_bad = 1;
            acc += min(c, cap);
            s_off[sp + 1] = acc;
        }
        s_total = acc;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < min(s_total, kSurvMax); i += blockDim.x) {
        int lo = 0, hi = splits;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (s_off[mid + 1] <= i) lo = mid + 1; else hi = mid;
        }
        s_keys[i] = surv[((size_t)row * splits + lo) * cap + (i - s_off[lo])];
    }
    __syncthreads();
    const int total = s_total;
    if (total > kSurvMax || total < nprobe) s_bad = 1;
    __syncthreads();
    if (s_bad) {
        if (threadIdx.x == 0) fallback_list[atomicAdd(fallback_cnt, 1u)] = (int32_t)row;
        return;
    }
    const int m = min(kc, total);
    // Only the m + 1 smallest (approx dist, id) keys matter: a radix select
    // of the (m+1)-th smallest dist, an order-keeping compaction of every key
    // up to it (ties included), and a sort of those give the same first
    // m + 1 keys as sorting them all.
    int n_sel = total;
    if (total > m + 1) {
        __shared__ KthState ks;
        uint32_t kth, need_eq;
        block_kth_key_of([](int64_t i) { return (uint32_t)(s_keys[i] >> 32); }, total, m + 1, ks, &kth, &need_eq);
        __shared__ uint32_t s_warp[33];
        __shared__ int s_kept;
        if (threadIdx.x == 0) s_kept = 0;
        __syncthreads();
        for (int base = 0; base < total; base += blockDim.x) {
            const int i = base + threadIdx.x;
            const uint64_t key = i < total ? s_keys[i] : ~0ull;
            const uint32_t keep = i < total && (uint32_t)(key >> 32) <= kth;
            uint32_t tot;
            const uint32_t r = blk_scan_excl(keep, s_warp, &tot);  // synchronises: reads before writes
            const int kept = s_kept;
            if (keep) s_keys[kept + (int)r] = key;  // kept + r <= i: in place
            __syncthreads();
            if (threadIdx.x == 0) s_kept = kept + (int)tot;
            __syncthreads();
        }
        n_sel = s_kept;
    }
    int n = 1;
    while (n < n_sel) n <<= 1;
    for (int i = n_sel + threadIdx.x; i < n; i += blockDim.x) s_keys[i] = ~0ull;
    __syncthreads();
    bitonic_asc(s_keys, n);
    // the smallest approximate dist left out of the candidate set
    const float a_star = (total > m) ? key_to_float_asc((uint32_t)(s_keys[m] >> 32)) : tau[row];  // (m+1)-th
    float qn = 0.0f;
    for (int k = 0; k < kDim; ++k) qn = fmaf(s_q[k], s_q[k], qn);
    const float e = err_bound(sqrtf(qn), *cnmax);
    int ne = 1;
    while (ne < m) ne <<= 1;
    for (int i = threadIdx.x; i < ne; i += blockDim.x) {
        uint64_t key = ~0ull;
        if (i < m) {
            const uint32_t col = (uint32_t)s_keys[i];
            const float d = exact_dist(s_q, centroids + (size_t)col * kDim, cn[col]);
            key = dist_key(d, col);
        }
        s_ex[i] = key;
    }
    __syncthreads();
    bitonic_asc(s_ex, ne);
    const float kth = key_to_float_asc((uint32_t)(s_ex[nprobe - 1] >> 32));
    const bool certified = kth < a_star - e;
    if (certified) {
        for (int i = threadIdx.x; i < nprobe; i += blockDim.x) labels[row * nprobe + i] = (uint32_t)s_ex[i];
        return;
    }
    // Second try before the exact fallback: every survivor gets its exact
    // dist.  Every centroid left out then has an approximate dist above tau,
    // so the row is proven when its k-th exact dist is below tau - E.  (With
    // many centroids per mixture component the gap after the k-th candidate is
    // often narrower than E, while tau sits well beyond it.)
    if (total > m) {
        for (int i = threadIdx.x; i < total; i += blockDim.x) {
            int lo = 0, hi = splits;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (s_off[mid + 1] <= i) lo = mid + 1; else hi = mid;
            }
            const uint32_t col = (uint32_t)surv[((size_t)row * splits + lo) * cap + (i - s_off[lo])];
            s_keys[i] = dist_key(exact_dist(s_q, centroids + (size_t)col * kDim, cn[col]), col);
        }
        int nt = 1;
        while (nt < total) nt <<= 1;
        for (int i = total + threadIdx.x; i < nt; i += blockDim.x) s_keys[i] = ~0ull;
        __syncthreads();
        bitonic_asc(s_keys, nt);
        const float kth2 = key_to_float_asc((uint32_t)(s_keys[nprobe - 1] >> 32));
        if (kth2 < tau[row] - e) {
            for (int i = threadIdx.x; i < nprobe; i += blockDim.x) labels[row * nprobe + i] = (uint32_t)s_keys[i];
            return;
        }
    }
    if (threadIdx.x == 0) fallback_list[atomicAdd(fallback_cnt, 1u)] = (int32_t)row;
}

// Assignment re-rank: one warp per row over its 16 x splits candidates.
__global__ void assign_rerank_kernel(const float* __restrict__ x, int64_t rows, const float* __restrict__ centroids,
                                     const float* __restrict__ cn, const uint64_t* __restrict__ top, int splits,
                                     const float* __restrict__ cnmax, uint32_t* __restrict__ assign,
                                     int32_t* __restrict__ fallback_list, uint32_t* __restrict__ fallback_cnt) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    if (fallback_cnt[1] != 0u) {  // tensor-core error flag: exact path for every row
        if (lane == 0) fallback_list[atomicAdd(fallback_cnt, 1u)] = (int32_t)row;
        return;
    }
    const float* q = x + row * kDim;
    float qn = 0.0f;
    for (int k = lane; k < kDim; k += 32) qn = fmaf(q[k], q[k], qn);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) qn += __shfl_xor_sync(0xffffffffu, qn, off);
    const float e = err_bound(sqrtf(qn), *cnmax);
    uint64_t best = ~0ull;
    float a_star = INFINITY;
    const int ncand = kTopA * splits;
    for (int i = lane; i < ncand; i += 32) {
        const uint64_t k = top[(size_t)row * ncand + i];
        if ((i % kTopA) == kTopA - 1) a_star = fminf(a_star, key_to_float_asc((uint32_t)(k >> 32)));
        if (k == ~0ull) continue;
        const uint32_t col = (uint32_t)k;
        const float d = exact_dist(q, centroids + (size_t)col * kDim, cn[col]);
        const uint64_t key = dist_key(d, col);
        best = key < best ? key : best;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const uint64_t o = __shfl_xor_sync(0xffffffffu, best, off);
        best = o < best ? o : best;
        a_star = fminf(a_star, __shfl_xor_sync(0xffffffffu, a_star, off));
    }
    if (lane == 0) {
        const float b = key_to_float_asc((uint32_t)(best >> 32));
        if (best != ~0ull && b < a_star - e) {
            assign[row] = (uint32_t)best;
        } else {
            fallback_list[atomicAdd(fallback_cnt, 1u)] = (int32_t)row;
        }
    }
}

// Exact fallback: one CTA per listed row computes every dist with the
// sequential fma chain into `scratch` and selects the k smallest (dist, id).

__global__ void __launch_bounds__(1024) exact_rows_kernel(const float* __restrict__ x, const float* __restrict__ centroids,
                                                          const float* __restrict__ cn, int64_t cols, int k,
                                                          const int32_t* __restrict__ list,
                                                          const uint32_t* __restrict__ count, float* __restrict__ scratch,
                                                          uint32_t* __restrict__ out_labels, uint32_t first = 0) {
    __shared__ alignas(16) float s_q[kDim];
    const uint32_t n = *count;
    float* d = scratch + (size_t)blockIdx.x * cols;
    for (uint32_t r = first + blockIdx.x; r < n; r += gridDim.x) {
        const int64_t row = list[r];
        __syncthreads();
        if (threadIdx.x < kDim) s_q[threadIdx.x] = x[row * kDim + threadIdx.x];
        __syncthreads();
        for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) d[c] = exact_dist(s_q, centroids + c * kDim, cn[c]);
        __syncthreads();
        block_select_smallest(d, cols, k, out_labels + row * k);
    }
}

// ---- host side ---------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// [rows x 128] bf16 row-major, 128 x 64 boxes with 128-byte swizzle.
static bool make_map(CUtensorMap* m, const void* base, int64_t rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)kK, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kK * 2};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE>
static size_t tc_smem_bytes() { return sizeof(TcSmem<MODE>) + 1024; }

template <int MODE>
static chm_status launch_tc(const __nv_bfloat16* a, int64_t rows, const __nv_bfloat16* b, int64_t cols,
                            int splits, TcArgs args, cudaStream_t st) {
    CUtensorMap ma, mb;
    if (!make_map(&ma, a, rows) || !make_map(&mb, b, cols)) return CHM_ERR_UNSUPPORTED;
    const int n_tiles = (int)((cols + kTN - 1) / kTN);
    splits = std::max(1, std::min(splits, n_tiles));
    args.tiles_per_split = (n_tiles + splits - 1) / splits;
    args.splits = splits;
    const size_t smem = tc_smem_bytes<MODE>();
    static_assert(sizeof(TcSmem<MODE>) + 1024 <= 227 * 1024, "tc_dist_kernel shared memory");
    CHM_CUDA(cudaFuncSetAttribute(tc_dist_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid(splits, (unsigned)((rows + kTM - 1) / kTM));
    tc_dist_kernel<MODE><<<grid, TcCfg<MODE>::kThreads, smem, st>>>(ma, mb, args);
    return launch_status("tc_dist_kernel");
}

}  // namespace chm


chm_status chm_probe_fallback_batch(const float* x, const int32_t* list, const uint32_t* count, int max_rows,
                                    const float* centroids, const float* cn, int64_t nc, int k, float* q_scratch,
                                    float* dist_scratch, uint32_t* labels, cudaStream_t st);

namespace chm {

struct ProbePlan {
    int64_t rows, nc;
    int nprobe, kc, kthr, prefix, splits, store_splits, cap;
};

// SMs of the current device (148 on B200; also the answer when no device is
// visible, so that workspace sizes can be computed anywhere).
static int device_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                   cudaSuccess || sms <= 0) {
        (void)cudaGetLastError();
        return 148;
    }
    return sms;
}

// Centroid-range splits per row tile.  The kernel runs one CTA per SM, so the
// grid executes in waves of `sms` CTAs; a CTA costs its tiles plus a fixed
// pipeline fill and drain of about kSplitFixedTiles tiles.  The split count
// minimises waves x (tiles per split + fixed), so that the last wave is not
// left mostly empty (320 CTAs on 148 SMs would run three waves, the last
// with 24 CTAs).  Each split keeps at least 8 tiles.
constexpr int kSplitFixedTiles = 4;
static int choose_splits(int64_t row_tiles, int n_tiles, int sms) {
    const int max_s = std::min(kMaxSplits, std::max(1, n_tiles / 8));
    int best = 1;
    double best_cost = 1e300;
    for (int sp = 1; sp <= max_s; ++sp) {
        const int64_t waves = (row_tiles * sp + sms - 1) / sms;
        const int tps = (n_tiles + sp - 1) / sp;
        const double cost = (double)waves * (tps + kSplitFixedTiles);
        if (cost < best_cost) {
            best_cost = cost;
            best = sp;
        }
    }
    return best;
}

static ProbePlan probe_plan(int64_t rows, int64_t nc, int nprobe) {
    ProbePlan p;
    p.rows = rows;
    p.nc = nc;
    p.nprobe = nprobe;
    p.kc = std::min<int64_t>(nc, std::min(512, nprobe + 64));
    // a prefix sample of nc / 32 centroids, at most 65,536 (at least 4 kc); a
    // larger sample costs more in the threshold pass (its dists are written
    // out and selected per row) than it saves in the re-rank
    p.prefix = (int)std::min<int64_t>(nc, std::max<int64_t>(4 * p.kc, std::min<int64_t>(nc / 32, 65536)));
    p.prefix = (int)std::min<int64_t>(nc, ((p.prefix + kTN - 1) / kTN) * kTN);
    // the threshold is the kthr-th smallest prefix dist, kthr chosen so that
    // about 4 kc centroids pass the filter: enough for the re-rank's kc + 1
    // (fewer: the row takes the exact path), a quarter of the survivors
    // (and of the re-rank's select work) of kthr = kc
    p.kthr = p.kc;
    if (p.prefix < nc)
        p.kthr = (int)std::max<int64_t>(1, std::min<int64_t>(p.kc, (4LL * p.kc * p.prefix + nc - 1) / nc));
    const int64_t row_tiles = (rows + kTM - 1) / kTM;
    const int sms = device_sms();
    // small batches split the centroid range across many CTAs, so that a
    // single query still uses the whole GPU
    p.splits = choose_splits(row_tiles, (int)((nc + kTN - 1) / kTN), sms);
    p.store_splits = choose_splits(row_tiles, (p.prefix + kTN - 1) / kTN, sms);
    const double expect = (double)p.kthr * nc / std::max(1, p.prefix);
    p.cap = (int)std::min<double>(kSurvMax, std::max(64.0, 4.0 * expect / p.splits + 64));
    return p;
}

}  // namespace chm

namespace chm {
__global__ void max_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
    __shared__ float s[32];
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? s[threadIdx.x] : -INFINITY;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (threadIdx.x == 0) *out = m;
    }
}
}  // namespace chm

extern "C" chm_status chm_to_bf16(const float* x, int64_t n, void* out, void* stream) {
    if (n <= 0) return CHM_OK;
    chm::to_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        x, n, static_cast<__nv_bfloat16*>(out));
    return chm::launch_status("to_bf16_kernel");
}

extern "C" chm_status chm_max_value(const float* x, int64_t n, float* out, void* stream) {
    if (n <= 0) return CHM_ERR_INVALID;
    chm::max_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(x, n, out);
    return chm::launch_status("max_kernel");
}

size_t chm_tc_probe_workspace_bytes(int64_t rows, int64_t nc, int nprobe) {
    const chm::ProbePlan p = chm::probe_plan(rows, nc, nprobe);
    chm::Sizer s;
    s.take<__nv_bfloat16>((size_t)rows * chm::kK);          // bf16 rows
    s.take<float>((size_t)rows * p.prefix);                  // threshold dists
    s.take<float>((size_t)rows);                             // tau
    s.take<uint64_t>((size_t)rows * p.splits * p.cap);       // survivors
    s.take<int32_t>((size_t)rows * p.splits);                // survivor counts
    s.take<uint32_t>((size_t)rows * p.kc);                   // threshold select labels
    s.take<int32_t>((size_t)rows);                           // fallback list
    s.take<uint32_t>(4);                                     // counters
    s.take<float>((size_t)chm::kFallbackRows * nc);        // fallback scratch rows
    s.take<float>((size_t)chm::kFallbackBatch * chm::kDim);  // batched fallback: rows
    s.take<float>((size_t)chm::kFallbackBatch * nc);         // batched fallback: dists
    return s.off;
}

// Row k-th key of the prefix dists (shared radix select in probe.cu).
chm_status chm_row_kth(const float* dist, int64_t rows, int64_t cols, int k, float* kth, uint32_t* labels,
                       void* stream);

chm_status chm_tc_probe(const float* rot, int64_t rows, const float* centroids, const __nv_bfloat16* cent_bf16,
                        const float* cn, const float* cnmax, int64_t nc, int nprobe, uint32_t* labels, void* ws,
                        size_t ws_bytes, cudaStream_t st) {
    using namespace chm;
    const ProbePlan p = probe_plan(rows, nc, nprobe);
    Arena a(ws, ws_bytes);
    auto* qb = a.take<__nv_bfloat16>((size_t)rows * kK);
    auto* pdist = a.take<float>((size_t)rows * p.prefix);
    auto* tau = a.take<float>((size_t)rows);
    auto* surv = a.take<uint64_t>((size_t)rows * p.splits * p.cap);
    auto* scnt = a.take<int32_t>((size_t)rows * p.splits);
    auto* tlab = a.take<uint32_t>((size_t)rows * p.kc);
    auto* fl = a.take<int32_t>((size_t)rows);
    auto* cnt = a.take<uint32_t>(4);
    auto* scratch = a.take<float>((size_t)kFallbackRows * nc);
    auto* fbq = a.take<float>((size_t)kFallbackBatch * kDim);
    auto* fbd = a.take<float>((size_t)kFallbackBatch * nc);
    if (a.overflow) return CHM_ERR_CAPACITY;
    CHM_CUDA(cudaMemsetAsync(cnt, 0, 16, st));
    const int64_t nel = rows * kK;
    to_bf16_kernel<<<(unsigned)((nel + 255) / 256), 256, 0, st>>>(rot, nel, qb);
    CHM_TRY(launch_status("to_bf16_kernel"));
    // 1) threshold from a prefix of the centroids
    TcArgs t1{};
    t1.rows = rows;
    t1.cols = p.prefix;
    t1.cn = cn;
    t1.dist = pdist;
    t1.ld = p.prefix;
    t1.err = cnt + 1;
    CHM_TRY(launch_tc<kStore>(qb, rows, cent_bf16, p.prefix, p.store_splits, t1, st));
    CHM_TRY(chm_row_kth(pdist, rows, p.prefix, p.kthr, tau, tlab, st));
    // 2) filter over all centroids
    TcArgs t2{};
    t2.rows = rows;
    t2.cols = nc;
    t2.cn = cn;
    t2.tau = tau;
    t2.surv = surv;
    t2.surv_cnt = scnt;
    t2.cap = p.cap;
    t2.err = cnt + 1;
    CHM_TRY(launch_tc<kFilter>(qb, rows, cent_bf16, nc, p.splits, t2, st));
    // 3) exact re-rank with the certificate, exact fallback for the rest
    probe_rerank_kernel<<<(unsigned)rows, kRerankThreads, 0, st>>>(rot, centroids, cn, surv, scnt, p.splits, p.cap,
                                                                   tau, p.kc, nprobe, cnmax, labels, fl, cnt);
    CHM_TRY(launch_status("probe_rerank_kernel"));
    // the first kFallbackBatch flagged rows in one exact GEMM pass, the rest row by row
    CHM_TRY(chm_probe_fallback_batch(rot, fl, cnt, kFallbackBatch, centroids, cn, nc, nprobe, fbq, fbd, labels, st));
    exact_rows_kernel<<<kFallbackRows, 1024, 0, st>>>(rot, centroids, cn, nc, nprobe, fl, cnt, scratch, labels,
                                                      (uint32_t)kFallbackBatch);
    return launch_status("exact_rows_kernel");
}

size_t chm_tc_assign_workspace_bytes(int64_t rows, int64_t nc) {
    chm::Sizer s;
    s.take<__nv_bfloat16>((size_t)rows * chm::kK);
    s.take<uint64_t>((size_t)rows * chm::kTopA * 2);
    s.take<int32_t>((size_t)rows);
    s.take<uint32_t>(4);
    s.take<float>((size_t)chm::kFallbackRows * nc);
    s.take<float>((size_t)chm::kFallbackBatch * chm::kDim);
    s.take<float>((size_t)chm::kFallbackBatch * nc);
    return s.off;
}

chm_status chm_tc_assign(const float* x128, int64_t rows, const float* centroids, const __nv_bfloat16* cent_bf16,
                         const float* cn, const float* cnmax, int64_t nc, uint32_t* assign, void* ws,
                         size_t ws_bytes, cudaStream_t st) {
    using namespace chm;
    Arena a(ws, ws_bytes);
    auto* xb = a.take<__nv_bfloat16>((size_t)rows * kK);
    auto* top = a.take<uint64_t>((size_t)rows * kTopA * 2);  // [rows][2 epilogue groups][16]
    auto* fl = a.take<int32_t>((size_t)rows);
    auto* cnt = a.take<uint32_t>(4);
    auto* scratch = a.take<float>((size_t)kFallbackRows * nc);
    auto* fbq = a.take<float>((size_t)kFallbackBatch * kDim);
    auto* fbd = a.take<float>((size_t)kFallbackBatch * nc);
    if (a.overflow) return CHM_ERR_CAPACITY;
    CHM_CUDA(cudaMemsetAsync(cnt, 0, 16, st));
    const int64_t nel = rows * kK;
    to_bf16_kernel<<<(unsigned)((nel + 255) / 256), 256, 0, st>>>(x128, nel, xb);
    CHM_TRY(launch_status("to_bf16_kernel"));
    TcArgs t{};
    t.rows = rows;
    t.cols = nc;
    t.cn = cn;
    t.top = top;
    t.err = cnt + 1;
    CHM_TRY(launch_tc<kTop16>(xb, rows, cent_bf16, nc, 1, t, st));
    assign_rerank_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(x128, rows, centroids, cn, top, 2,
                                                                             cnmax, assign, fl, cnt);
    CHM_TRY(launch_status("assign_rerank_kernel"));
    CHM_TRY(chm_probe_fallback_batch(x128, fl, cnt, kFallbackBatch, centroids, cn, nc, 1, fbq, fbd, assign, st));
    exact_rows_kernel<<<kFallbackRows, 1024, 0, st>>>(x128, centroids, cn, nc, 1, fl, cnt, scratch, assign,
                                                      (uint32_t)kFallbackBatch);
    return launch_status("exact_rows_kernel");
}

extern "C" size_t chm_probe_tc_workspace_bytes(int64_t nrows, int64_t n_clusters, int32_t nprobe) {
    return chm_tc_probe_workspace_bytes(nrows, n_clusters, nprobe);
}

extern "C" chm_status chm_probe_tc(const float* rot, int64_t nrows, const float* centroids, const void* cent_bf16,
                                   const float* cn, const float* cnmax, int64_t nc, int32_t nprobe, uint32_t* labels,
                                   void* ws, size_t ws_bytes, void* stream) {
    if (nrows <= 0) return CHM_OK;
    if (nprobe <= 0 || nprobe > 448 || nprobe > nc || !cent_bf16 || !cnmax) return CHM_ERR_INVALID;
    return chm_tc_probe(rot, nrows, centroids, static_cast<const __nv_bfloat16*>(cent_bf16), cn, cnmax, nc, nprobe,
                        labels, ws, ws_bytes, (cudaStream_t)stream);
}
