// Refinement with a tensor-core candidate filter: the 1-bit document score
// (same results as refine_1bit_kernel) and the full-bit document score (same
// results as fullbit_kernel), bit for bit.
//
// Both scores are, per query token t, the max over the document's tokens of
// dist = (ip - cb[t]) * factor, then a fixed reduction over t (the reference's
// 128-thread tree, kernels.cu:557-570, or the full-bit 16-lane sum,
// search_impl.cu:569-572).  ip is the 1-bit LUT sum (kernels.cu:363-373) or
// the (1+ex_bits)-bit code dot in the AVX-512 lane order (space.hpp:806-851).
// Only the max matters, so most (token, t) pairs never need the exact ip:
//
//  1. int8 tensor-core pass (tcgen05.mma.kind::i8, M=128 tokens, N=64, K=128):
//     A = the tokens' code levels as bytes (0/1 bits, or 0..2^w-1), B = the
//     query token in 16-bit fixed point as two int8 limbs
//     (q ~ (256*hi + lo) / 2^14).  The int32 accumulators are exact, so the
//     estimate differs from the real inner product by at most
//     (2^w - 1) * E_t, E_t = sum_d |q_d - qfix_d/2^14|.
//  2. With the exact path's own rounding (the LUT sum's 34 adds, or the 8
//     fmas and 4 tree adds of the lane order), the int->float conversion and
//     the two dist roundings of both paths, every token's exact dist lies
//     within M = max|factor| * margin_t of its estimate, so the max token's
//     estimate is at least (max estimate) - 2M: only tokens above that are
//     candidates (about one per document and query token).
//  3. Candidates get the exact ip and dist with the plain kernels' fp32
//     operations; their max is the exact max.
//
// Work items: the docs of a query packed greedily, in refined order, into
// groups of at most 128 tokens and 16 docs (one M tile); docs longer than 128
// tokens go to a list the SIMT kernels score.  A fill kernel writes per item
// a record (doc row offsets) and every row's code index, so staging an item is
// one coalesced load plus the code gather.  One CTA (4 warps, one row per
// thread) loops over items with a three-stage pipeline: while item k is
// reduced, item k+1 is expanded and multiplied and item k+2's data lands.
#include "codes.cuh"
#include "common.cuh"
#include "select.cuh"
#include "sm100.cuh"

namespace chm {

constexpr int kRtThreads = 128;
constexpr int kRtRows = 128;         // tokens per tile (MMA M)
constexpr int kRtN = 64;             // 32 query tokens x {hi, lo} limbs
constexpr int kRtMaxDocs = 16;       // docs per packed item
constexpr int kRtTmemCols = 64;      // one accumulator: item k+1's MMA is issued once item k's is read
constexpr float kFix = 16384.0f;     // fixed-point scale of the query limbs
// idesc kind::i8: D s32 (bits 4-5 = 2), A s8 (bits 7-9 = 1), B s8 (bits 10-12 = 1), K-major
constexpr uint32_t kRtIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kRtN >> 3) << 17) |
                              ((uint32_t)(kRtRows >> 4) << 24);

constexpr int kRtMaxCand = 512;      // candidates per tile (more: the query is rescored by the SIMT kernel)
constexpr uint32_t kRtNoRow = 0xFFFFFFFFu;  // code index of a row past the item's tokens

// Per-item record, filled in parallel after planning: the first token and
// the row offset of each of the item's docs, and which docs belong to
// another shard (-1 ids).  Row i of doc j is token tstart[j] + i - tok0[j]
// (token order).  A part item holds 128-token part p of one longer doc:
// nd = 1 and tstart[0] is the part's first token.
struct RtItem {
    int64_t tstart[kRtMaxDocs];  // first token of doc j's rows
    int r0, nd, ntok;
    uint32_t foreign;            // bit j: doc j of the item is not this shard's
    int tok0[kRtMaxDocs + 1];    // first row of doc j; entries past nd hold ntok
    int pad[3];
};
static_assert(sizeof(RtItem) == 224, "RtItem is fourteen 16-byte chunks");
// Long docs of at most this many 128-token parts become part items.
constexpr int kRtMaxParts = 16;
constexpr int kRtRecWords = (int)sizeof(RtItem) / 4;

// Pipeline slots.  While item k is reduced, item k+1 is multiplied, item
// k+2's codes and factors land and item k+3's record lands (item k+2's row
// code indices come from its record), so records rotate through four slots
// and factors and code indices through three (item k in slot k % 4, k % 3).
template <bool kFull, int kW>
struct RtShape {
    static constexpr int kA = kFull ? 2 : 1;
    static constexpr int kRaw = kFull ? 2 : 3;
    static constexpr int kRowChunks = kFull ? kW : 1;  // 16-byte chunks of one row's packed code
};

template <bool kFull, int kW>
struct __align__(1024) RtSmem {
    uint8_t a[RtShape<kFull, kW>::kA][kRtRows * 128];  // code levels as bytes, K-major SW128
    uint8_t b[kRtN * 128];                              // query limbs, K-major SW128
    uint4 raw[RtShape<kFull, kW>::kRaw][kRtRows * RtShape<kFull, kW>::kRowChunks];  // packed codes as loaded
    float fac[3][kRtRows];
    int row_doc[2][kRtRows];         // item-local doc of each row (-1: past the item's tokens)
    alignas(16) int rec[4][kRtRecWords];  // item k's record in slot k % 4
    uint32_t ridx[3][kRtRows];       // each row's code index (factor slot), for the candidate hand-off
    alignas(16) uint32_t mx[kRtMaxDocs][32];  // max estimate per (doc, query token) as an ordered key, then the threshold
    uint32_t maxf[kRtMaxDocs];       // max |factor| per doc (float bits, >= 0)
    uint32_t cand[kRtMaxCand];       // (row << 5 | t)
    int n_cand;
    int cand_base;                   // 1-bit: this item's first slot in the query's candidate list
    float em[32];                    // margin per unit |factor|
    alignas(16) float cb1[32];
    uint64_t bar;
    uint32_t tmem_base;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm100::smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sm100::smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// byte offset of (row, k) in a K-major SW128 tile with 128-byte rows
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk16) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk16 ^ (row & 7)) << 4));
}

// 4 bits -> 4 bytes of 0/1
__device__ __forceinline__ uint32_t nib_bytes(uint32_t x) { return (x * 0x00204081u) & 0x01010101u; }

// Levels of dims 16c..16c+15 (one 16-byte chunk of the K-major tile) from a
// packed (1+ex_bits)-bit code held as 32-bit words, four dims per word
// operation.  The layouts (code_at states them per dim; r = dim within a
// 64-dim group):
//   w = 2: byte 4(i>>4) + (i&3), bits 2((i&15)>>2)
//   w = 3: per 64 dims (24 bytes): two bits in byte r&15 at 2(r>>4); the
//          third in byte 16 + (r&7), bit r>>3
//   w = 4: byte 8(i>>4) + (i&7), nibble (i&15)>>3
//   w = 5: per 64 dims (40 bytes): low nibbles in byte 16(r>>5) + (r&15),
//          nibble (r>>4)&1; the fifth bit in byte 32 + (r&7), bit r>>3
//   w = 6: per 16 dims j (12 bytes): nibble j>>3 of byte j&7; two bits
//          2(j>>2) of byte 8 + (j&3)
//   w = 7: per 64 dims (56 bytes): six bits in byte r (r < 48), or the top
//          two bits of bytes r-48, r-32 and r-16 (r >= 48); the seventh in
//          byte 48 + (r&7), bit r>>3
// Other widths return false and the caller uses code_at.
template <int kW>
__device__ __forceinline__ bool expand_chunk_fast(const uint32_t* pw, int c, uint32_t (&out)[4]) {
    if (kW == 3) {
        const int g = c >> 2, q = c & 3;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t lo = (pw[6 * g + k] >> (2 * q)) & 0x03030303u;
            const uint32_t hi = (pw[6 * g + 4 + (k & 1)] >> (2 * q + (k >> 1))) & 0x01010101u;
            out[k] = lo | (hi << 2);
        }
        return true;
    } else if (kW == 6) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t lo = (pw[3 * c + (k & 1)] >> (4 * (k >> 1))) & 0x0F0F0F0Fu;
            const uint32_t hi = (pw[3 * c + 2] >> (2 * k)) & 0x03030303u;
            out[k] = lo | (hi << 4);
        }
        return true;
    } else if (kW == 7) {
        const int g = c >> 2, q = c & 3;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t lo;
            if (q < 3) {
                lo = pw[14 * g + 4 * q + k] & 0x3F3F3F3Fu;
            } else {
                lo = ((pw[14 * g + k] >> 6) & 0x03030303u) | (((pw[14 * g + 4 + k] >> 6) & 0x03030303u) << 2) |
                     (((pw[14 * g + 8 + k] >> 6) & 0x03030303u) << 4);
            }
            const uint32_t hi = (pw[14 * g + 12 + (k & 1)] >> (2 * q + (k >> 1))) & 0x01010101u;
            out[k] = lo | (hi << 6);
        }
        return true;
    } else if (kW == 2) {
#pragma unroll
        for (int k = 0; k < 4; ++k) out[k] = (pw[c] >> (2 * k)) & 0x03030303u;
        return true;
    } else if (kW == 4) {
        out[0] = pw[2 * c] & 0x0F0F0F0Fu;
        out[1] = pw[2 * c + 1] & 0x0F0F0F0Fu;
        out[2] = (pw[2 * c] >> 4) & 0x0F0F0F0Fu;
        out[3] = (pw[2 * c + 1] >> 4) & 0x0F0F0F0Fu;
        return true;
    } else if (kW == 5) {
        const int g = c >> 2, cc = c & 3;  // 64-dim group, 16-dim quarter within it
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lo = (pw[10 * g + 4 * (cc >> 1) + j] >> (4 * (cc & 1))) & 0x0F0F0F0Fu;
            const uint32_t hi = (pw[10 * g + 8 + (j & 1)] >> (2 * cc + (j >> 1))) & 0x01010101u;
            out[j] = lo | (hi << 4);
        }
        return true;
    }
    return false;
}

// Greedy packing of each query's refined docs into items, in refined order:
// an item takes consecutive docs while it holds at most kRtMaxDocs docs and
// kRtRows tokens; a doc longer than kRtRows closes the item before it and is
// listed for the SIMT kernel.  The walk is computed in parallel: next(r) is
// where it continues from r (r + 1 after a listed doc, else the end of the
// longest run that fits), and the walk from 0 visits c_i = next^i(0), found
// by composing the tables next^(2^k), k < levels (2^levels > k_refine).
// Shared memory: the tables as 16-bit positions ([levels][k_refine + 1];
// the top one holds the doc lengths until it is built) and a bitmask of the
// listed docs.
__global__ void __launch_bounds__(1024) refine_plan_kernel(const int64_t* __restrict__ doc_ptrs,
                                                           const int32_t* __restrict__ refined_docs,
                                                           const int32_t* __restrict__ num_refined, int k_refine,
                                                           int icap, int levels, int2* __restrict__ items,
                                                           int32_t* __restrict__ n_items, int32_t* __restrict__ big,
                                                           int32_t* __restrict__ n_big) {
    extern __shared__ uint16_t s_j[];
    __shared__ uint32_t s_warp[33];
    const int q = blockIdx.x, tid = threadIdx.x;
    const int R = num_refined[q];
    const int W = k_refine + 1;
    uint32_t* s_big = reinterpret_cast<uint32_t*>(s_j + (size_t)levels * W + ((levels * W) & 1));
    uint16_t* len = s_j + (size_t)(levels - 1) * W;
    for (int w = tid; w < (k_refine + 31) / 32; w += blockDim.x) s_big[w] = 0;
    for (int r = tid; r < R; r += blockDim.x) {
        const int64_t d = refined_docs[(size_t)q * k_refine + r];
        const int64_t l = d < 0 ? 0 : doc_ptrs[d + 1] - doc_ptrs[d];
        len[r] = (uint16_t)(l < 0xFFFF ? l : 0xFFFF);
    }
    __syncthreads();
    for (int r = tid; r <= R; r += blockDim.x) {
        int nx = R;
        if (r < R) {
            if (len[r] > kRtRows) {
                nx = r + 1;
                atomicOr(&s_big[r >> 5], 1u << (r & 31));
            } else {
                int e = r + 1, tok = len[r];
                while (e < R && e - r < kRtMaxDocs && len[e] <= kRtRows && tok + len[e] <= kRtRows) tok += len[e++];
                nx = e;
            }
        }
        s_j[r] = (uint16_t)nx;
    }
    __syncthreads();
    for (int k = 1; k < levels; ++k) {  // the last level overwrites the lengths
        const uint16_t* a = s_j + (size_t)(k - 1) * W;
        uint16_t* b = s_j + (size_t)k * W;
        for (int r = tid; r <= R; r += blockDim.x) b[r] = a[a[r]];
        __syncthreads();
    }
    auto walk = [&](int i) {
        int pos = 0;
        for (int k = 0; k < levels; ++k)
            if ((i >> k) & 1) pos = s_j[(size_t)k * W + pos];
        return pos;
    };
    // walk steps [i0, i1) per thread, in order: count, scan, then write
    const int per = (R + (int)blockDim.x - 1) / (int)blockDim.x;
    const int i0 = min(R, tid * per), i1 = min(R, i0 + per);
    uint32_t cnt_it = 0, cnt_bg = 0;
    for (int i = i0; i < i1; ++i) {
        const int c = walk(i);
        if (c < R) {
            if ((s_big[c >> 5] >> (c & 31)) & 1u) ++cnt_bg; else ++cnt_it;
        }
    }
    uint32_t tot_it, tot_bg;
    uint32_t at_it = blk_scan_excl(cnt_it, s_warp, &tot_it);
    uint32_t at_bg = blk_scan_excl(cnt_bg, s_warp, &tot_bg);
    for (int i = i0; i < i1; ++i) {
        const int c = walk(i);
        if (c < R) {
            if ((s_big[c >> 5] >> (c & 31)) & 1u) big[(size_t)q * k_refine + at_bg++] = c;
            else items[(size_t)q * icap + at_it++] = make_int2(c, (int)s_j[c]);
        }
    }
    // Long docs of at most kRtMaxParts parts become part items (r, -(p + 1))
    // after the others, in refined order while the item array has room; the
    // rest stay in the big list for the SIMT kernels.
    __syncthreads();
    constexpr int kPer = 8;  // big docs per thread: k_refine <= 8192 over 1024 threads
    const int nb = (int)tot_bg;
    const int b0 = min(nb, tid * kPer), b1 = min(nb, b0 + kPer);
    int br[kPer], bp[kPer];
    uint32_t cnt_parts = 0, cnt_keep = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        br[u] = -1;
        bp[u] = 0;
        if (b0 + u < b1) {
            const int r = big[(size_t)q * k_refine + b0 + u];
            const int64_t d = refined_docs[(size_t)q * k_refine + r];
            const int64_t l = doc_ptrs[d + 1] - doc_ptrs[d];
            const int np = (int)((l + kRtRows - 1) / kRtRows);
            br[u] = r;
            bp[u] = np <= kRtMaxParts ? np : 0;
            if (bp[u]) cnt_parts += np; else ++cnt_keep;
        }
    }
    // a doc's parts fit when they end within the room the other items leave
    const uint32_t room = (uint32_t)icap - tot_it;
    uint32_t tot_parts;
    const uint32_t start_p = blk_scan_excl(cnt_parts, s_warp, &tot_parts);
    uint32_t at = start_p, fit_parts = 0;
    cnt_keep = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        if (br[u] < 0) continue;
        if (bp[u] && at + bp[u] <= room) fit_parts += bp[u];
        else {
            if (bp[u]) bp[u] = -bp[u];  // does not fit: stays in the big list
            ++cnt_keep;
        }
        at += bp[u] > 0 ? bp[u] : -bp[u];  // eligible docs advance the running part offset
    }
    // fitting docs are a prefix in refined order (their parts start earlier),
    // so their items are contiguous from tot_it
    uint32_t tot_fit, tot_keep;
    uint32_t at_p = blk_scan_excl(fit_parts, s_warp, &tot_fit);
    uint32_t at_k = blk_scan_excl(cnt_keep, s_warp, &tot_keep);
    // every thread has read its big entries (the scans synchronise)
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        if (br[u] < 0) continue;
        if (bp[u] > 0) {
            for (int pp = 0; pp < bp[u]; ++pp)
                items[(size_t)q * icap + tot_it + at_p++] = make_int2(br[u], -(pp + 1));
        } else {
            big[(size_t)q * k_refine + at_k++] = br[u];
        }
    }
    if (tid == 0) {
        n_items[q] = (int32_t)(tot_it + tot_fit);
        n_big[q] = (int32_t)tot_keep;
    }
}

// Levels of the planner's doubling tables (2^levels > cap, at least 2) and
// its shared memory.
static int rt_plan_levels(int cap) {
    int l = 0;
    while ((1 << l) <= cap) ++l;
    return l < 2 ? 2 : l;
}
static size_t rt_plan_smem(int cap) {
    const int levels = rt_plan_levels(cap);
    const size_t w = (size_t)cap + 1;
    return 2 * ((size_t)levels * w + ((levels * w) & 1)) + 4 * (size_t)((cap + 31) / 32);
}

// One warp per item: its record.  A normal item (x, y) holds refined docs
// x..y-1; a part item (r, -(p + 1)) holds tokens 128 p .. 128 p + 127 of doc r.
__global__ void rt_fill_kernel(const int64_t* __restrict__ doc_ptrs, const int32_t* __restrict__ docs, int cap,
                               int icap, const int2* __restrict__ items, const int32_t* __restrict__ n_items,
                               RtItem* __restrict__ meta) {
    const int q = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const int NI = n_items[q];
    // warps stride over the query's items
    for (int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); item < NI;
         item += gridDim.x * (blockDim.x >> 5)) {
        const int2 rr = items[(size_t)q * icap + item];
        RtItem* m = meta + (size_t)q * icap + item;
        if (rr.y < 0) {
            const int part = -rr.y - 1;
            const int64_t d = docs[(size_t)q * cap + rr.x];
            const int64_t t0 = doc_ptrs[d], len = doc_ptrs[d + 1] - t0;
            const int64_t rem = len - (int64_t)part * kRtRows;
            const int ntok = (int)(rem < kRtRows ? rem : kRtRows);
            if (lane == 0) {
                m->tstart[0] = t0 + (int64_t)part * kRtRows;
                m->r0 = rr.x;
                m->nd = 1;
                m->ntok = ntok;
                m->foreign = 0u;
                m->tok0[0] = 0;
            }
            if (lane < kRtMaxDocs) m->tok0[lane + 1] = ntok;
            continue;
        }
        const int nd = rr.y - rr.x;
        int64_t first = 0;
        int len = 0;
        bool foreign = false;
        if (lane < nd) {
            const int64_t d = docs[(size_t)q * cap + rr.x + lane];
            foreign = d < 0;
            if (!foreign) {
                first = doc_ptrs[d];
                len = (int)(doc_ptrs[d + 1] - first);
            }
        }
        int incl = len;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        const int ntok = __shfl_sync(0xffffffffu, incl, 31);
        const uint32_t fmask = __ballot_sync(0xffffffffu, foreign);
        if (lane == 0) {
            m->r0 = rr.x;
            m->nd = nd;
            m->ntok = ntok;
            m->foreign = fmask;
            m->tok0[0] = 0;
        }
        if (lane < kRtMaxDocs) {
            m->tok0[lane + 1] = incl;  // docs past nd repeat the total
            m->tstart[lane] = first;
        }
    }
}

// Starts the asynchronous load of one item's record into record slot rs.
template <bool kFull, int kW>
__device__ __forceinline__ void rt_issue_rec(RtSmem<kFull, kW>& s, int rs, const RtItem* rec) {
    if (threadIdx.x < kRtRecWords / 4)
        cp_async16(&s.rec[rs][4 * threadIdx.x], reinterpret_cast<const uint4*>(rec) + threadIdx.x);
}

// Starts the asynchronous loads of this thread's row of the item whose
// record is in slot rs (landed): the packed code into code slot cs and the
// factor into factor slot fs; the row's code index (the token, or its
// cluster position through tok2pos; kRtNoRow past the item's tokens) goes to
// ridx[fs].
template <bool kFull, int kW>
__device__ __forceinline__ void rt_issue_rows(RtSmem<kFull, kW>& s, int rs, int fs, int cs,
                                              const uint8_t* __restrict__ codes, const float* __restrict__ factors,
                                              const uint32_t* __restrict__ tok2pos) {
    constexpr int kC = RtShape<kFull, kW>::kRowChunks;
    const int tid = threadIdx.x;
    const RtItem& rec = *reinterpret_cast<const RtItem*>(s.rec[rs]);
    uint32_t idx = kRtNoRow;
    if (tid < rec.ntok) {
        int j = 0;
        while (rec.tok0[j + 1] <= tid) ++j;
        const int64_t tok = rec.tstart[j] + (tid - rec.tok0[j]);
        idx = tok2pos != nullptr ? __ldg(tok2pos + tok) : (uint32_t)tok;
    }
    s.ridx[fs][tid] = idx;
    if (idx != kRtNoRow) {
        const uint4* src = reinterpret_cast<const uint4*>(codes) + (size_t)idx * kC;
#pragma unroll
        for (int v = 0; v < kC; ++v) cp_async16(&s.raw[cs][tid * kC + v], src + v);
        cp_async4(&s.fac[fs][tid], factors + idx);
    }
}

// Expands this thread's row of the item in record slot rs / code slot cs
// into tile ab (levels as bytes) and records the row's item-local doc in
// row_doc[db].  Rows past the item's tokens keep stale bytes: their
// accumulators are never read.
// kFull: the (1+ex_bits)-bit codes (width w) expanded to 0..2^w-1; else the
// 1-bit codes expanded to 0/1.
template <bool kFull, int kW>
__device__ __forceinline__ void rt_expand(RtSmem<kFull, kW>& s, int rs, int cs, int ab, int db) {
    const int tid = threadIdx.x;
    const RtItem& rec = *reinterpret_cast<const RtItem*>(s.rec[rs]);
    uint8_t* a = s.a[ab];
    int ld = -1;
    if (tid < rec.ntok) {
        ld = 0;
        while (rec.tok0[ld + 1] <= tid) ++ld;
        if (kFull) {
            constexpr int bytes = kDim * kW / 8;
            uint32_t pw[bytes / 4];
#pragma unroll
            for (int v = 0; v < kW; ++v) {
                const uint4 x = s.raw[cs][tid * kW + v];
                pw[4 * v] = x.x;
                pw[4 * v + 1] = x.y;
                pw[4 * v + 2] = x.z;
                pw[4 * v + 3] = x.w;
            }
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t wd[4];
                if (!expand_chunk_fast<kW>(pw, c, wd)) {
                    const uint8_t* pk = reinterpret_cast<const uint8_t*>(pw);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t x = 0;
#pragma unroll
                        for (int b = 0; b < 4; ++b) x |= (uint32_t)code_at(pk, c * 16 + j * 4 + b, kW) << (8 * b);
                        wd[j] = x;
                    }
                }
                *reinterpret_cast<uint4*>(a + sw128_off(tid, c)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
            }
        } else {
            const uint4 code = s.raw[cs][tid];
            const uint32_t wv[4] = {code.x, code.y, code.z, code.w};
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t h = wv[c >> 1] >> ((c & 1) * 16);
                *reinterpret_cast<uint4*>(a + sw128_off(tid, c)) =
                    make_uint4(nib_bytes(h & 0xF), nib_bytes((h >> 4) & 0xF), nib_bytes((h >> 8) & 0xF),
                               nib_bytes((h >> 12) & 0xF));
            }
        }
    }
    s.row_doc[db][tid] = ld;
}

// One thread: the K = 128 product of tile ab with the query limbs into the
// accumulator, completion on the barrier.
template <bool kFull, int kW>
__device__ __forceinline__ void rt_mma(RtSmem<kFull, kW>& s, int ab, uint32_t tmem) {
    const uint32_t a_base = sm100::smem_addr(s.a[ab]), b_base = sm100::smem_addr(s.b);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
        mma_i8(tmem, sm100::smem_desc_sw128(a_base + kk * 32), sm100::smem_desc_sw128(b_base + kk * 32), kRtIdesc,
               kk > 0 ? 1u : 0u);
    sm100::mma_commit(&s.bar);
}

// Per query, once per call: the B operand (each query token in 16-bit fixed
// point as two int8 limbs, K-major SW128, the byte image of the tensor-core
// kernel's B tile) and the error margin per query token (per unit |factor|):
//   kFull: code levels up to W = 2^w - 1: the quantisation error times W, the
//          exact sum's 12 roundings (8 fmas + 4 tree adds) and the int->float
//          conversion of the estimate, then the two dist roundings of both paths;
//   else:  quantisation + LUT-sum rounding (34 adds) + the two dist roundings.
// E_t = sum_d |q_d - qfix_d / 2^14| and sum_d |q_d| are summed in double by a
// warp; the 2^-20 safety factor covers the order of those sums.
template <bool kFull, int kW>
__global__ void __launch_bounds__(256) rt_query_kernel(const float* __restrict__ rot, const float* __restrict__ cb,
                                                       uint8_t* __restrict__ qtile, float* __restrict__ qem) {
    const int q = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    {
        // thread tid: row n = tid >> 2 (limb n >> 5 of token n & 31), chunks 2 (tid & 3) + {0, 1}
        const int n = tid >> 2, t = n & 31;
        const bool lo_limb = n >= 32;
        const float* qv = rot + ((size_t)q * kQ + t) * kDim;
        uint8_t* out = qtile + (size_t)q * kRtN * 128;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int chunk = (tid & 3) * 2 + cc;
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t word = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int d = chunk * 16 + j * 4 + b;
                    int fx = __float2int_rn(qv[d] * kFix);
                    fx = max(-16384, min(16384, fx));
                    const int lo = ((fx + 128) & 255) - 128;
                    const int hi = (fx - lo) >> 8;
                    word |= (uint32_t)(uint8_t)(int8_t)(lo_limb ? lo : hi) << (8 * b);
                }
                w[j] = word;
            }
            *reinterpret_cast<uint4*>(out + sw128_off(n, chunk)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    for (int t = warp; t < kQ; t += 8) {
        const float* qt = rot + ((size_t)q * kQ + t) * kDim;
        double e = 0.0, s1 = 0.0;
        for (int d = lane; d < kDim; d += 32) {
            const float v = qt[d];
            int fx = __float2int_rn(v * kFix);
            fx = max(-16384, min(16384, fx));
            e += fabs((double)v - (double)fx / 16384.0);
            s1 += fabs((double)v);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            e += __shfl_xor_sync(0xffffffffu, e, off);
            s1 += __shfl_xor_sync(0xffffffffu, s1, off);
        }
        if (lane == 0) {
            const double c = fabs((double)cb[q * kQ + t]);
            double m;
            if (kFull) {
                const double W = (double)((1 << kW) - 1);
                m = W * e + 24.0 * 0x1p-24 * W * s1 + 0x1p-21 * (W * s1 + c);
            } else {
                m = e + 40.0 * 0x1p-24 * s1 + 0x1p-21 * (s1 + c);
            }
            qem[q * kQ + t] = __double2float_ru(m * (1.0 + 0x1p-20));
        }
    }
}

// Candidates handed to the exact pass (rt_exact_kernel): per query, every
// candidate row's code index and (refined index, query token).
struct RtCandOut {
    uint2* ent;      // [nq][ccap]: code index, refined index << 5 | query token
    int32_t* count;  // [nq] (may run past ccap: the query is then flagged)
    int ccap;
};

// kFull: the full-bit MaxSim of fullbit_kernel (codes at width w, cb = cbex,
// the AVX-512 lane order for the exact sums, its 16-lane document reduction);
// else the 1-bit score of refine_1bit_kernel (cb = cb1).  The candidates go
// to rt_exact_kernel, which holds the query's LUTs (1-bit) or rotated query
// (full-bit) in shared memory, and rt_tree_kernel makes the scores.
//
// Item k (the CTA's k-th) goes through: record loaded (iteration k-3),
// codes and factors loaded (iteration k-2), tile expanded and multiplied
// (iteration k-1), accumulators reduced (iteration k).
template <bool kFull, int kW>
__global__ void __launch_bounds__(kRtThreads, kFull ? 3 : 5) refine_tc_kernel(
    const RtItem* __restrict__ meta, const uint32_t* __restrict__ tok2pos, const uint8_t* __restrict__ codes,
    const float* __restrict__ factors, const float* __restrict__ cb1, const uint8_t* __restrict__ qtile,
    const float* __restrict__ qem, int icap, const int32_t* __restrict__ n_items, uint32_t* __restrict__ status,
    unsigned long long* __restrict__ stats, RtCandOut co) {
    using Sh = RtShape<kFull, kW>;
    extern __shared__ uint8_t smem_raw[];
    RtSmem<kFull, kW>& s =
        *reinterpret_cast<RtSmem<kFull, kW>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q = blockIdx.y;
    const int NI = n_items[q];
    if ((int)blockIdx.x >= NI) return;

    // ---- prologue: the query's B tile and margins (rt_query_kernel), TMEM, barrier
    {
        const uint4* qb = reinterpret_cast<const uint4*>(qtile + (size_t)q * kRtN * 128);
        for (int i = tid; i < kRtN * 128 / 16; i += kRtThreads) reinterpret_cast<uint4*>(s.b)[i] = __ldg(qb + i);
        if (tid < 32) {
            s.cb1[tid] = cb1[q * kQ + tid];
            s.em[tid] = qem[q * kQ + tid];
        }
        for (int i = tid; i < kRtMaxDocs * 32; i += kRtThreads) (&s.mx[0][0])[i] = 0u;
        if (tid < kRtMaxDocs) s.maxf[tid] = 0u;
        if (tid == 0) {
            s.n_cand = 0;
            sm100::mbar_init(&s.bar, 1);
            sm100::fence_mbar_init();
        }
        if (warp == 0) {
            sm100::tmem_alloc(&s.tmem_base, kRtTmemCols);
            sm100::tmem_relinquish();
        }
        fence_proxy_async_smem();
        sm100::tc_fence_before();
        __syncthreads();
        sm100::tc_fence_after();
    }
    const uint32_t tmem = s.tmem_base;
    const float inv_fix = 1.0f / kFix;
    const size_t qb = (size_t)q * icap;
    const int G = gridDim.x;
    int it = blockIdx.x;
    // records of items 0..2 loaded; item 0's rows loaded, expanded and
    // multiplied; item 1's rows loaded
    rt_issue_rec(s, 0, meta + qb + it);
    if (it + G < NI) rt_issue_rec(s, 1, meta + qb + it + G);
    if (it + 2 * G < NI) rt_issue_rec(s, 2, meta + qb + it + 2 * G);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    rt_issue_rows(s, 0, 0, 0, codes, factors, tok2pos);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    rt_expand(s, 0, 0, 0, 0);
    fence_proxy_async_smem();
    sm100::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        sm100::tc_fence_after();
        rt_mma(s, 0, tmem);
    }
    if (it + G < NI) rt_issue_rows(s, 1, 1, 1 % Sh::kRaw, codes, factors, tok2pos);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();

    bool failed = false;  // uniform across the CTA (set from __syncthreads_or)
    unsigned long long n_rows = 0, n_cand = 0;
    int k = 0;
    for (; it < NI; it += G, ++k) {
        const bool has1 = it + G < NI, has2 = it + 2 * G < NI, has3 = it + 3 * G < NI;
        const int rs = k % 4, fs = k % 3;  // record slot; factor and code-index slot
        // ---- item k's accumulators, one row per thread.  Every thread waits
        // for the MMA itself; a wait that ran out is acted on at the barrier
        // below (what was read or expanded meanwhile is then discarded).
        const bool ok = sm100::mbar_wait(&s.bar, (uint32_t)(k & 1));
        sm100::tc_fence_after();
        uint32_t hi[32], lo[32];
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
        sm100::tmem_ld32_async(taddr, hi);
        sm100::tmem_ld32_async(taddr + 32, lo);
        sm100::tmem_wait_ld();
        // ---- item k+1: expanded and multiplied while item k is reduced
        if (has1) rt_expand(s, (k + 1) % 4, (k + 1) % Sh::kRaw, (k + 1) % Sh::kA, (k + 1) & 1);
        fence_proxy_async_smem();
        sm100::tc_fence_before();
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
        if (has1 && tid == 0) {
            sm100::tc_fence_after();
            rt_mma(s, (k + 1) % Sh::kA, tmem);
        }
        // ---- item k+2's rows and item k+3's record, in flight during the reduction
        if (has2) rt_issue_rows(s, (k + 2) % 4, (k + 2) % 3, (k + 2) % Sh::kRaw, codes, factors, tok2pos);
        if (has3) rt_issue_rec(s, (k + 3) % 4, meta + qb + it + 3 * G);
        cp_async_commit();
        // ---- estimated dists, kept in registers
        const RtItem& rec = *reinterpret_cast<const RtItem*>(s.rec[rs]);
        const int T = rec.ntok;
        const int ld = tid < T ? s.row_doc[k & 1][tid] : -1;
        const float f = tid < T ? s.fac[fs][tid] : 0.0f;
        // (x * 2^-14 is exact, so the fma rounds exactly as the subtraction
        // of the product would)
        float da[32];
#pragma unroll
        for (int t4 = 0; t4 < 8; ++t4) {
            const float4 c4 = reinterpret_cast<const float4*>(s.cb1)[t4];
            const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int t = 4 * t4 + e;
                const float a = (float)((int)hi[t] * 256 + (int)lo[t]);
                da[t] = __fmul_rn(__fmaf_rn(a, inv_fix, -cc[e]), f);
            }
        }
        // ---- pass 1: per (doc, query token) max of the estimates and per doc
        // max |factor|.  For each doc among the warp's rows (docs are runs of
        // rows): a transposing butterfly over the 32 x 32 estimates (other
        // docs' lanes as -inf) leaves lane t with the doc's max for query
        // token t, then one shared atomic per lane.  (A warp reduction per
        // query token over the run's lanes measured nine times slower.)  The
        // max is only used for the threshold below, where +0 and -0 give the
        // same value.
        {
            const uint32_t grp = __match_any_sync(0xffffffffu, ld);
            for (uint32_t rem = __ballot_sync(0xffffffffu, ld >= 0); rem;) {
                const int l = __ffs(rem) - 1;
                const uint32_t g = __shfl_sync(0xffffffffu, grp, l);
                rem &= ~g;
                const bool in = (g >> lane) & 1u;
                const int gd = __shfl_sync(0xffffffffu, ld, l);
                const uint32_t fm = __reduce_max_sync(0xffffffffu, in ? __float_as_uint(fabsf(f)) : 0u);
                if (lane == 0) atomicMax(&s.maxf[gd], fm);
                float v[32];
#pragma unroll
                for (int t = 0; t < 32; ++t) v[t] = in ? da[t] : -INFINITY;
                // halving h: lanes with bit h keep the upper half of the window
                // and take their partner's, so after h = 1 v[0] is token lane's
#pragma unroll
                for (int h = 16; h >= 1; h >>= 1) {
                    const bool up = (lane & h) != 0;
#pragma unroll
                    for (int i = 0; i < h; ++i) {
                        const float send = up ? v[i] : v[i + h];
                        const float keep = up ? v[i + h] : v[i];
                        v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, h));
                    }
                }
                atomicMax(&s.mx[gd][lane], float_key_asc(v[0]));
            }
        }
        __syncthreads();
        // ---- pass 2: candidates.  Every row's exact dist is within M =
        // max|f| * em of its estimate, so the max row's estimate is at least
        // (max estimate) - 2M: that threshold per (doc, query token), in
        // place of the max, then a bit per query token for each row and a
        // block scan that places each row's candidates.
        const int nd = rec.nd;
        for (int i = tid; i < nd * 32; i += kRtThreads) {
            const int d = i >> 5, t = i & 31;
            const float M = __fmul_ru(__uint_as_float(s.maxf[d]), s.em[t]);
            s.mx[d][t] = __float_as_uint(__fsub_rd(key_to_float_asc(s.mx[d][t]), __fadd_ru(M, M)));
        }
        __syncthreads();
        uint32_t cmask = 0;
        if (ld >= 0) {
            const uint4* th = reinterpret_cast<const uint4*>(s.mx[ld]);
#pragma unroll
            for (int t4 = 0; t4 < 8; ++t4) {
                const uint4 v = th[t4];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) cmask |= (da[4 * t4 + e] >= __uint_as_float(w[e]) ? 1u : 0u) << (4 * t4 + e);
            }
        }
        const int cnt = __popc(cmask);
        int incl = cnt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        int wbase = 0;
        if (lane == 31 && incl > 0) wbase = atomicAdd(&s.n_cand, incl);  // one slot range per warp
        int at = __shfl_sync(0xffffffffu, wbase, 31) + incl - cnt;
        if (at + cnt <= kRtMaxCand)
            for (uint32_t mm = cmask; mm; mm &= mm - 1) s.cand[at++] = ((uint32_t)tid << 5) | (uint32_t)(__ffs(mm) - 1);
        __syncthreads();
        const int nc = s.n_cand;
        // ---- the candidates go to the exact pass
        if (nc > kRtMaxCand) {
            if (tid == 0) atomicOr(status + q, 1u);  // rescored by the SIMT kernel
        } else {
            if (tid == 0) s.cand_base = nc > 0 ? atomicAdd(co.count + q, nc) : 0;
            __syncthreads();
            const int base = s.cand_base;
            if (base + nc > co.ccap) {
                if (tid == 0) atomicOr(status + q, 1u);  // list full: rescored by the SIMT kernel
            } else {
                for (int c = tid; c < nc; c += kRtThreads) {
                    const uint32_t e = s.cand[c];
                    const int row = (int)(e >> 5);
                    co.ent[(size_t)q * co.ccap + base + c] =
                        make_uint2(s.ridx[fs][row], ((uint32_t)(rec.r0 + s.row_doc[k & 1][row]) << 5) | (e & 31u));
                }
            }
        }
        n_cand += (unsigned long long)(tid == 0 ? nc : 0);
        __syncthreads();
        // ---- document scores: the reference's 128-thread tree (kernels.cu:557-570)
        // (rt_tree_kernel makes the scores once every candidate's exact sum is in)
        for (int j = warp; j < nd; j += kRtThreads / 32) {
            s.mx[j][lane] = 0u;
            if (lane == 0) s.maxf[j] = 0u;
        }
        if (tid == 0) {
            n_rows += (unsigned long long)T;
            s.n_cand = 0;  // every thread read it before the barrier above
        }
        cp_async_wait_all();  // item k+2 landed
        __syncthreads();
    }
    if (failed && tid == 0) {
        // item k's MMA (whose wait ran out) may still be in flight: wait for it
        // again, bounded, before TMEM is released
        sm100::mbar_wait(&s.bar, (uint32_t)(k & 1));
        atomicOr(status + q, 1u);
    }
    cp_async_wait_all();
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) n_cand += __shfl_xor_sync(0xffffffffu, n_cand, off);
    if (lane == 0 && n_cand) atomicAdd(stats + 1, n_cand);
    if (tid == 0 && n_rows) atomicAdd(stats, n_rows);
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 0) sm100::tmem_dealloc(tmem, kRtTmemCols);
}

// Exact sums of the candidates the tensor-core kernel handed off, one per
// thread, the max per (refined doc, query token) by atomicMax on ordered
// keys.  kFull: fullbit_kernel's arithmetic (16 lane chains over the 8
// chunks of 16 levels, reduce16 in the AVX-512 order, search_impl.cu:
// 510-574) against the rotated query; else refine_1bit_kernel's LUT sum
// (kernels.cu:363-375).  The query's 32 LUTs (or 32 rotated tokens) sit in
// shared memory with padded rows, so that lanes on different query tokens
// spread over the banks.  Flagged queries are skipped: the SIMT kernels
// rescore them.
constexpr int kRxThreads = 256;
template <bool kFull>
constexpr int rx_stride() { return kFull ? kDim + 4 : kLutPerQ + 1; }
template <bool kFull>
size_t rt_exact_smem() { return sizeof(float) * (size_t)kQ * rx_stride<kFull>(); }

template <bool kFull, int kW>
__global__ void __launch_bounds__(kRxThreads) rt_exact_kernel(RtCandOut co, const uint8_t* __restrict__ codes,
                                                               const float* __restrict__ factors,
                                                               const float* __restrict__ table,
                                                               const float* __restrict__ cb,
                                                               const uint32_t* __restrict__ status, int cap,
                                                               uint32_t* __restrict__ exact) {
    constexpr int kS = rx_stride<kFull>();
    constexpr int kRow = kFull ? kDim : kLutPerQ;  // floats per query token in `table`
    extern __shared__ float s_tab[];
    __shared__ float s_cb[kQ];
    const int q = blockIdx.y;
    if (status[q]) return;
    const int n = min(co.count[q], co.ccap);
    if ((int)blockIdx.x * kRxThreads >= n) return;
    const float* src = table + (size_t)q * kQ * kRow;
    for (int i = threadIdx.x; i < kQ * kRow; i += kRxThreads) s_tab[(i / kRow) * kS + (i % kRow)] = __ldg(src + i);
    if (threadIdx.x < kQ) s_cb[threadIdx.x] = cb[q * kQ + threadIdx.x];
    __syncthreads();
    const uint2* ent = co.ent + (size_t)q * co.ccap;
    for (int i = blockIdx.x * kRxThreads + threadIdx.x; i < n; i += gridDim.x * kRxThreads) {
        const uint2 m = ent[i];
        const int t = (int)(m.y & 31u);
        const float* tab = s_tab + t * kS;
        float ip;
        if (kFull) {
            uint32_t pw[kW * 4];
            const uint4* cp = reinterpret_cast<const uint4*>(codes) + (size_t)m.x * kW;
#pragma unroll
            for (int v = 0; v < kW; ++v) {
                const uint4 x = __ldg(cp + v);
                pw[4 * v] = x.x;
                pw[4 * v + 1] = x.y;
                pw[4 * v + 2] = x.z;
                pw[4 * v + 3] = x.w;
            }
            float acc[16];
#pragma unroll
            for (int l = 0; l < 16; ++l) acc[l] = 0.0f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t wd[4];
                if (!expand_chunk_fast<kW>(pw, c, wd)) {
                    const uint8_t* pk = reinterpret_cast<const uint8_t*>(pw);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t x = 0;
#pragma unroll
                        for (int b = 0; b < 4; ++b) x |= (uint32_t)code_at(pk, c * 16 + j * 4 + b, kW) << (8 * b);
                        wd[j] = x;
                    }
                }
#pragma unroll
                for (int l4 = 0; l4 < 4; ++l4) {
                    const float4 qv = *reinterpret_cast<const float4*>(tab + 16 * c + 4 * l4);
                    const float qq[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        acc[4 * l4 + e] = __fmaf_rn((float)((wd[l4] >> (8 * e)) & 0xFFu), qq[e], acc[4 * l4 + e]);
                }
            }
            ip = reduce16_avx512(acc);
        } else {
            ip = lut_ip(tab, __ldg(reinterpret_cast<const uint4*>(codes) + m.x));
        }
        const float dist = fmul(fsub(ip, s_cb[t]), __ldg(factors + m.x));
        atomicMax(exact + ((size_t)q * cap + (m.y >> 5)) * kQ + t, float_key_asc(dist));
    }
}

// Document scores from the exact maxima, one warp per refined doc.  kFull:
// fullbit_kernel's reduction (max[0:16] + max[16:32] lane-wise, then the
// 16-lane tree); else the reference's 128-thread tree (kernels.cu:557-570:
// strides 64 and 32 add zeros, then 16..1).  Docs without maxima (longer
// than one tile: the SIMT kernels score them) are left alone; other shards'
// docs (-1) score -inf.
template <bool kFull>
__global__ void rt_tree_kernel(const uint32_t* __restrict__ exact, const int32_t* __restrict__ docs,
                               const int32_t* __restrict__ counts, int cap, float* __restrict__ scores) {
    const int q = blockIdx.y, lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= counts[q]) return;
    const size_t at = (size_t)q * cap + r;
    if (docs[at] < 0) {
        if (lane == 0) scores[at] = -INFINITY;
        return;
    }
    const uint32_t key = exact[at * kQ + lane];
    if (__shfl_sync(0xffffffffu, key, 0) == 0u) return;
    const float m = key_to_float_asc(key);
    float x;
    if (kFull) {
        x = fadd(m, __shfl_down_sync(0xffffffffu, m, 16));
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off, 16));
    } else {
        x = fadd(fadd(fadd(0.0f, m), 0.0f), 0.0f);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off));
    }
    if (lane == 0) scores[at] = x;
}

// The exact pass and the scores after a tensor-core launch.  table: the
// LUTs (1-bit) or the rotated queries (full-bit); cb: cb1 or cbex.
template <bool kFull, int kW>
static chm_status rt_finish(const RtCandOut& co, const uint8_t* codes, const float* factors, const float* table,
                            const float* cb, const uint32_t* status, int nq, int cap, uint32_t* exact,
                            const int32_t* docs, const int32_t* counts, float* scores, cudaStream_t st) {
    const size_t smem = rt_exact_smem<kFull>();
    CHM_CUDA(cudaFuncSetAttribute(rt_exact_kernel<kFull, kW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    // about four resident waves over the batch
    const int per_sm = kFull ? 8 : 3;
    const int gx = std::max(1, std::min(64, (148 * per_sm * 4 + nq - 1) / nq));
    rt_exact_kernel<kFull, kW><<<dim3((unsigned)gx, (unsigned)nq), kRxThreads, smem, st>>>(co, codes, factors, table,
                                                                                           cb, status, cap, exact);
    CHM_TRY(launch_status("rt_exact_kernel"));
    rt_tree_kernel<kFull><<<dim3((unsigned)((cap + 7) / 8), (unsigned)nq), 256, 0, st>>>(exact, docs, counts, cap,
                                                                                         scores);
    return launch_status("rt_tree_kernel");
}

// Queries whose tensor-core launch gave up on a bounded wait are scored
// again by the SIMT kernel (status bit set); others return at once.
__global__ void refine_status_clear_kernel(uint32_t* status, int nq, unsigned long long* stats) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nq) status[i] = 0;
    if (i < 2) stats[i] = 0;
}

}  // namespace chm

namespace chm {
template <bool kFull, int kW>
size_t refine_tc_smem_bytes() { return sizeof(RtSmem<kFull, kW>) + 1024; }

// Workspace of one tensor-core refinement call.
struct RtWork {
    int icap;        // items per query (parts of long docs included)
    int2* items;
    int32_t* n_items;
    uint32_t* status;
    unsigned long long* stats;
    int32_t* big;
    int32_t* n_big;
    RtItem* meta;
    uint8_t* qtile;  // per query: the B tile (rt_query_kernel)
    float* qem;      // per query token: the margin
    RtCandOut cand;  // the candidates of each query
    uint32_t* exact; // [nq][cap][32] exact max per (refined doc, query token), ordered keys
};

// Candidate slots per item: every (doc or part, query token) has at least
// one, about 1.03 on average (more: the query is flagged).
constexpr int kRtCandPerItem = 36;

template <typename A>
static void rt_layout(A& a, int nq, int cap, int icap, RtWork* w) {
    auto items = a.template take<int2>((size_t)nq * icap);
    auto n_items = a.template take<int32_t>((size_t)nq);
    auto status = a.template take<uint32_t>((size_t)nq);
    auto stats = a.template take<unsigned long long>(2);  // rows scored, exact candidates (last call)
    auto big = a.template take<int32_t>((size_t)nq * cap);
    auto n_big = a.template take<int32_t>((size_t)nq);
    auto meta = a.template take<RtItem>((size_t)nq * icap);
    auto qtile = a.template take<uint8_t>((size_t)nq * kRtN * 128);
    auto qem = a.template take<float>((size_t)nq * kQ);
    const int ccap = kRtCandPerItem * icap;
    auto cent = a.template take<uint2>((size_t)nq * ccap);
    auto ccount = a.template take<int32_t>((size_t)nq);
    auto exact = a.template take<uint32_t>((size_t)nq * cap * kQ);
    if (w)
        *w = RtWork{icap, (int2*)items, (int32_t*)n_items, (uint32_t*)status, (unsigned long long*)stats,
                    (int32_t*)big, (int32_t*)n_big, (RtItem*)meta, (uint8_t*)qtile, (float*)qem,
                    RtCandOut{(uint2*)cent, (int32_t*)ccount, ccap}, (uint32_t*)exact};
}

struct RtSizer {
    Sizer s;
    template <typename T>
    void* take(size_t n) {
        s.take<T>(n);
        return nullptr;
    }
};

static size_t rt_bytes(int nq, int cap, int icap) {
    RtSizer s;
    rt_layout(s, nq, cap, icap, nullptr);
    return s.s.off;
}

// Items per query with room for the parts of long docs: per refined doc one
// item, plus three times the mean doc length in parts (refined docs run
// longer than the mean), at most kRtMaxParts - 1 more.  Parts that do not
// fit go to the SIMT kernels.
static int rt_icap(const chm_index* idx, int cap) {
    if (idx == nullptr || idx->max_doc_len <= kRtRows || idx->num_docs <= 0) return cap;
    const double mean = (double)idx->n_tokens / (double)idx->num_docs;
    const int extra = (int)std::min<double>(kRtMaxParts - 1, std::ceil(3.0 * mean / kRtRows));
    return (int)std::min<int64_t>((int64_t)cap * (1 + extra), (int64_t)1 << 30);
}

// The item capacity a call's workspace affords: the room for long docs'
// parts when it is large enough, else one item per refined doc.
static int rt_call_icap(const chm_index* idx, int nq, int cap, size_t ws_bytes) {
    const int full = rt_icap(idx, cap);
    return ws_bytes >= rt_bytes(nq, cap, full) ? full : cap;
}

static chm_status rt_plan(const chm_index* idx, int nq, const int32_t* docs, const int32_t* counts, int cap,
                          const RtWork& w, cudaStream_t st) {
    refine_status_clear_kernel<<<(nq + 255) / 256, 256, 0, st>>>(w.status, nq, w.stats);
    CHM_TRY(launch_status("refine_status_clear_kernel"));
    const size_t plan_smem = rt_plan_smem(cap);
    CHM_CUDA(cudaFuncSetAttribute(refine_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan_smem));
    refine_plan_kernel<<<nq, 1024, plan_smem, st>>>(idx->doc_ptrs, docs, counts, cap, w.icap, rt_plan_levels(cap),
                                                    w.items, w.n_items, w.big, w.n_big);
    CHM_TRY(launch_status("refine_plan_kernel"));
    // one warp per item, 4 warps per block, 128 blocks per query striding over its items
    rt_fill_kernel<<<dim3(128u, (unsigned)nq), 128, 0, st>>>(idx->doc_ptrs, docs, cap, w.icap, w.items, w.n_items,
                                                            w.meta);
    return launch_status("rt_fill_kernel");
}

// About eight waves of the resident CTAs: items per CTA vary by query, so
// finer-grained CTAs balance the tail.  Resident CTAs per SM come from the
// kernel's shared memory, registers and TMEM columns (the runtime's occupancy
// query answers 1 for these kernels).
template <typename Kernel>
static chm_status rt_grid(Kernel kernel, size_t smem, int nq, int cap, dim3* grid) {
    int dev = 0, sms = 0, smem_sm = 0, resv = 0, regs_sm = 0;
    CHM_CUDA(cudaGetDevice(&dev));
    CHM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    CHM_CUDA(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    CHM_CUDA(cudaDeviceGetAttribute(&resv, cudaDevAttrReservedSharedMemoryPerBlock, dev));
    CHM_CUDA(cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev));
    // the largest shared-memory carveout, so that those CTAs fit
    CHM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                  (int)cudaSharedmemCarveoutMaxShared));
    cudaFuncAttributes fa;
    CHM_CUDA(cudaFuncGetAttributes(&fa, kernel));
    const size_t smem_blk = smem + fa.sharedSizeBytes + (size_t)resv;
    const int by_smem = (int)((size_t)smem_sm / std::max<size_t>(smem_blk, 1));
    const int regs_warp = ((fa.numRegs * 32 + 255) / 256) * 256;  // allocated per warp in units of 256
    const int by_regs = regs_sm / std::max(1, regs_warp * (kRtThreads / 32));
    const int by_tmem = 512 / kRtTmemCols;
    const int occ = std::max(1, std::min(std::min(by_smem, by_regs), std::min(by_tmem, 32)));
    int gx = (occ * sms * 8 + nq - 1) / nq;
    gx = std::max(1, std::min(gx, cap));
    *grid = dim3((unsigned)gx, (unsigned)nq);
    return CHM_OK;
}

template <int kW>
static chm_status launch_fullbit_tc(const chm_index* idx, int nq, const float* rot, const float* cbex,
                                   const int32_t* fb_docs, const int32_t* num_fb, int fb_cap, const RtWork& w,
                                   float* scores, cudaStream_t st) {
    rt_query_kernel<true, kW><<<nq, 256, 0, st>>>(rot, cbex, w.qtile, w.qem);
    CHM_TRY(launch_status("rt_query_kernel"));
    const size_t smem = refine_tc_smem_bytes<true, kW>();
    CHM_CUDA(cudaFuncSetAttribute(refine_tc_kernel<true, kW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid;
    CHM_TRY(rt_grid(refine_tc_kernel<true, kW>, smem, nq, w.icap, &grid));
    CHM_CUDA(cudaMemsetAsync(w.cand.count, 0, sizeof(int32_t) * nq, st));
    CHM_CUDA(cudaMemsetAsync(w.exact, 0, sizeof(uint32_t) * (size_t)nq * fb_cap * kQ, st));
    refine_tc_kernel<true, kW><<<grid, kRtThreads, smem, st>>>(w.meta, nullptr, idx->full_codes, idx->full_factors,
                                                               cbex, w.qtile, w.qem, w.icap, w.n_items, w.status,
                                                               w.stats, w.cand);
    CHM_TRY(launch_status("fullbit_tc_kernel"));
    return rt_finish<true, kW>(w.cand, idx->full_codes, idx->full_factors, rot, cbex, w.status, nq, fb_cap, w.exact,
                               fb_docs, num_fb, scores, st);
}

// full-bit rescoring of the queries flagged in `status` by the plain kernel
__global__ void flagged_counts_kernel(const uint32_t* status, const int32_t* num_fb, int32_t* out, int nq) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nq) out[i] = status[i] ? num_fb[i] : 0;
}
}  // namespace chm

chm_status chm_fullbit_flagged(const chm_index* idx, int32_t nq, const float* rot, const float* cbex,
                               const int32_t* fb_docs, const int32_t* counts, int32_t fb_cap, float* scores,
                               cudaStream_t st);

namespace chm {
static chm_status rescore_flagged_fullbit(const chm_index* idx, int nq, const float* rot, const float* cbex,
                                          const int32_t* fb_docs, const int32_t* num_fb, int fb_cap, float* scores,
                                          uint32_t* status, cudaStream_t st) {
    // the status array is reused as the per-query doc counts: 0 for queries
    // that succeeded, num_fb for flagged ones
    int32_t* counts = reinterpret_cast<int32_t*>(status);
    flagged_counts_kernel<<<(nq + 255) / 256, 256, 0, st>>>(status, num_fb, counts, nq);
    CHM_TRY(launch_status("flagged_counts_kernel"));
    return chm_fullbit_flagged(idx, nq, rot, cbex, fb_docs, counts, fb_cap, scores, st);
}
}  // namespace chm

extern "C" size_t chm_refine_1bit_tc_workspace_bytes(int32_t nq, int32_t k_refine) {
    if (nq <= 0 || k_refine <= 0) return 0;
    return chm::rt_bytes(nq, k_refine, k_refine);
}

extern "C" size_t chm_refine_tc_workspace_bytes(const chm_index* idx, int32_t nq, int32_t cap) {
    if (nq <= 0 || cap <= 0) return 0;
    return chm::rt_bytes(nq, cap, chm::rt_icap(idx, cap));
}

chm_status chm_refine_1bit_complete(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                                    const int32_t* refined_docs, const int32_t* num_refined, int32_t k_refine,
                                    float* scores, const int32_t* list, const int32_t* list_count,
                                    const uint32_t* status, cudaStream_t st);

extern "C" chm_status chm_refine_1bit_tc(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                                         const float* rot, const int32_t* refined_docs, const int32_t* num_refined,
                                         int32_t k_refine, float* scores, void* ws, size_t ws_bytes, void* stream) {
    if (nq <= 0) return CHM_OK;
    if (!idx || k_refine <= 0 || k_refine > CHM_MAX_K_REFINE) return CHM_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    chm::Arena a(ws, ws_bytes);
    chm::RtWork w;
    chm::rt_layout(a, nq, k_refine, chm::rt_call_icap(idx, nq, k_refine, ws_bytes), &w);
    if (a.overflow) return CHM_ERR_CAPACITY;
    // the token-order copies make each refined doc one contiguous span of codes
    const bool tok_order = idx->codes1_tok != nullptr && idx->factor1_tok != nullptr;
    const uint8_t* codes = tok_order ? idx->codes1_tok : idx->codes1;
    const float* factors = tok_order ? idx->factor1_tok : idx->factor1;
    CHM_TRY(chm::rt_plan(idx, nq, refined_docs, num_refined, k_refine, w, st));
    chm::rt_query_kernel<false, 1><<<nq, 256, 0, st>>>(rot, cb1, w.qtile, w.qem);
    CHM_TRY(chm::launch_status("rt_query_kernel"));
    const size_t smem = chm::refine_tc_smem_bytes<false, 1>();
    CHM_CUDA(cudaFuncSetAttribute(chm::refine_tc_kernel<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    dim3 grid;
    CHM_TRY(chm::rt_grid(chm::refine_tc_kernel<false, 1>, smem, nq, w.icap, &grid));
    CHM_CUDA(cudaMemsetAsync(w.cand.count, 0, sizeof(int32_t) * nq, st));
    CHM_CUDA(cudaMemsetAsync(w.exact, 0, sizeof(uint32_t) * (size_t)nq * k_refine * chm::kQ, st));
    chm::refine_tc_kernel<false, 1><<<grid, chm::kRtThreads, smem, st>>>(
        w.meta, tok_order ? nullptr : idx->tok2pos, codes, factors, cb1, w.qtile, w.qem, w.icap, w.n_items, w.status,
        w.stats, w.cand);
    CHM_TRY(chm::launch_status("refine_tc_kernel"));
    const chm_status fin = chm::rt_finish<false, 1>(w.cand, codes, factors, lut, cb1, w.status, nq, k_refine, w.exact,
                                                    refined_docs, num_refined, scores, st);
    if (fin != CHM_OK) return fin;
    return chm_refine_1bit_complete(idx, nq, lut, cb1, refined_docs, num_refined, k_refine, scores, w.big, w.n_big,
                                    w.status, st);
}

chm_status chm_fullbit_listed(const chm_index* idx, int32_t nq, const float* rot, const float* cbex,
                              const int32_t* fb_docs, const int32_t* num_fb, int32_t fb_cap, float* scores,
                              const int32_t* list, const int32_t* list_count, cudaStream_t st);

extern "C" size_t chm_fullbit_score_tc_workspace_bytes(int32_t nq, int32_t fb_cap) {
    return chm_refine_1bit_tc_workspace_bytes(nq, fb_cap);
}

extern "C" chm_status chm_fullbit_score_tc(const chm_index* idx, int32_t nq, const float* rot, const float* cbex,
                                           const int32_t* fb_docs, const int32_t* num_fb, int32_t fb_cap,
                                           float* scores, void* ws, size_t ws_bytes, void* stream) {
    if (nq <= 0) return CHM_OK;
    if (!idx || fb_cap <= 0 || fb_cap > CHM_MAX_K_REFINE) return CHM_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    const int w_bits = 1 + idx->ex_bits;
    if (w_bits < 2 || w_bits > 7)  // levels up to 255 (w = 8) do not fit the signed 8-bit operand
        return chm_fullbit_score(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, scores, stream);
    chm::Arena a(ws, ws_bytes);
    chm::RtWork w;
    chm::rt_layout(a, nq, fb_cap, chm::rt_call_icap(idx, nq, fb_cap, ws_bytes), &w);
    if (a.overflow) return CHM_ERR_CAPACITY;
    CHM_TRY(chm::rt_plan(idx, nq, fb_docs, num_fb, fb_cap, w, st));
    switch (w_bits) {
        case 2: CHM_TRY(chm::launch_fullbit_tc<2>(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, w, scores, st)); break;
        case 3: CHM_TRY(chm::launch_fullbit_tc<3>(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, w, scores, st)); break;
        case 4: CHM_TRY(chm::launch_fullbit_tc<4>(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, w, scores, st)); break;
        case 5: CHM_TRY(chm::launch_fullbit_tc<5>(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, w, scores, st)); break;
        case 6: CHM_TRY(chm::launch_fullbit_tc<6>(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, w, scores, st)); break;
        case 7: CHM_TRY(chm::launch_fullbit_tc<7>(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, w, scores, st)); break;
        default: return CHM_ERR_INVALID;
    }
    // long docs; then every doc of a query whose tensor-core launch failed
    CHM_TRY(chm_fullbit_listed(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, scores, w.big, w.n_big, st));
    return chm::rescore_flagged_fullbit(idx, nq, rot, cbex, fb_docs, num_fb, fb_cap, scores, w.status, st);
}
