// Stage 1: candidate generation and partial scoring.
//
// Replaces, for a batch of queries and with no host round trip, the
// reference's mark -> count -> ExclusiveSum -> host sync -> materialize ->
// partial_score -> sum_partial_scores -> full radix sort pipeline
// (kernels.cu:117-400, search_impl.cu:118-262).
//
//  score   : one CTA per (query token t, split, query); streams t's probed
//            lists in cluster order (coalesced 16 B code + 4 B factor + 4 B
//            doc id per element), 1-bit LUT inner product in the reference
//            order, and for dist > 0 inserts (doc, t, dist) into the query's
//            open-addressing table with max semantics.
//  combine : one warp per table bin; the entries homed at a bin are grouped
//            by doc and summed over the 32 query tokens with the reference's
//            tree (kernels.cu:192-198), giving 64-bit keys
//            (partial score bits << 32 | ~doc).
//  select  : one CTA per query; exact radix select of the top k_refine keys
//            and a bitonic sort (score desc, doc asc == stable descending
//            sort of ascending doc ids, search_impl.cu:245-261).
//  mark    : only for queries with fewer positive docs than k_refine: marks
//            every visited doc so zero-score candidates fill the refined list
//            in ascending doc order, as the reference's bitmap does.
//
// Table layout: u64 slots, key (doc << 5 | t) in the high word and the
// float bits of the max positive distance in the low word (positive floats
// order like their bit patterns, so a 64-bit atomicMax on a slot holding the
// same key keeps the larger distance).  A doc's entries are homed in one
// 32-slot bin (slot = bin * 32 + t) with linear probing, so every entry
// homed at bin b lies between slot 32b and the first empty slot at or after
// slot 32b + 31.
#include "common.cuh"

namespace chm {

constexpr uint64_t kEmpty = ~0ull;
constexpr int kScoreThreads = 256;
constexpr int kSelectThreads = 1024;

// Docs hash to 32-slot bins; a doc's entry for query token t starts probing
// at slot bin * 32 + t, so one warp load covers a bin.
constexpr int kBinShift = 5;

__device__ __forceinline__ uint32_t bin_of(uint32_t doc, uint32_t nbins_mask) {
    return (doc * 0x9E3779B1u) >> 7 & nbins_mask;
}

struct Stage1Ctx {
    const int64_t* cluster_pos;
    const uint8_t* codes1;
    const float* factor1;
    const int32_t* doc_ids;
    int64_t n_clusters;
    int64_t num_docs;
    const float* lut;       // [nq][32][512]
    const float* cb1;       // [nq][32]
    const uint32_t* labels; // [nq][32][nprobe]
    int nprobe;
    uint64_t* tables;       // [nq][H]
    int log2h;
    uint32_t* flags;        // [nq] bit0: table overflow
    const uint32_t* active; // [nq] nonzero: run this query (NULL: every query)
};

__device__ __forceinline__ bool inactive(const uint32_t* active, int q) { return active != nullptr && active[q] == 0u; }

__global__ void set_ones_kernel(uint32_t* out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = 1u;
}

// Clears the tables of the active queries (cudaMemsetAsync covers the all-active case).
__global__ void __launch_bounds__(256) stage1_clear_kernel(uint64_t* __restrict__ tables, int log2h,
                                                           const uint32_t* __restrict__ active) {
    const int q = blockIdx.y;
    if (inactive(active, q)) return;
    uint4* t = reinterpret_cast<uint4*>(tables + ((size_t)q << log2h));
    const size_t n = ((size_t)1 << log2h) / 2;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        t[i] = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
}

// Exclusive prefix over list lengths of one query token's probed lists.
__device__ void probe_prefix(const Stage1Ctx& c, const uint32_t* labels, int64_t* s_start,
                             int* s_prefix) {
    for (int p = threadIdx.x; p < c.nprobe; p += blockDim.x) {
        const uint32_t label = labels[p];
        if ((int64_t)label < c.n_clusters) {
            const int64_t st = c.cluster_pos[label];
            s_start[p] = st;
            s_prefix[p + 1] = (int)(c.cluster_pos[label + 1] - st);
        } else {
            s_start[p] = 0;
            s_prefix[p + 1] = 0;
        }
    }
    if (threadIdx.x == 0) s_prefix[0] = 0;
    __syncthreads();
    // Block-wide inclusive scan of s_prefix[1..nprobe] (nprobe <= 1024).
    for (int off = 1; off < c.nprobe; off <<= 1) {
        int add[4];
        int n = 0;
        for (int p = threadIdx.x; p < c.nprobe; p += blockDim.x, ++n)
            add[n] = (p >= off) ? s_prefix[p + 1 - off] : 0;
        __syncthreads();
        n = 0;
        for (int p = threadIdx.x; p < c.nprobe; p += blockDim.x, ++n) s_prefix[p + 1] += add[n];
        __syncthreads();
    }
}

__device__ __forceinline__ void table_insert(uint64_t* table, uint32_t hmask, uint32_t nbins_mask,
                                             uint32_t doc, int t, float dist, uint32_t* flag) {
    const uint32_t key = (doc << 5) | (uint32_t)t;
    const uint64_t val = ((uint64_t)key << 32) | __float_as_uint(dist);
    uint32_t slot = (bin_of(doc, nbins_mask) << kBinShift) + (uint32_t)t;
    for (uint32_t probe = 0; probe <= hmask; ++probe, slot = (slot + 1) & hmask) {
        uint64_t cur = table[slot];
        if (cur == kEmpty) {
            cur = atomicCAS((unsigned long long*)&table[slot], kEmpty, val);
            if (cur == kEmpty) return;
        }
        if ((uint32_t)(cur >> 32) == key) {
            if (val > cur) atomicMax((unsigned long long*)&table[slot], val);
            return;
        }
    }
    atomicOr(flag, 1u);
}

__global__ void __launch_bounds__(kScoreThreads) stage1_score_kernel(Stage1Ctx c, int splits) {
    __shared__ float s_lut[kLutPerQ];
    __shared__ int64_t s_start[CHM_MAX_NPROBE];
    __shared__ int s_prefix[CHM_MAX_NPROBE + 1];
    const int t = blockIdx.x / splits;
    const int split = blockIdx.x % splits;
    const int q = blockIdx.y;
    if (inactive(c.active, q)) return;
    const float* lut = c.lut + ((size_t)q * kQ + t) * kLutPerQ;
    for (int i = threadIdx.x; i < kLutPerQ; i += blockDim.x) s_lut[i] = lut[i];
    probe_prefix(c, c.labels + ((size_t)q * kQ + t) * c.nprobe, s_start, s_prefix);
    const int total = s_prefix[c.nprobe];
    const int per = (total + splits - 1) / splits;
    const int lo = split * per;
    const int hi = min(total, lo + per);
    const float cb1 = c.cb1[q * kQ + t];
    uint64_t* table = c.tables + ((size_t)q << c.log2h);
    const uint32_t hmask = (1u << c.log2h) - 1;
    const uint32_t nbins_mask = (1u << (c.log2h - kBinShift)) - 1;
    for (int v = lo + threadIdx.x; v < hi; v += blockDim.x) {
        // upper_bound over the prefix (lists are visited in label order)
        int a = 0, b = c.nprobe;
        while (a < b) {
            const int mid = (a + b) >> 1;
            if (s_prefix[mid + 1] <= v) a = mid + 1; else b = mid;
        }
        const int64_t pos = s_start[a] + (v - s_prefix[a]);
        const uint4 code = __ldg(reinterpret_cast<const uint4*>(c.codes1) + pos);
        const float f = __ldg(c.factor1 + pos);
        const int32_t doc = __ldg(c.doc_ids + pos);
        const float ip = lut_ip(s_lut, code);
        const float dist = fmul(fsub(ip, cb1), f);
        if (dist > 0.0f && doc >= 0 && (int64_t)doc < c.num_docs)
            table_insert(table, hmask, nbins_mask, (uint32_t)doc, t, dist, c.flags + q);
    }
}

// Marks every visited document (reference mark_candidate_documents_kernel,
// kernels.cu:206-278) for queries whose positive candidates fall short of
// k_refine.
__global__ void __launch_bounds__(kScoreThreads) stage1_mark_kernel(
    Stage1Ctx c, int splits, const uint32_t* n_pos, int k_refine, uint32_t* bitmaps,
    int64_t words) {
    __shared__ int64_t s_start[CHM_MAX_NPROBE];
    __shared__ int s_prefix[CHM_MAX_NPROBE + 1];
    const int t = blockIdx.x / splits;
    const int split = blockIdx.x % splits;
    const int q = blockIdx.y;
    if (inactive(c.active, q) || (int)n_pos[q] >= k_refine) return;
    probe_prefix(c, c.labels + ((size_t)q * kQ + t) * c.nprobe, s_start, s_prefix);
    const int total = s_prefix[c.nprobe];
    const int per = (total + splits - 1) / splits;
    const int lo = split * per;
    const int hi = min(total, lo + per);
    uint32_t* bm = bitmaps + (size_t)q * words;
    for (int v = lo + threadIdx.x; v < hi; v += blockDim.x) {
        int a = 0, b = c.nprobe;
        while (a < b) {
            const int mid = (a + b) >> 1;
            if (s_prefix[mid + 1] <= v) a = mid + 1; else b = mid;
        }
        const int64_t pos = s_start[a] + (v - s_prefix[a]);
        const int32_t doc = c.doc_ids[pos];
        if (doc >= 0 && (int64_t)doc < c.num_docs) atomicOr(bm + (doc >> 5), 1u << (doc & 31));
    }
}

constexpr int kCombineWarps = 8;
constexpr int kBinCap = 128;   // entries homed at one bin held in shared memory

// Tree sum (kernels.cu:192-198) of one doc whose entries sit in the warp's
// staged list: lane t picks the value for query token t (0 when absent) and
// the shuffle-down tree adds them in the reference order.
__device__ __forceinline__ float doc_tree_sum(const uint64_t* ent, int n, uint32_t doc, float* scratch) {
    const int lane = threadIdx.x & 31;
    scratch[lane] = 0.0f;
    __syncwarp();
    for (int j = lane; j < n; j += 32) {
        const uint64_t e = ent[j];
        if ((uint32_t)(e >> 37) == doc) scratch[(e >> 32) & 31] = __uint_as_float((uint32_t)e);
    }
    __syncwarp();
    float x = scratch[lane];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) x = fadd(x, __shfl_down_sync(0xffffffffu, x, off));
    __syncwarp();
    return __shfl_sync(0xffffffffu, x, 0);
}

// One warp per 32-slot bin.  The bin's own entries (homed here; the probe
// chain may run past the bin) are staged in shared memory and grouped by doc.
// A doc's partial score is the reference's tree over its 32 per-token maxima
// with zeros for absent tokens: with one entry that is the entry itself and
// with two it is their sum (adding zeros is exact), so only docs with three or
// more entries need the ordered tree.
__global__ void __launch_bounds__(kCombineWarps * 32) stage1_combine_kernel(
    const uint64_t* __restrict__ tables, int log2h, uint64_t* __restrict__ keys, int64_t key_cap,
    uint32_t* __restrict__ n_pos, uint32_t* __restrict__ flags, const uint32_t* __restrict__ active) {
    __shared__ uint64_t s_ent[kCombineWarps][kBinCap];
    __shared__ uint64_t s_out[kCombineWarps][2 * kBinCap];
    __shared__ float s_scr[kCombineWarps][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // queries vary fastest across the grid so that concurrently running blocks
    // spread their output-counter atomics over many queries
    const int q = blockIdx.x;
    if (inactive(active, q)) return;
    const uint32_t hmask = (1u << log2h) - 1;
    const uint32_t nbins = 1u << (log2h - kBinShift);
    const uint32_t nbins_mask = nbins - 1;
    const uint64_t* table = tables + ((size_t)q << log2h);
    uint64_t* out = keys + (size_t)q * key_cap;
    uint64_t* ent = s_ent[warp];
    int n_buf = 0;  // keys buffered in s_out[warp] over several bins, one counter atomic per flush
    auto flush = [&]() {
        uint32_t at = 0;
        if (lane == 0) at = atomicAdd(n_pos + q, (uint32_t)n_buf);
        at = __shfl_sync(0xffffffffu, at, 0);
        for (int j = lane; j < n_buf; j += 32) {
            if ((int64_t)at + j < key_cap) out[at + j] = s_out[warp][j];
            else atomicOr(flags + q, 4u);
        }
        n_buf = 0;
        __syncwarp();
    };
    // each warp walks bins with a stride of all the query's warps; no block barriers
    for (uint32_t bin = blockIdx.y * kCombineWarps + warp; bin < nbins; bin += gridDim.y * kCombineWarps) {
        const uint32_t first = bin << kBinShift;
        // 1) stage the bin's own entries
        int n = 0;
        for (uint32_t base = 0; base <= hmask; base += 32) {
            const uint64_t e = __ldcs(table + ((first + base + lane) & hmask));
            const bool empty = (e == kEmpty);
            const bool mine = !empty && bin_of((uint32_t)(e >> 37), nbins_mask) == bin;
            const uint32_t mb = __ballot_sync(0xffffffffu, mine);
            if (mine) {
                const int at = n + __popc(mb & ((1u << lane) - 1));
                if (at < kBinCap) ent[at] = e;
            }
            n += __popc(mb);
            // the chain ends at the first empty slot at or after slot 32 * bin + 31
            if (__ballot_sync(0xffffffffu, empty && (base + lane) >= 31)) break;
        }
        if (n > kBinCap) {
            if (lane == 0) atomicOr(flags + q, 2u);
            n = kBinCap;
        }
        __syncwarp();
        if (n_buf > kBinCap) flush();  // room for this bin's (at most kBinCap) keys
        uint64_t* outb = s_out[warp] + n_buf;
        int n_out = 0;
        if (n <= 32) {
            const bool act = lane < n;
            const uint64_t e = act ? ent[lane] : kEmpty;
            const uint32_t doc = act ? (uint32_t)(e >> 37) : 0xFFFFFFFFu;
            const float val = __uint_as_float((uint32_t)e);
            const uint32_t grp = __match_any_sync(0xffffffffu, doc);
            const int cnt = __popc(grp);
            const int lead = __ffs(grp) - 1;
            const float partner = __shfl_sync(0xffffffffu, val, 31 - __clz(grp));  // highest lane of the group
            const bool leader = act && lane == lead;
            // singles and pairs finish lane-parallel
            const bool easy = leader && cnt <= 2;
            const uint32_t eb = __ballot_sync(0xffffffffu, easy);
            if (easy) {
                const float x = cnt == 1 ? val : fadd(val, partner);
                outb[__popc(eb & ((1u << lane) - 1))] = ((uint64_t)__float_as_uint(x) << 32) | (uint32_t)(~doc);
            }
            n_out = __popc(eb);
            // docs with three or more entries: ordered tree, one doc at a time
            uint32_t hard = __ballot_sync(0xffffffffu, leader && cnt > 2);
            while (hard) {
                const int l = __ffs(hard) - 1;
                hard &= hard - 1;
                const uint32_t d = __shfl_sync(0xffffffffu, doc, l);
                const float x = doc_tree_sum(ent, n, d, s_scr[warp]);
                if (lane == 0) outb[n_out] = ((uint64_t)__float_as_uint(x) << 32) | (uint32_t)(~d);
                ++n_out;
            }
        } else {
            // rare (a crowded bin): the first entry of each doc in the staged list
            // leads its doc through the ordered tree
            for (int i = 0; i < n; ++i) {
                const uint32_t d = (uint32_t)(ent[i] >> 37);
                bool seen = false;
                for (int j = lane; j < i; j += 32) seen |= ((uint32_t)(ent[j] >> 37) == d);
                if (__any_sync(0xffffffffu, seen)) continue;
                const float x = doc_tree_sum(ent, n, d, s_scr[warp]);
                if (lane == 0 && n_out < kBinCap) outb[n_out] = ((uint64_t)__float_as_uint(x) << 32) | (uint32_t)(~d);
                ++n_out;
            }
        }
        n_buf += n_out;
        __syncwarp();  // the staging buffer is reused by the next bin
    }
    if (n_buf) flush();
}

// ---- block helpers for the select kernel ---------------------------------
// Exclusive scan over one value per thread (blockDim 1024), in thread order.
__device__ uint32_t block_excl_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
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
        uint32_t w = s_warp[lane];
        uint32_t z = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, z, off);
            if (lane >= off) z += y;
        }
        s_warp[lane] = z - w;  // exclusive warp offsets
        if (lane == 31) s_warp[32] = z;
    }
    __syncthreads();
    const uint32_t r = s_warp[warp] + x - v;
    *total = s_warp[32];
    __syncthreads();
    return r;
}

// Bitonic sort, descending, of n (power of two) 64-bit keys in shared memory.
__device__ void block_sort_desc(uint64_t* a, int n) {
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

// Is `doc` present in the query's table (any query token)?
__device__ bool table_has_doc(const uint64_t* table, uint32_t hmask, uint32_t nbins_mask,
                              uint32_t doc) {
    const uint32_t first = bin_of(doc, nbins_mask) << kBinShift;
    for (uint32_t i = 0; i <= hmask; ++i) {
        const uint64_t e = table[(first + i) & hmask];
        if (e == kEmpty) { if (i >= 31) return false; else continue; }
        if ((uint32_t)(e >> 37) == doc) return true;
    }
    return false;
}

// ---- pre-selection for long key lists ------------------------------------
// The select kernel runs one CTA per query; over a list of ~10^6 keys its
// radix passes are bound by one SM's bandwidth.  Three wide passes first cut
// each long list down to the keys at or above the 12-bit bucket that holds
// the k_refine-th largest key: a histogram of the top 12 bits per (query,
// slice), the bucket per query, and a compaction.  The select kernel then
// runs on the compacted keys, which hold every key of the top k_refine.
constexpr int kPreThreads = 256;
constexpr int64_t kPreCap = 65536;        // compacted keys per query (more: the full list is used)
constexpr uint32_t kNoPivot = 0xFFFFFFFFu;

__global__ void __launch_bounds__(kPreThreads) stage1_hist_kernel(const uint64_t* __restrict__ keys, int64_t key_cap,
                                                                  const uint32_t* __restrict__ n_pos, int k_refine,
                                                                  uint32_t* __restrict__ hist) {
    __shared__ uint32_t h[4096];
    const int q = blockIdx.y;
    const int64_t n = min((int64_t)n_pos[q], key_cap);
    for (int i = threadIdx.x; i < 4096; i += blockDim.x) h[i] = 0;
    __syncthreads();
    if (n > k_refine) {
        const int64_t per = (n + gridDim.x - 1) / gridDim.x;
        const int64_t i0 = blockIdx.x * per, i1 = min(n, i0 + per);
        const uint64_t* qk = keys + (size_t)q * key_cap;
        for (int64_t i = i0 + threadIdx.x; i < i1; i += 4 * (int64_t)blockDim.x) {
            uint64_t k4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t j = i + u * (int64_t)blockDim.x;
                k4[u] = j < i1 ? __ldcs(qk + j) : 0;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i + u * (int64_t)blockDim.x < i1) atomicAdd(&h[(uint32_t)(k4[u] >> 52)], 1u);
        }
    }
    __syncthreads();
    uint32_t* out = hist + ((size_t)q * gridDim.x + blockIdx.x) * 4096;
    for (int i = threadIdx.x; i < 4096; i += blockDim.x) out[i] = h[i];
}

// Per query: the highest bucket d such that the keys in buckets >= d number
// at least k_refine (kNoPivot for lists of at most k_refine keys).
__global__ void __launch_bounds__(kSelectThreads) stage1_pivot_kernel(const uint32_t* __restrict__ hist, int slices,
                                                                      const uint32_t* __restrict__ n_pos,
                                                                      int64_t key_cap, int k_refine,
                                                                      uint32_t* __restrict__ pivot,
                                                                      uint32_t* __restrict__ ccnt) {
    __shared__ uint32_t s_warp[33];
    const int q = blockIdx.x;
    const int64_t n = min((int64_t)n_pos[q], key_cap);
    if (n <= k_refine) {
        if (threadIdx.x == 0) {
            pivot[q] = kNoPivot;
            ccnt[q] = 0;
        }
        return;
    }
    // thread t owns buckets [4095 - 4t - 3, 4095 - 4t] (descending order)
    const int top = 4095 - 4 * threadIdx.x;
    uint32_t c[4] = {0, 0, 0, 0};
    for (int sl = 0; sl < slices; ++sl) {
        const uint32_t* hs = hist + ((size_t)q * slices + sl) * 4096;
#pragma unroll
        for (int j = 0; j < 4; ++j) c[j] += hs[top - j];
    }
    const uint32_t mine = c[0] + c[1] + c[2] + c[3];
    uint32_t total;
    const uint32_t before = block_excl_scan(mine, s_warp, &total);
    if ((int64_t)before < k_refine && (int64_t)(before + mine) >= k_refine) {
        uint32_t cum = before;
        for (int j = 0; j < 4; ++j) {
            cum += c[j];
            if ((int64_t)cum >= k_refine) {
                pivot[q] = (uint32_t)(top - j);
                break;
            }
        }
    }
    if (threadIdx.x == 0) ccnt[q] = 0;
}

// Appends each query's keys in buckets >= pivot to its compacted list.
__global__ void __launch_bounds__(kPreThreads) stage1_compact_kernel(const uint64_t* __restrict__ keys, int64_t key_cap,
                                                                     const uint32_t* __restrict__ n_pos,
                                                                     const uint32_t* __restrict__ pivot,
                                                                     uint64_t* __restrict__ ckeys,
                                                                     uint32_t* __restrict__ ccnt) {
    const int q = blockIdx.y;
    const uint32_t d = pivot[q];
    if (d == kNoPivot) return;
    const int64_t n = min((int64_t)n_pos[q], key_cap);
    const int64_t per = (n + gridDim.x - 1) / gridDim.x;
    const int64_t i0 = blockIdx.x * per, i1 = min(n, i0 + per);
    const uint64_t* qk = keys + (size_t)q * key_cap;
    uint64_t* out = ckeys + (size_t)q * kPreCap;
    const int lane = threadIdx.x & 31;
    // uniform trip count (the ballots need every lane); four loads in flight per thread
    for (int64_t b = i0; b < i1; b += 4 * (int64_t)blockDim.x) {
        uint64_t k4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t i = b + u * (int64_t)blockDim.x + threadIdx.x;
            k4[u] = i < i1 ? __ldcs(qk + i) : 0;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t i = b + u * (int64_t)blockDim.x + threadIdx.x;
            const bool keep = i < i1 && (uint32_t)(k4[u] >> 52) >= d;
            const uint32_t m = __ballot_sync(0xffffffffu, keep);
            if (m) {
                uint32_t base = 0;
                if (lane == 0) base = atomicAdd(ccnt + q, (uint32_t)__popc(m));
                base = __shfl_sync(0xffffffffu, base, 0);
                const uint32_t at = base + __popc(m & ((1u << lane) - 1));
                if (keep && at < (uint32_t)kPreCap) out[at] = k4[u];
            }
        }
    }
}

__global__ void __launch_bounds__(kSelectThreads) stage1_select_kernel(
    const uint64_t* __restrict__ keys, int64_t key_cap, const uint32_t* __restrict__ n_pos,
    int k_refine, const uint32_t* __restrict__ bitmaps, int64_t words,
    const uint64_t* __restrict__ tables, int log2h, int marks_all,
    int32_t* __restrict__ refined_docs, float* __restrict__ refined_partial,
    int32_t* __restrict__ num_refined, int64_t* __restrict__ num_candidates,
    uint32_t* __restrict__ flags, const uint64_t* __restrict__ ckeys, const uint32_t* __restrict__ ccnt,
    const uint32_t* __restrict__ pivot, const uint32_t* __restrict__ active) {
    extern __shared__ uint64_t s_dyn[];
    uint64_t* s_out = s_dyn;                                   // [sort_n]
    __shared__ uint32_t s_hist[4096];
    __shared__ uint32_t s_warp[33];
    __shared__ uint32_t s_cnt;
    __shared__ uint64_t s_prefix, s_pmask;
    __shared__ int s_need, s_done;
    const int q = blockIdx.x;
    if (inactive(active, q)) return;
    // a long list's compacted keys (all keys of its top k_refine), unless they overflowed
    const bool compacted = pivot[q] != kNoPivot && ccnt[q] <= (uint32_t)kPreCap;
    const uint64_t* qk = compacted ? ckeys + (size_t)q * kPreCap : keys + (size_t)q * key_cap;
    const int64_t n = compacted ? (int64_t)ccnt[q] : min((int64_t)n_pos[q], key_cap);
    if ((int64_t)n_pos[q] > key_cap && threadIdx.x == 0) atomicOr(flags + q, 4u);
    const int k_eff = (int)min((int64_t)k_refine, n);
    if (threadIdx.x == 0) { s_cnt = 0; s_prefix = 0; s_pmask = 0; s_need = k_eff; s_done = 0; }
    __syncthreads();
    if (n <= k_refine) {
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s_out[i] = qk[i];
        if (threadIdx.x == 0) s_cnt = (uint32_t)n;
        __syncthreads();
    } else {
        // radix select of the k_eff largest keys: 12-bit digits from the top
        const int shifts[6] = {52, 40, 28, 16, 4, 0};
        const int widths[6] = {12, 12, 12, 12, 12, 4};
        for (int lv = 0; lv < 6; ++lv) {
            if (s_done) break;
            const int sh = shifts[lv];
            const uint32_t dmask = (1u << widths[lv]) - 1;
            for (int i = threadIdx.x; i < 4096; i += blockDim.x) s_hist[i] = 0;
            __syncthreads();
            const uint64_t prefix = s_prefix, pmask = s_pmask;
            // four independent loads in flight per thread
            for (int64_t i0 = threadIdx.x; i0 < n; i0 += 4 * (int64_t)blockDim.x) {
                uint64_t k4[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t i = i0 + u * (int64_t)blockDim.x;
                    k4[u] = i < n ? __ldcg(qk + i) : ~prefix;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (i0 + u * (int64_t)blockDim.x < n && (k4[u] & pmask) == prefix)
                        atomicAdd(&s_hist[(k4[u] >> sh) & dmask], 1u);
            }
            __syncthreads();
            // thread t owns digits [4095-4t-3, 4095-4t] (descending order)
            uint32_t mine = 0;
            const int top = 4095 - 4 * threadIdx.x;
            for (int j = 0; j < 4; ++j) mine += s_hist[top - j];
            uint32_t total;
            const uint32_t before = block_excl_scan(mine, s_warp, &total);
            const int need = s_need;
            if ((int)before < need && need <= (int)(before + mine)) {
                uint32_t cum = before;
                for (int j = 0; j < 4; ++j) {
                    const uint32_t h = s_hist[top - j];
                    if ((int)(cum + h) >= need) {
                        const uint32_t d = (uint32_t)(top - j);
                        s_prefix = prefix | ((uint64_t)d << sh);
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
        for (int64_t i0 = threadIdx.x; i0 < n; i0 += 4 * (int64_t)blockDim.x) {
            uint64_t k4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t i = i0 + u * (int64_t)blockDim.x;
                k4[u] = i < n ? __ldcg(qk + i) : 0;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (i0 + u * (int64_t)blockDim.x < n && (k4[u] & pmask) >= prefix) {
                    const uint32_t at = atomicAdd(&s_cnt, 1u);
                    if (at < (uint32_t)k_eff) s_out[at] = k4[u];
                }
            }
        }
        __syncthreads();
        if (threadIdx.x == 0 && s_cnt != (uint32_t)k_eff) atomicOr(flags + q, 8u);
        if (threadIdx.x == 0) s_cnt = (uint32_t)k_eff;
        __syncthreads();
    }
    // zero-score fill in ascending doc order (only when positives < k_refine)
    int64_t n_cand = -1;
    const bool short_list = (int64_t)n_pos[q] < k_refine;
    if ((short_list || marks_all) && bitmaps != nullptr) {
        const uint32_t* bm = bitmaps + (size_t)q * words;
        const uint64_t* table = tables + ((size_t)q << log2h);
        const uint32_t hmask = (1u << log2h) - 1;
        const uint32_t nbins_mask = (1u << (log2h - kBinShift)) - 1;
        const int64_t per = (words + blockDim.x - 1) / blockDim.x;
        const int64_t w0 = threadIdx.x * per, w1 = min(words, w0 + per);
        uint32_t zeros = 0, marked = 0;
        for (int64_t w = w0; w < w1; ++w) {
            uint32_t bits = bm[w];
            marked += __popc(bits);
            while (bits) {
                const int b = __ffs(bits) - 1;
                bits &= bits - 1;
                if (!table_has_doc(table, hmask, nbins_mask, (uint32_t)(w * 32 + b))) ++zeros;
            }
        }
        uint32_t tot_marked;
        block_excl_scan(marked, s_warp, &tot_marked);
        uint32_t tot_zero;
        uint32_t at = block_excl_scan(zeros, s_warp, &tot_zero);
        const int base = (int)s_cnt;
        const int room = short_list ? k_refine - base : 0;
        for (int64_t w = w0; w < w1 && (int)at < room; ++w) {
            uint32_t bits = bm[w];
            while (bits && (int)at < room) {
                const int b = __ffs(bits) - 1;
                bits &= bits - 1;
                const uint32_t doc = (uint32_t)(w * 32 + b);
                if (!table_has_doc(table, hmask, nbins_mask, doc)) s_out[base + at++] = (uint32_t)(~doc);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0 && short_list) s_cnt = (uint32_t)min(k_refine, base + (int)tot_zero);
        n_cand = tot_marked;
        __syncthreads();
    }
    const int cnt = (int)s_cnt;
    int sort_n = 1;
    while (sort_n < cnt) sort_n <<= 1;
    for (int i = cnt + threadIdx.x; i < sort_n; i += blockDim.x) s_out[i] = 0;
    __syncthreads();
    block_sort_desc(s_out, sort_n);
    for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
        const uint64_t key = s_out[i];
        refined_docs[(size_t)q * k_refine + i] = (int32_t)(~(uint32_t)key);
        refined_partial[(size_t)q * k_refine + i] = __uint_as_float((uint32_t)(key >> 32));
    }
    if (threadIdx.x == 0) {
        num_refined[q] = cnt;
        if (num_candidates) num_candidates[q] = n_cand;
    }
}

}  // namespace chm

namespace chm {
int stage1_log2h(const chm_index* idx, int nprobe, int extra) {
    const double mean_list = idx->n_clusters > 0 ? (double)idx->n_tokens / (double)idx->n_clusters : 0;
    double want = 2.0 * kQ * (double)nprobe * (mean_list > 1 ? mean_list : 1);
    if (want < 4096) want = 4096;
    int l = 12;
    while ((double)(1ull << l) < want && l < 30) ++l;
    l += extra;
    return l > 31 ? 31 : l;
}
int64_t stage1_key_cap(const chm_index* idx) { return idx->num_docs; }
// CTAs per query of the pre-selection passes: about four per SM in all.
// nq x slices stays within max(nq, kPreSlots), so the histogram area sized
// for a batch also holds any smaller chunk's.
constexpr int kPreSlots = 640;
int stage1_pre_slices(int nq) { return std::max(1, std::min(64, kPreSlots / std::max(1, nq))); }
size_t stage1_hist_words(int nq) { return (size_t)std::max(nq, kPreSlots) * 4096; }
int64_t stage1_words(const chm_index* idx) { return (idx->num_docs + 31) / 32; }
}  // namespace chm

namespace chm {
size_t bound_bytes(const chm_index* idx, int nq, int nprobe, int k_refine);
bool bound_enabled(const chm_index* idx, int nprobe, int k_refine);
chm_status bound_run(const chm_index* idx, int nq, const float* lut, const float* cb1, const uint32_t* labels,
                     int nprobe, int k_refine, int32_t* refined_docs, float* refined_partial, int32_t* num_refined,
                     uint32_t* need_fb, void* ws, size_t ws_bytes, cudaStream_t st);

// Workspace: the hash-table path's arrays, then (when the index enables it)
// the dense-bound path's.
template <typename A>
struct Stage1Layout {
    uint64_t* tables;
    uint64_t* keys;
    uint32_t* bitmaps;
    uint32_t* n_pos;
    uint32_t* flags;
    uint32_t* hist;
    uint32_t* pivot;
    uint32_t* ccnt;
    uint64_t* ckeys;
    uint32_t* need_fb;
    void* bound_ws;
    size_t bound_bytes;
};

template <typename A>
static void stage1_layout(A& a, const chm_index* idx, int nq, int nprobe, int extra, size_t bbytes,
                          Stage1Layout<A>* o) {
    const int l = stage1_log2h(idx, nprobe, extra);
    auto tables = a.template take<uint64_t>((size_t)nq << l);
    auto keys = a.template take<uint64_t>((size_t)nq * stage1_key_cap(idx));
    auto bitmaps = a.template take<uint32_t>((size_t)nq * stage1_words(idx));
    auto n_pos = a.template take<uint32_t>((size_t)nq);
    auto flags = a.template take<uint32_t>((size_t)nq);
    auto hist = a.template take<uint32_t>(stage1_hist_words(nq));
    auto pivot = a.template take<uint32_t>((size_t)nq);
    auto ccnt = a.template take<uint32_t>((size_t)nq);
    auto ckeys = a.template take<uint64_t>((size_t)nq * kPreCap);
    auto need_fb = a.template take<uint32_t>((size_t)nq);
    auto bws = a.template take<char>(bbytes);
    if (o)
        *o = Stage1Layout<A>{(uint64_t*)tables, (uint64_t*)keys, (uint32_t*)bitmaps, (uint32_t*)n_pos,
                             (uint32_t*)flags, (uint32_t*)hist, (uint32_t*)pivot, (uint32_t*)ccnt, (uint64_t*)ckeys,
                             (uint32_t*)need_fb, (void*)bws, bbytes};
}

struct S1Sizer {
    Sizer s;
    template <typename T>
    void* take(size_t n) {
        s.take<T>(n);
        return nullptr;
    }
};

size_t stage1_bytes(const chm_index* idx, int32_t nq, int32_t nprobe, int extra, int k_refine) {
    S1Sizer s;
    stage1_layout(s, idx, nq, nprobe, extra, bound_bytes(idx, nq, nprobe, k_refine), (Stage1Layout<S1Sizer>*)nullptr);
    return s.s.off;
}
}  // namespace chm

extern "C" size_t chm_stage1_workspace_bytes(const chm_index* idx, int32_t nq, int32_t nprobe,
                                             int32_t k_refine) {
    return chm::stage1_bytes(idx, nq, nprobe, 0, k_refine);
}

namespace chm {
// The hash-table path over the queries `active` selects (NULL: all).
static chm_status stage1_table_run(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                                   const uint32_t* labels, int32_t nprobe, int32_t k_refine, int32_t* refined_docs,
                                   float* refined_partial, int32_t* num_refined, int64_t* num_candidates,
                                   const Stage1Layout<Arena>& w, int l, cudaStream_t st, bool force_marks,
                                   const uint32_t* active) {
    const int64_t key_cap = stage1_key_cap(idx);
    const int64_t words = stage1_words(idx);
    const int slices = stage1_pre_slices(nq);
    if (active == nullptr) {
        CHM_CUDA(cudaMemsetAsync(w.tables, 0xFF, sizeof(uint64_t) * ((size_t)nq << l), st));
    } else {
        stage1_clear_kernel<<<dim3(256u, (unsigned)nq), 256, 0, st>>>(w.tables, l, active);
        CHM_TRY(launch_status("stage1_clear_kernel"));
    }
    Stage1Ctx c{idx->cluster_pos, idx->codes1, idx->factor1, idx->doc_ids, idx->n_clusters,
                idx->num_docs, lut, cb1, labels, nprobe, w.tables, l, w.flags, active};
    const double mean_list = (double)idx->n_tokens / (double)(idx->n_clusters > 0 ? idx->n_clusters : 1);
    const double visits_per_t = nprobe * mean_list;
    int splits = (int)(visits_per_t / (kScoreThreads * 8));
    if (splits < 1) splits = 1;
    if (splits > 64) splits = 64;
    dim3 g1(kQ * splits, nq);
    stage1_score_kernel<<<g1, kScoreThreads, 0, st>>>(c, splits);
    CHM_TRY(launch_status("stage1_score_kernel"));
    const int64_t nbins = 1ll << (l - kBinShift);
    // enough blocks for about 8 resident per SM over all queries; warps stride over bins
    const int64_t want_blocks = std::max<int64_t>(1, (int64_t)148 * 8 * 4 / std::max(1, nq));
    dim3 g2(nq, (unsigned)std::min<int64_t>(std::min<int64_t>(nbins / kCombineWarps, want_blocks), 65535));
    stage1_combine_kernel<<<g2, kCombineWarps * 32, 0, st>>>(w.tables, l, w.keys, key_cap, w.n_pos, w.flags, active);
    CHM_TRY(launch_status("stage1_combine_kernel"));
    CHM_CUDA(cudaMemsetAsync(w.bitmaps, 0, sizeof(uint32_t) * (size_t)nq * words, st));
    // queries whose positives fall short of k_refine get the visited-doc bitmap
    stage1_mark_kernel<<<g1, kScoreThreads, 0, st>>>(c, splits, w.n_pos, force_marks ? (1 << 30) : k_refine,
                                                     w.bitmaps, words);
    CHM_TRY(launch_status("stage1_mark_kernel"));
    int sort_cap = 1;
    while (sort_cap < k_refine) sort_cap <<= 1;
    const size_t smem = sizeof(uint64_t) * sort_cap;
    // static (histogram) + dynamic (sort buffer) can exceed the 48 KB default
    CHM_CUDA(cudaFuncSetAttribute(stage1_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    stage1_hist_kernel<<<dim3((unsigned)slices, (unsigned)nq), kPreThreads, 0, st>>>(w.keys, key_cap, w.n_pos,
                                                                                    k_refine, w.hist);
    CHM_TRY(launch_status("stage1_hist_kernel"));
    stage1_pivot_kernel<<<nq, kSelectThreads, 0, st>>>(w.hist, slices, w.n_pos, key_cap, k_refine, w.pivot, w.ccnt);
    CHM_TRY(launch_status("stage1_pivot_kernel"));
    stage1_compact_kernel<<<dim3((unsigned)slices, (unsigned)nq), kPreThreads, 0, st>>>(w.keys, key_cap, w.n_pos,
                                                                                       w.pivot, w.ckeys, w.ccnt);
    CHM_TRY(launch_status("stage1_compact_kernel"));
    stage1_select_kernel<<<nq, kSelectThreads, smem, st>>>(
        w.keys, key_cap, w.n_pos, k_refine, w.bitmaps, words, w.tables, l, force_marks ? 1 : 0, refined_docs,
        refined_partial, num_refined, num_candidates, w.flags, w.ckeys, w.ccnt, w.pivot, active);
    return launch_status("stage1_select_kernel");
}

// extra_log2h lets the host retry a query batch with a larger table.
chm_status stage1_run(const chm_index* idx, int32_t nq, const float* lut, const float* cb1,
                      const uint32_t* labels, int32_t nprobe, int32_t k_refine,
                      int32_t* refined_docs, float* refined_partial, int32_t* num_refined,
                      int64_t* num_candidates, void* ws, size_t ws_bytes, cudaStream_t st,
                      bool force_marks, uint32_t* flags_out, int log2_extra) {
    if (nq <= 0) return CHM_OK;
    if (nprobe <= 0 || nprobe > CHM_MAX_NPROBE || k_refine <= 0 || k_refine > CHM_MAX_K_REFINE)
        return CHM_ERR_INVALID;
    if (idx->num_docs >= (1ll << 27)) return CHM_ERR_UNSUPPORTED;
    const int l = stage1_log2h(idx, nprobe, log2_extra);
    // the dense-bound path first (not for the candidate counts, which need
    // every visited doc); the hash-table path redoes the queries it flags
    const bool bound = !force_marks && bound_enabled(idx, nprobe, k_refine);
    Arena a(ws, ws_bytes);
    Stage1Layout<Arena> w;
    stage1_layout(a, idx, nq, nprobe, log2_extra, bound ? bound_bytes(idx, nq, nprobe, k_refine) : 0, &w);
    if (a.overflow) return CHM_ERR_CAPACITY;
    CHM_CUDA(cudaMemsetAsync(w.n_pos, 0, sizeof(uint32_t) * nq, st));
    CHM_CUDA(cudaMemsetAsync(w.flags, 0, sizeof(uint32_t) * nq, st));
    if (bound) {
        CHM_TRY(bound_run(idx, nq, lut, cb1, labels, nprobe, k_refine, refined_docs, refined_partial, num_refined,
                          w.need_fb, w.bound_ws, w.bound_bytes, st));
        CHM_TRY(stage1_table_run(idx, nq, lut, cb1, labels, nprobe, k_refine, refined_docs, refined_partial,
                                 num_refined, num_candidates, w, l, st, force_marks, w.need_fb));
    } else {
        set_ones_kernel<<<(nq + 255) / 256, 256, 0, st>>>(w.need_fb, nq);  // for chm_stage1_table_queries
        CHM_TRY(launch_status("set_ones_kernel"));
        CHM_TRY(stage1_table_run(idx, nq, lut, cb1, labels, nprobe, k_refine, refined_docs, refined_partial,
                                 num_refined, num_candidates, w, l, st, force_marks, nullptr));
    }
    if (flags_out) CHM_CUDA(cudaMemcpyAsync(flags_out, w.flags, sizeof(uint32_t) * nq, cudaMemcpyDeviceToDevice, st));
    return CHM_OK;
}
}  // namespace chm

extern "C" chm_status chm_stage1(const chm_index* idx, int32_t nq, const float* lut,
                                 const float* cb1, const uint32_t* labels, int32_t nprobe,
                                 int32_t k_refine, int32_t* refined_docs, float* refined_partial,
                                 int32_t* num_refined, int64_t* num_candidates, void* ws,
                                 size_t ws_bytes, void* stream) {
    return chm::stage1_run(idx, nq, lut, cb1, labels, nprobe, k_refine, refined_docs,
                           refined_partial, num_refined, num_candidates, ws, ws_bytes,
                           (cudaStream_t)stream, num_candidates != nullptr, nullptr, 0);
}

extern "C" chm_status chm_stage1_table_queries(const chm_index* idx, int32_t nq, int32_t nprobe, int32_t k_refine,
                                               int32_t table_log2_extra, const void* ws, size_t ws_bytes,
                                               uint32_t* out, void* stream) {
    if (!idx || nq <= 0 || !out) return CHM_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    const bool bound = chm::bound_enabled(idx, nprobe, k_refine);
    if (!bound) {  // every query took the hash-table path
        chm::set_ones_kernel<<<(nq + 255) / 256, 256, 0, st>>>(out, nq);
        return chm::launch_status("set_ones_kernel");
    }
    chm::Arena a(const_cast<void*>(ws), ws_bytes);
    chm::Stage1Layout<chm::Arena> w;
    chm::stage1_layout(a, idx, nq, nprobe, table_log2_extra, chm::bound_bytes(idx, nq, nprobe, k_refine), &w);
    if (a.overflow) return CHM_ERR_CAPACITY;
    CHM_CUDA(cudaMemcpyAsync(out, w.need_fb, sizeof(uint32_t) * nq, cudaMemcpyDeviceToDevice, st));
    return CHM_OK;
}
