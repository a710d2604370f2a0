// Chimera::chimera_index on top of the chimera_b200 C ABI.
//
// Public behaviour follows the reference (cpp/src/chimera_index.cu,
// build_index.cu, search_impl.cu): the same input validation and exception
// types, the same six-file index directory (with the rotated centroids in
// centroids.f32 instead of a cuVS CAGRA graph), lazy search-state set-up after
// build(), device 0, not thread-safe.  The work itself runs on the GPU:
// assignment, rotation and RaBitQ encoding at build time, and the whole search
// (including the full-bit stage the reference runs on the CPU) at query time.
#include "chimera/chimera_index.cuh"

#include <algorithm>
#include <array>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <limits>
#include <numeric>

#include "chimera_b200.h"

extern "C" void chm_host_fhtkac_flips(uint64_t seed, uint8_t* out, size_t n);
extern "C" void chm_host_sample_centroids(uint64_t num_embeddings, uint64_t n_clusters, uint64_t seed,
                                          uint64_t* ids);

namespace Chimera {
namespace {

constexpr size_t kPadded = CHM_PADDED_DIM;
constexpr size_t kQ = CHM_QLEN;
constexpr uint64_t kRotatorSeed = 42;
constexpr uint64_t kCentroidSeed = 42;
constexpr const char* kCentroidFile = "centroids.f32";

struct IndexHeader {  // cpp/include/chimera/chimera_index.cuh:75-81
    size_t num_embeddings;
    size_t dimension;
    size_t num_clusters;
    size_t ex_bits;
    size_t padded_dimension;
};

// The rotated centroids inside a cuVS CAGRA file (centroids.carga, written
// by the reference's IVF_PG::save, ivf_pg.cpp:136-137, over the rotated
// centroids, build_index.cu:440-446).  cuVS serialises the index's arrays as
// NumPy .npy blocks (magic "\x93NUMPY", a header dict with 'descr' and
// 'shape', then the raw data); the dataset block is the little-endian fp32
// array of shape (n_clusters, d), d <= 128, when the file was written with
// the dataset included (cuVS's default).  Scans the file's .npy blocks for
// it; false when there is none.
bool read_carga_centroids(const std::string& path, size_t n_clusters, std::vector<float>& out) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) return false;
    const std::streamoff size = f.tellg();
    static const char kMagic[6] = {'\x93', 'N', 'U', 'M', 'P', 'Y'};
    std::vector<char> buf(1 << 20);
    std::streamoff pos = 0;
    while (pos + 10 <= size) {
        // next magic at or after pos
        f.seekg(pos);
        const std::streamoff want = std::min<std::streamoff>((std::streamoff)buf.size(), size - pos);
        f.read(buf.data(), want);
        if (!f) return false;
        std::streamoff hit = -1;
        for (std::streamoff i = 0; i + 6 <= want; ++i)
            if (std::memcmp(buf.data() + i, kMagic, 6) == 0) {
                hit = pos + i;
                break;
            }
        if (hit < 0) {
            if (pos + want >= size) return false;
            pos += want - 5;  // a magic may straddle the block boundary
            continue;
        }
        // preamble: magic, major, minor, header length (2 bytes in 1.x, 4 after)
        unsigned char pre[12] = {0};
        f.seekg(hit);
        f.read(reinterpret_cast<char*>(pre), 12);
        if (!f) return false;
        const int major = pre[6];
        size_t hlen = 0, off = 0;
        if (major == 1) {
            hlen = pre[8] | (size_t(pre[9]) << 8);
            off = 10;
        } else {
            hlen = pre[8] | (size_t(pre[9]) << 8) | (size_t(pre[10]) << 16) | (size_t(pre[11]) << 24);
            off = 12;
        }
        if (hlen > (1 << 16)) {  // not a real header: keep scanning
            pos = hit + 1;
            continue;
        }
        std::string hdr(hlen, '\0');
        f.seekg(hit + (std::streamoff)off);
        f.read(&hdr[0], (std::streamsize)hlen);
        if (!f) return false;
        const std::streamoff data = hit + (std::streamoff)(off + hlen);
        auto field = [&](const char* key) {
            const size_t k = hdr.find(key);
            return k == std::string::npos ? std::string() : hdr.substr(k + std::strlen(key));
        };
        std::string descr = field("'descr':");
        descr = descr.substr(0, descr.find(','));
        std::string shape = field("'shape':");
        const size_t lp = shape.find('('), rp = shape.find(')');
        std::vector<size_t> dims;
        if (lp != std::string::npos && rp != std::string::npos && rp > lp) {
            std::string inner = shape.substr(lp + 1, rp - lp - 1);
            size_t i = 0;
            while (i < inner.size()) {
                while (i < inner.size() && (inner[i] < '0' || inner[i] > '9')) ++i;
                size_t v = 0;
                bool any = false;
                while (i < inner.size() && inner[i] >= '0' && inner[i] <= '9') {
                    v = v * 10 + size_t(inner[i++] - '0');
                    any = true;
                }
                if (any) dims.push_back(v);
            }
        }
        size_t item = 0;
        if (descr.find("f4") != std::string::npos || descr.find("i4") != std::string::npos ||
            descr.find("u4") != std::string::npos)
            item = 4;
        else if (descr.find("8") != std::string::npos)
            item = 8;
        else if (descr.find("2") != std::string::npos)
            item = 2;
        else if (descr.find("1") != std::string::npos)
            item = 1;
        size_t count = dims.empty() ? 0 : 1;
        for (size_t d : dims) count *= d;
        const std::string fo = field("'fortran_order':");
        const size_t fo0 = fo.find_first_not_of(' ');
        const bool fortran = fo0 != std::string::npos && fo.compare(fo0, 4, "True") == 0;
        if (dims.size() == 2 && dims[0] == n_clusters && dims[1] >= 1 && dims[1] <= kPadded && !fortran &&
            descr.find("<f4") != std::string::npos && data + (std::streamoff)(count * 4) <= size) {
            std::vector<float> raw(count);
            f.seekg(data);
            f.read(reinterpret_cast<char*>(raw.data()), (std::streamsize)(count * 4));
            if (!f) return false;
            out.assign(n_clusters * kPadded, 0.0f);
            for (size_t c = 0; c < n_clusters; ++c)
                std::memcpy(&out[c * kPadded], &raw[c * dims[1]], dims[1] * 4);
            return true;
        }
        // another array (the graph): skip its data when its size is known
        pos = (item && count) ? data + (std::streamoff)(item * count) : hit + 1;
    }
    return false;
}

void throw_status(chm_status s, const char* what) {
    if (s == CHM_OK) return;
    if (s == CHM_ERR_INVALID) throw std::invalid_argument(std::string(what) + ": invalid argument");
    std::string msg = std::string(what) + " failed";
    if (s == CHM_ERR_CUDA) msg += std::string(": ") + chm_last_error();
    if (s == CHM_ERR_CAPACITY) msg += ": capacity exceeded";
    throw std::runtime_error(msg);
}

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { reset(); }
    void reset() noexcept {
        if (p) (void)cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    void alloc(size_t n) {
        if (n <= bytes && p) return;
        reset();
        check_cuda(cudaMalloc(&p, n ? n : 1), "cudaMalloc");
        bytes = n;
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
    template <typename T>
    void upload(const T* src, size_t count) {
        alloc(count * sizeof(T));
        check_cuda(cudaMemcpy(p, src, count * sizeof(T), cudaMemcpyHostToDevice), "upload");
    }
    template <typename T>
    void download(std::vector<T>& dst, size_t count) const {
        dst.resize(count);
        if (count) check_cuda(cudaMemcpy(dst.data(), p, count * sizeof(T), cudaMemcpyDeviceToHost), "download");
    }
    // Takes over o's allocation.
    void take(DevBuf& o) {
        reset();
        p = o.p;
        bytes = o.bytes;
        o.p = nullptr;
        o.bytes = 0;
    }
};

void validate_search_options(const SearchOptions& o) {  // chimera_index.cu:27-36
    if (o.nprobe <= 0 || o.k_refine <= 0 || o.k_full_bit <= 0 || o.cagra_itopk_size <= 0 ||
        o.num_chunks <= 0)
        throw std::invalid_argument("All Chimera search options must be positive");
    if (o.k_full_bit > o.k_refine) throw std::invalid_argument("k_full_bit must not exceed k_refine");
    if (o.nprobe > CHM_MAX_NPROBE)
        throw std::invalid_argument("nprobe must not exceed " + std::to_string(CHM_MAX_NPROBE));
    if (o.k_refine > CHM_MAX_K_REFINE)
        throw std::invalid_argument("k_refine must not exceed " + std::to_string(CHM_MAX_K_REFINE));
    if (o.batch <= 0) throw std::invalid_argument("batch must be positive");
}

size_t validate_build_inputs(const std::vector<float>& emb, size_t dim, const std::vector<int>& doc_lens,
                             size_t n_clusters, size_t ex_bits) {  // build_index.cu:75-126
    if (dim < 64 || dim > kPadded)
        throw std::invalid_argument("Embedding dimension must be in [64, " + std::to_string(kPadded) + "]");
    if (emb.empty() || emb.size() % dim != 0)
        throw std::invalid_argument("Embedding storage must contain a non-empty whole number of vectors");
    const size_t n = emb.size() / dim;
    if (n > static_cast<size_t>(std::numeric_limits<int>::max()))
        throw std::invalid_argument("Embedding count exceeds the int32 index format limit");
    if (n_clusters == 0 || n_clusters > n)
        throw std::invalid_argument("n_clusters must be between 1 and the number of embeddings");
    if (ex_bits < 1 || ex_bits > 7)
        throw std::invalid_argument("ex_bits must be in [1, 7] so full codes fit in 2-8 bits per dimension");
    if (doc_lens.empty()) throw std::invalid_argument("doc_lens must not be empty");
    size_t total = 0;
    for (int len : doc_lens) {
        if (len <= 0) throw std::invalid_argument("Every document length must be positive");
        if (total > n || static_cast<size_t>(len) > n - total)
            throw std::invalid_argument("Document lengths exceed the number of embeddings");
        total += static_cast<size_t>(len);
    }
    if (total != n) throw std::invalid_argument("Document lengths do not sum to the number of embeddings");
    return n;
}

template <typename T>
void write_vec(std::ofstream& out, const T* data, size_t count) {
    out.write(reinterpret_cast<const char*>(data), static_cast<std::streamsize>(count * sizeof(T)));
}

std::ofstream open_out(const std::string& path) {
    std::ofstream o(path, std::ios::binary | std::ios::trunc);
    if (!o.is_open()) throw std::runtime_error("Failed to open output file: " + path);
    return o;
}

void finish(std::ofstream& o, const std::string& path) {
    o.flush();
    if (!o) throw std::runtime_error("Failed to write output file: " + path);
}

}  // namespace

struct chimera_index::Impl {
    size_t n = 0, d = 0, n_clusters = 0, ex_bits = 0;
    SearchOptions opts;
    std::vector<uint8_t> flips;
    std::vector<uint64_t> one_bit_codes;  // token order, 2 words per token
    std::vector<float> one_bit_factors;   // token order
    std::vector<float> full_factors;      // token order
    std::vector<uint8_t> full_codes;      // token order
    std::vector<uint32_t> inv_list;
    std::vector<size_t> cluster_pos;
    std::vector<char> clustered;          // cluster_1bit.bin payload
    std::vector<int> doc_lens;
    std::vector<float> centroids_rot;     // [n_clusters * 128]
    bool has_index = false;
    bool ready = false;
    bool host_current = true;  // false after a device build: save() downloads the arrays

    DevBuf d_cluster_pos, d_codes1, d_factor1, d_doc_ids, d_tok2pos, d_doc_ptrs, d_full, d_ff, d_cent,
        d_cnorm, d_flips, d_cent_bf16, d_cnmax, d_ws, d_q, d_res, d_nres, d_codes1_tok, d_factor1_tok,
        d_tok_cluster, d_inv;
    size_t ws_bytes = 0;
    int ws_batch = 0;
    int table_extra = 0;
    cudaStream_t stream = nullptr;
    chm_index view{};
    std::vector<float> h_q;

    ~Impl() { release(); }

    void release() noexcept {
        if (stream) {
            (void)cudaStreamSynchronize(stream);
            (void)cudaStreamDestroy(stream);
            stream = nullptr;
        }
        for (DevBuf* b : {&d_cluster_pos, &d_codes1, &d_factor1, &d_doc_ids, &d_tok2pos, &d_doc_ptrs, &d_full,
                          &d_ff, &d_cent, &d_cnorm, &d_flips, &d_cent_bf16, &d_cnmax, &d_ws, &d_q, &d_res,
                          &d_nres, &d_codes1_tok, &d_factor1_tok, &d_tok_cluster, &d_inv})
            b->reset();
        ready = false;
        ws_bytes = 0;
        ws_batch = 0;
    }

    void clear() noexcept {
        release();
        flips.clear();
        one_bit_codes.clear();
        one_bit_factors.clear();
        full_factors.clear();
        full_codes.clear();
        inv_list.clear();
        cluster_pos.clear();
        clustered.clear();
        doc_lens.clear();
        centroids_rot.clear();
        n = d = n_clusters = ex_bits = 0;
        has_index = false;
        host_current = true;
    }

    // The host copies save() writes, from the device index a device build left.
    void ensure_host() {
        if (host_current) return;
        std::vector<int64_t> cpos;
        d_cluster_pos.download(cpos, n_clusters + 1);
        cluster_pos.assign(cpos.begin(), cpos.end());
        d_inv.download(inv_list, n);
        d_codes1_tok.download(one_bit_codes, n * 2);
        d_factor1_tok.download(one_bit_factors, n);
        d_full.download(full_codes, n * full_stride());
        d_ff.download(full_factors, n);
        d_cent.download(centroids_rot, n_clusters * kPadded);
        clustered.resize(n * 28);  // cluster_1bit.bin: codes, factors, doc ids, token positions
        check_cuda(cudaMemcpy(clustered.data(), d_codes1.p, n * 16, cudaMemcpyDeviceToHost), "download");
        check_cuda(cudaMemcpy(clustered.data() + n * 16, d_factor1.p, n * 4, cudaMemcpyDeviceToHost), "download");
        check_cuda(cudaMemcpy(clustered.data() + n * 20, d_doc_ids.p, n * 4, cudaMemcpyDeviceToHost), "download");
        check_cuda(cudaMemcpy(clustered.data() + n * 24, d_tok2pos.p, n * 4, cudaMemcpyDeviceToHost), "download");
        host_current = true;
    }

    static void select_device() {
        int count = 0;
        check_cuda(cudaGetDeviceCount(&count), "Querying CUDA devices");
        if (count == 0) throw std::runtime_error("No CUDA device is available");
        check_cuda(cudaSetDevice(0), "Selecting CUDA device 0");
    }

    size_t full_stride() const { return kPadded * (1 + ex_bits) / 8; }

    void init_device() {
        if (ready) return;
        if (!has_index) throw std::runtime_error("Cannot initialize an empty Chimera index");
        if (static_cast<size_t>(opts.nprobe) > n_clusters)
            throw std::invalid_argument("nprobe must not exceed the number of clusters");
        select_device();
        const size_t num_docs = doc_lens.size();
        std::vector<int64_t> ptrs(num_docs + 1, 0);
        for (size_t i = 0; i < num_docs; ++i) ptrs[i + 1] = ptrs[i] + doc_lens[i];
        if (static_cast<size_t>(ptrs.back()) != n)
            throw std::runtime_error("Document lengths do not match the number of indexed embeddings");
        if (clustered.size() != n * 28) throw std::runtime_error("Invalid in-memory clustered index payload");
        size_t free_mem = 0, total_mem = 0;
        check_cuda(cudaMemGetInfo(&free_mem, &total_mem), "cudaMemGetInfo");
        const size_t need = clustered.size() + full_codes.size() + n * 28 + centroids_rot.size() * 4;
        if (free_mem <= need)
            throw std::runtime_error("Insufficient GPU memory for the index: need " + std::to_string(need) +
                                     " bytes, have " + std::to_string(free_mem) + " bytes free");
        std::vector<int64_t> cpos(cluster_pos.begin(), cluster_pos.end());
        d_cluster_pos.upload(cpos.data(), cpos.size());
        d_codes1.upload(clustered.data(), n * 16);
        d_factor1.upload(reinterpret_cast<const float*>(clustered.data() + n * 16), n);
        d_doc_ids.upload(reinterpret_cast<const int32_t*>(clustered.data() + n * 20), n);
        d_tok2pos.upload(reinterpret_cast<const uint32_t*>(clustered.data() + n * 24), n);
        d_doc_ptrs.upload(ptrs.data(), ptrs.size());
        d_full.upload(full_codes.data(), full_codes.size());
        d_ff.upload(full_factors.data(), full_factors.size());
        d_cent.upload(centroids_rot.data(), centroids_rot.size());
        d_flips.upload(flips.data(), flips.size());
        check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
        // token-order copies of the 1-bit arrays: refinement reads each doc as one span
        d_codes1_tok.alloc(n * 16);
        d_factor1_tok.alloc(n * sizeof(float));
        throw_status(chm_token_order_1bit(d_codes1.as<uint8_t>(), d_factor1.as<float>(), d_tok2pos.as<uint32_t>(),
                                          static_cast<int64_t>(n), d_codes1_tok.as<uint8_t>(),
                                          d_factor1_tok.as<float>(), stream),
                     "token-order 1-bit copy");
        // every token's cluster (stage 1's dense-bound path)
        d_tok_cluster.alloc(n * sizeof(uint32_t));
        throw_status(chm_token_clusters(d_cluster_pos.as<int64_t>(), static_cast<int64_t>(n_clusters),
                                        d_tok2pos.as<uint32_t>(), static_cast<int64_t>(n), d_tok_cluster.as<uint32_t>(),
                                        stream),
                     "token clusters");
        int32_t max_list = 0;
        for (size_t c = 0; c < n_clusters; ++c)
            max_list = std::max<int32_t>(max_list, static_cast<int32_t>(cluster_pos[c + 1] - cluster_pos[c]));
        finalize_device(max_list);
    }

    // Centroid norms, their bf16 copy and max, and the chm_index view over the
    // device arrays (cluster- and token-order 1-bit data, full codes,
    // token clusters) a load or a device build left.
    void finalize_device(int32_t max_list) {
        d_cnorm.alloc(n_clusters * sizeof(float));
        throw_status(chm_row_norms(d_cent.as<float>(), static_cast<int64_t>(n_clusters), d_cnorm.as<float>(), stream),
                     "centroid norms");
        d_cent_bf16.alloc(n_clusters * kPadded * 2);
        d_cnmax.alloc(sizeof(float));
        throw_status(chm_to_bf16(d_cent.as<float>(), static_cast<int64_t>(n_clusters * kPadded), d_cent_bf16.p, stream),
                     "centroid bf16 copy");
        throw_status(chm_max_value(d_cnorm.as<float>(), static_cast<int64_t>(n_clusters), d_cnmax.as<float>(), stream),
                     "centroid norm max");
        int32_t max_doc = 0;
        for (int len : doc_lens) max_doc = std::max<int32_t>(max_doc, len);
        view = chm_index{static_cast<int64_t>(n), static_cast<int64_t>(doc_lens.size()),
                         static_cast<int64_t>(n_clusters), static_cast<int32_t>(ex_bits), static_cast<int32_t>(d),
                         max_list, max_doc, d_cluster_pos.as<int64_t>(), d_codes1.as<uint8_t>(),
                         d_factor1.as<float>(), d_doc_ids.as<int32_t>(), d_tok2pos.as<uint32_t>(),
                         d_doc_ptrs.as<int64_t>(), d_full.as<uint8_t>(), d_ff.as<float>(), d_cent.as<float>(),
                         d_cnorm.as<float>(), d_flips.as<uint8_t>(), d_cent_bf16.p, d_cnmax.as<float>(),
                         d_codes1_tok.as<uint8_t>(), d_factor1_tok.as<float>(), d_tok_cluster.as<uint32_t>()};
        check_cuda(cudaStreamSynchronize(stream), "index upload");
        ready = true;
    }

    chm_search_params params(int batch, size_t k) const {
        return chm_search_params{opts.nprobe, opts.k_refine, opts.k_full_bit, opts.num_chunks,
                                 static_cast<int32_t>(k), batch, table_extra};
    }

    void ensure_workspace(const chm_search_params& p) {
        const size_t need = chm_search_workspace_bytes(&view, &p);
        if (need == 0) throw std::invalid_argument("Invalid Chimera search parameters");
        if (need > ws_bytes) {
            d_ws.alloc(need);
            ws_bytes = need;
        }
    }

    std::vector<std::vector<size_t>> run(const float* queries, size_t nq, size_t k) {
        if (k == 0) throw std::invalid_argument("k must be positive");
        if (k > CHM_MAX_K) throw std::invalid_argument("k must not exceed " + std::to_string(CHM_MAX_K));
        init_device();
        const size_t qfloats = kQ * d;
        d_q.alloc(nq * qfloats * sizeof(float));
        d_res.alloc(nq * k * sizeof(int64_t));
        d_nres.alloc(nq * sizeof(int32_t));
        check_cuda(cudaMemcpyAsync(d_q.p, queries, nq * qfloats * sizeof(float), cudaMemcpyHostToDevice, stream),
                   "query upload");
        std::vector<int32_t> counts(nq);
        std::vector<int64_t> ids(nq * k);
        for (int attempt = 0;; ++attempt) {
            const int batch = static_cast<int>(std::min<size_t>(nq, static_cast<size_t>(opts.batch)));
            chm_search_params p = params(batch, k);
            ensure_workspace(p);
            throw_status(chm_search(&view, &p, d_q.as<float>(), static_cast<int64_t>(nq), d_res.as<int64_t>(),
                                    d_nres.as<int32_t>(), d_ws.p, ws_bytes, stream),
                         "Chimera search");
            check_cuda(cudaMemcpyAsync(counts.data(), d_nres.p, nq * sizeof(int32_t), cudaMemcpyDeviceToHost, stream),
                       "result count copy");
            check_cuda(cudaMemcpyAsync(ids.data(), d_res.p, nq * k * sizeof(int64_t), cudaMemcpyDeviceToHost, stream),
                       "result copy");
            check_cuda(cudaStreamSynchronize(stream), "Chimera search");
            const bool overflow = std::any_of(counts.begin(), counts.end(), [](int32_t c) { return c < 0; });
            if (!overflow) break;
            if (table_extra >= 6 || attempt >= 6)
                throw std::runtime_error("Candidate table capacity exceeded");
            ++table_extra;  // rerun the batch with tables twice as large
        }
        std::vector<std::vector<size_t>> out(nq);
        for (size_t i = 0; i < nq; ++i)
            for (int j = 0; j < counts[i]; ++j) out[i].push_back(static_cast<size_t>(ids[i * k + j]));
        return out;
    }
};

chimera_index::chimera_index() : impl_(std::make_unique<Impl>()) {}
chimera_index::~chimera_index() = default;

void chimera_index::build(const std::vector<float>& embeddings, size_t dimension, const std::vector<int>& doc_lens,
                          size_t n_clusters, size_t ex_bits, const SearchOptions& options) {
    const size_t n = validate_build_inputs(embeddings, dimension, doc_lens, n_clusters, ex_bits);
    Impl::select_device();
    Impl& m = *impl_;
    m.clear();
    validate_search_options(options);
    m.opts = options;
    m.n = n;
    m.d = dimension;
    m.n_clusters = n_clusters;
    m.ex_bits = ex_bits;
    m.doc_lens = doc_lens;
    m.flips.assign(64, 0);
    chm_host_fhtkac_flips(kRotatorSeed, m.flips.data(), m.flips.size());
    std::vector<uint64_t> ids(n_clusters);
    chm_host_sample_centroids(n, n_clusters, kCentroidSeed, ids.data());

    cudaStream_t st = nullptr;
    check_cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
    struct StreamGuard {
        cudaStream_t s;
        ~StreamGuard() { (void)cudaStreamDestroy(s); }
    } guard{st};
    const size_t d = dimension;
    DevBuf x_raw, x128, c_raw, c128, cn_raw, assign_d, ws, flips_d, cent_rot, cb1, cbex, codes1, f1, full, ff;
    x_raw.upload(embeddings.data(), embeddings.size());
    const float* x_pad = x_raw.as<float>();
    if (d != kPadded) {
        x128.alloc(n * kPadded * sizeof(float));
        check_cuda(cudaMemsetAsync(x128.p, 0, n * kPadded * sizeof(float), st), "pad");
        check_cuda(cudaMemcpy2DAsync(x128.p, kPadded * 4, x_raw.p, d * 4, d * 4, n, cudaMemcpyDeviceToDevice, st),
                   "pad");
        x_pad = x128.as<float>();
    }
    std::vector<float> cent(n_clusters * d);
    for (size_t c = 0; c < n_clusters; ++c)  // sample_centroids, build_index.cu:176-182
        std::memcpy(cent.data() + c * d, embeddings.data() + ids[c] * d, d * sizeof(float));
    c_raw.upload(cent.data(), cent.size());
    c128.alloc(n_clusters * kPadded * sizeof(float));
    check_cuda(cudaMemsetAsync(c128.p, 0, c128.bytes, st), "pad");
    check_cuda(cudaMemcpy2DAsync(c128.p, kPadded * 4, c_raw.p, d * 4, d * 4, n_clusters, cudaMemcpyDeviceToDevice, st),
               "pad");
    cn_raw.alloc(n_clusters * sizeof(float));
    throw_status(chm_row_norms(c128.as<float>(), static_cast<int64_t>(n_clusters), cn_raw.as<float>(), st), "norms");
    assign_d.alloc(n * sizeof(uint32_t));
    const size_t wsb = chm_build_assign_workspace_bytes(static_cast<int64_t>(n), static_cast<int64_t>(n_clusters));
    ws.alloc(wsb);
    throw_status(chm_build_assign(x_pad, static_cast<int64_t>(n), static_cast<int32_t>(d), c128.as<float>(),
                                  cn_raw.as<float>(), static_cast<int64_t>(n_clusters), assign_d.as<uint32_t>(),
                                  ws.p, wsb, st),
                 "centroid assignment");
    flips_d.upload(m.flips.data(), m.flips.size());
    cent_rot.alloc(n_clusters * kPadded * sizeof(float));
    cb1.alloc(n_clusters * sizeof(float));
    cbex.alloc(n_clusters * sizeof(float));
    throw_status(chm_prepare_queries(flips_d.as<uint8_t>(), static_cast<int32_t>(d), static_cast<int32_t>(ex_bits),
                                     c_raw.as<float>(), static_cast<int64_t>(n_clusters), cent_rot.as<float>(),
                                     cb1.as<float>(), cbex.as<float>(), nullptr, st),
                 "centroid rotation");
    const size_t fstride = kPadded * (1 + ex_bits) / 8;
    codes1.alloc(n * 16);
    f1.alloc(n * 4);
    full.alloc(n * fstride);
    ff.alloc(n * 4);
    throw_status(chm_build_encode(flips_d.as<uint8_t>(), x_raw.as<float>(), static_cast<int64_t>(n),
                                  static_cast<int32_t>(d), static_cast<int32_t>(ex_bits), codes1.as<uint8_t>(),
                                  f1.as<float>(), full.as<uint8_t>(), ff.as<float>(), nullptr, st),
                 "encoding");
    // IVF_PG::build_from_assignments + reorder_by_cluster (ivf_pg.cpp:110-126,
    // build_index.cu:328-363) on the device; the result stays there as the
    // search index (host copies are made only if the index is saved)
    std::vector<int64_t> ptrs(doc_lens.size() + 1, 0);
    for (size_t i = 0; i < doc_lens.size(); ++i) ptrs[i + 1] = ptrs[i] + doc_lens[i];
    m.d_doc_ptrs.upload(ptrs.data(), ptrs.size());
    m.d_cluster_pos.alloc((n_clusters + 1) * sizeof(int64_t));
    m.d_inv.alloc(n * sizeof(uint32_t));
    m.d_codes1.alloc(n * 16);
    m.d_factor1.alloc(n * sizeof(float));
    m.d_doc_ids.alloc(n * sizeof(int32_t));
    m.d_tok2pos.alloc(n * sizeof(uint32_t));
    DevBuf status, ows;
    status.alloc(sizeof(uint32_t));
    const size_t owb = chm_build_cluster_order_workspace_bytes(static_cast<int64_t>(n), static_cast<int64_t>(n_clusters));
    ows.alloc(owb);
    throw_status(chm_build_cluster_order(assign_d.as<uint32_t>(), static_cast<int64_t>(n),
                                         static_cast<int64_t>(n_clusters), m.d_doc_ptrs.as<int64_t>(),
                                         static_cast<int64_t>(doc_lens.size()), codes1.as<uint8_t>(), f1.as<float>(),
                                         m.d_cluster_pos.as<int64_t>(), m.d_inv.as<uint32_t>(), m.d_codes1.as<uint8_t>(),
                                         m.d_factor1.as<float>(), m.d_doc_ids.as<int32_t>(),
                                         m.d_tok2pos.as<uint32_t>(), status.as<uint32_t>(), ows.p, owb, st),
                 "cluster order");
    uint32_t bad = 0;
    check_cuda(cudaMemcpyAsync(&bad, status.p, sizeof(bad), cudaMemcpyDeviceToHost, st), "copy");
    std::vector<int64_t> cpos(n_clusters + 1);
    check_cuda(cudaMemcpyAsync(cpos.data(), m.d_cluster_pos.p, cpos.size() * 8, cudaMemcpyDeviceToHost, st), "copy");
    check_cuda(cudaStreamSynchronize(st), "index build");
    if (bad) throw std::runtime_error(bad & 2 ? "An inverted list exceeds 32768 tokens" : "Invalid assignment");
    m.cluster_pos.assign(cpos.begin(), cpos.end());
    m.d_full.take(full);
    m.d_ff.take(ff);
    m.d_cent.take(cent_rot);
    m.d_flips.take(flips_d);
    m.d_codes1_tok.take(codes1);
    m.d_factor1_tok.take(f1);
    m.d_tok_cluster.take(assign_d);
    int32_t max_list = 0;
    for (size_t c = 0; c < n_clusters; ++c)
        max_list = std::max<int32_t>(max_list, static_cast<int32_t>(cpos[c + 1] - cpos[c]));
    check_cuda(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    m.has_index = true;
    m.host_current = false;
    m.finalize_device(max_list);
}

std::vector<size_t> chimera_index::search(const std::vector<float>& query, size_t k) {
    return search(query.data(), query.size(), k);
}

std::vector<size_t> chimera_index::search(const float* query, size_t query_size, size_t k) {
    Impl& m = *impl_;
    if (!m.has_index) throw std::runtime_error("Cannot search an empty Chimera index");
    if (query == nullptr || query_size != kQ * m.d)
        throw std::invalid_argument("A Chimera query must have shape [" + std::to_string(kQ) + ", " +
                                    std::to_string(m.d) + "]");
    if (k == 0) throw std::invalid_argument("k must be positive");
    try {
        return m.run(query, 1, k).front();
    } catch (const std::invalid_argument&) {
        throw;
    } catch (...) {
        if (!m.ready) m.release();
        throw;
    }
}

std::vector<std::vector<size_t>> chimera_index::search_batch(const float* queries, size_t num_queries, size_t k) {
    Impl& m = *impl_;
    if (!m.has_index) throw std::runtime_error("Cannot search an empty Chimera index");
    if (queries == nullptr && num_queries > 0) throw std::invalid_argument("queries must not be null");
    if (k == 0) throw std::invalid_argument("k must be positive");
    if (num_queries == 0) return {};
    return m.run(queries, num_queries, k);
}

void chimera_index::save(const std::string& index_dir) const {
    Impl& m = *impl_;
    if (!m.has_index) throw std::runtime_error("Cannot save an empty Chimera index");
    m.ensure_host();
    namespace fs = std::filesystem;
    std::error_code ec;
    fs::create_directories(index_dir, ec);
    if (ec) throw std::runtime_error("Failed to create index directory " + index_dir + ": " + ec.message());
    const std::array<const char*, 7> names = {"doclens.bin", "doc_1bit.bin", "doc_full.bin", "cluster_1bit.bin",
                                              "ivf.bin", "centroids.carga", kCentroidFile};
    for (const char* f : names) {
        ec.clear();
        fs::remove(fs::path(index_dir) / f, ec);
        if (ec) throw std::runtime_error("Failed to remove stale index output " + std::string(f) + ": " + ec.message());
    }
    const fs::path dir(index_dir);
    {
        const auto p = (dir / "doclens.bin").string();
        auto o = open_out(p);
        const int count = static_cast<int>(m.doc_lens.size());
        write_vec(o, &count, 1);
        write_vec(o, m.doc_lens.data(), m.doc_lens.size());
        finish(o, p);
    }
    {
        const auto p = (dir / "ivf.bin").string();
        auto o = open_out(p);
        const size_t cnt = m.inv_list.size();
        write_vec(o, &cnt, 1);
        write_vec(o, m.inv_list.data(), m.inv_list.size());
        write_vec(o, m.cluster_pos.data(), m.cluster_pos.size());
        finish(o, p);
    }
    {
        const auto p = (dir / "doc_1bit.bin").string();
        auto o = open_out(p);
        const IndexHeader h{m.n, m.d, m.n_clusters, m.ex_bits, kPadded};
        write_vec(o, &h, 1);
        write_vec(o, m.flips.data(), m.flips.size());
        write_vec(o, m.one_bit_codes.data(), m.one_bit_codes.size());
        write_vec(o, m.one_bit_factors.data(), m.one_bit_factors.size());
        write_vec(o, m.full_factors.data(), m.full_factors.size());
        finish(o, p);
    }
    {
        const auto p = (dir / "doc_full.bin").string();
        auto o = open_out(p);
        write_vec(o, m.full_codes.data(), m.full_codes.size());
        finish(o, p);
    }
    {
        const auto p = (dir / "cluster_1bit.bin").string();
        auto o = open_out(p);
        write_vec(o, m.clustered.data(), m.clustered.size());
        finish(o, p);
    }
    {
        const auto p = (dir / kCentroidFile).string();
        auto o = open_out(p);
        const int64_t hdr[2] = {static_cast<int64_t>(m.n_clusters), static_cast<int64_t>(kPadded)};
        write_vec(o, hdr, 2);
        write_vec(o, m.centroids_rot.data(), m.centroids_rot.size());
        finish(o, p);
    }
}

void chimera_index::load(const std::string& index_dir, const SearchOptions& options) {
    namespace fs = std::filesystem;
    const fs::path dir(index_dir);
    if (!fs::is_directory(dir)) throw std::runtime_error("Chimera index directory does not exist: " + index_dir);
    Impl::select_device();
    Impl& m = *impl_;
    m.clear();
    validate_search_options(options);
    m.opts = options;
    const auto one = (dir / "doc_1bit.bin").string();
    std::ifstream in(one, std::ios::binary);
    IndexHeader h{};
    in.read(reinterpret_cast<char*>(&h), sizeof(h));
    if (!in || h.num_embeddings == 0 || h.num_embeddings > static_cast<size_t>(std::numeric_limits<int>::max()) ||
        h.dimension < 64 || h.dimension > kPadded || h.num_clusters == 0 || h.num_clusters > h.num_embeddings ||
        h.ex_bits < 1 || h.ex_bits > 7)
        throw std::runtime_error("Invalid Chimera index header: " + one);
    m.n = h.num_embeddings;
    m.d = h.dimension;
    m.n_clusters = h.num_clusters;
    m.ex_bits = h.ex_bits;
    if (static_cast<size_t>(m.opts.nprobe) > m.n_clusters) {
        m.clear();
        throw std::invalid_argument("nprobe must not exceed the number of clusters");
    }
    if (h.padded_dimension != kPadded)
        throw std::runtime_error("Index file padded_dim=" + std::to_string(h.padded_dimension) +
                                 " does not match compiled PADDED_DIM=" + std::to_string(kPadded));
    try {
        m.flips.resize(64);
        in.read(reinterpret_cast<char*>(m.flips.data()), 64);
        if (!in) throw std::runtime_error("Failed to read rotator from " + one);
        m.one_bit_codes.resize(m.n * 2);
        m.one_bit_factors.resize(m.n);
        m.full_factors.resize(m.n);
        m.full_codes.resize(m.n * m.full_stride());
        in.read(reinterpret_cast<char*>(m.one_bit_codes.data()), static_cast<std::streamsize>(m.n * 16));
        in.read(reinterpret_cast<char*>(m.one_bit_factors.data()), static_cast<std::streamsize>(m.n * 4));
        in.read(reinterpret_cast<char*>(m.full_factors.data()), static_cast<std::streamsize>(m.n * 4));
        if (!in) throw std::runtime_error("Failed to read quantized payload from " + one);
        {
            std::ifstream f((dir / "doc_full.bin").string(), std::ios::binary);
            f.read(reinterpret_cast<char*>(m.full_codes.data()), static_cast<std::streamsize>(m.full_codes.size()));
            if (!f) throw std::runtime_error("Failed to read full-code payload from " + (dir / "doc_full.bin").string());
        }
        {
            const auto p = (dir / "ivf.bin").string();
            std::ifstream f(p, std::ios::binary);
            size_t cnt = 0;
            f.read(reinterpret_cast<char*>(&cnt), sizeof(cnt));
            if (!f || cnt != m.n) throw std::runtime_error("Invalid IVF payload: " + p);
            m.inv_list.resize(cnt);
            m.cluster_pos.resize(m.n_clusters + 1);
            f.read(reinterpret_cast<char*>(m.inv_list.data()), static_cast<std::streamsize>(cnt * 4));
            f.read(reinterpret_cast<char*>(m.cluster_pos.data()), static_cast<std::streamsize>((m.n_clusters + 1) * 8));
            if (!f) throw std::runtime_error("Invalid IVF payload: " + p);
        }
        {
            const auto p = (dir / kCentroidFile).string();
            std::ifstream f(p, std::ios::binary);
            int64_t hdr[2] = {0, 0};
            f.read(reinterpret_cast<char*>(hdr), sizeof(hdr));
            if (!f) {
                // an index written by the reference: the rotated centroids are the
                // dataset inside its cuVS CAGRA file
                const auto pc = (dir / "centroids.carga").string();
                if (!read_carga_centroids(pc, m.n_clusters, m.centroids_rot))
                    throw std::runtime_error("Missing " + p + ", and " + pc +
                                             " holds no (n_clusters, dim) fp32 dataset block");
            } else {
                if (hdr[0] != static_cast<int64_t>(m.n_clusters) || hdr[1] != static_cast<int64_t>(kPadded))
                    throw std::runtime_error("Invalid centroid payload: " + p);
                m.centroids_rot.resize(m.n_clusters * kPadded);
                f.read(reinterpret_cast<char*>(m.centroids_rot.data()),
                       static_cast<std::streamsize>(m.centroids_rot.size() * 4));
                if (!f) throw std::runtime_error("Invalid centroid payload: " + p);
            }
        }
        {
            const auto p = (dir / "doclens.bin").string();
            std::ifstream f(p, std::ios::binary);
            int cnt = 0;
            f.read(reinterpret_cast<char*>(&cnt), sizeof(cnt));
            if (!f || cnt <= 0) throw std::runtime_error("Failed to read document lengths: " + p);
            m.doc_lens.resize(static_cast<size_t>(cnt));
            f.read(reinterpret_cast<char*>(m.doc_lens.data()), static_cast<std::streamsize>(cnt * 4));
            if (!f) throw std::runtime_error("Failed to read document lengths: " + p);
        }
        {
            const auto p = (dir / "cluster_1bit.bin").string();
            const size_t want = m.n * 28;
            std::ifstream f(p, std::ios::binary | std::ios::ate);
            if (!f || f.tellg() < 0 || static_cast<size_t>(f.tellg()) != want)
                throw std::runtime_error("Invalid clustered index payload: " + p);
            m.clustered.resize(want);
            f.seekg(0);
            f.read(m.clustered.data(), static_cast<std::streamsize>(want));
            if (!f) throw std::runtime_error("Failed to read clustered index: " + p);
        }
        m.has_index = true;
        m.init_device();
    } catch (...) {
        m.clear();
        throw;
    }
}

}  // namespace Chimera
