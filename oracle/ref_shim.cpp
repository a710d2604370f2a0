// Test infrastructure only: a C-ABI wrapper around the Chimera reference's own
// CPU code (rabitqlib rotator / packer / AVX-512 unpack+GEMV and Chimera's
// quantization.cpp), compiled from the reference sources where they lie by
// oracle/Makefile into oracle/_ref/libchimera_ref.so.  Nothing in the product
// links this file.  It exists so the plain-C restatement in chimera_oracle.c
// and the CUDA kernels can be checked against the reference's real code (the
// pins in tests/test_cpu_oracle.py run it on the same inputs as the oracle).
//
// Reference interfaces wrapped (paths inside the Chimera project):
//   rabitqlib::choose_rotator_with_seed / FhtKacRotator::rotate
//       cpp/third_party/rabitqlib/utils/rotator.hpp:281-307, 369-398
//   Chimera::encode_one_bit / encode_full_code / best_rescale_factor
//       cpp/src/quantization.cpp:47-193
//   rabitqlib::quant::rabitq_impl::ex_bits::packing_rabitqplus_code
//       cpp/third_party/rabitqlib/quantization/pack_excode.hpp:274-297
//   rabitqlib::select_excode_unpackfunc / gemv_batch8_avx512
//       cpp/third_party/rabitqlib/utils/space.hpp:790-851
// The per-document loop in cref_fullbit_doc_scores restates
// chimera_index::compute_full_bit_scores (cpp/src/search_impl.cu:510-574)
// around those reference primitives, with the same intrinsics sequence.
#define EIGEN_NO_CUDA
#include <immintrin.h>

#include <unistd.h>

#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <limits>
#include <numeric>
#include <random>
#include <string>
#include <vector>

#include "chimera/quantization.hpp"
#include "rabitqlib/quantization/pack_excode.hpp"
#include "rabitqlib/utils/rotator.hpp"
#include "rabitqlib/utils/space.hpp"

using rabitqlib::Rotator;

extern "C" {

// ---- rotator ---------------------------------------------------------------
void* cref_rotator_create(size_t dim, size_t padded_dim, uint64_t seed) {
    return rabitqlib::choose_rotator_with_seed<float>(
        dim, rabitqlib::RotatorType::FhtKacRotator, padded_dim, seed);
}

void cref_rotator_destroy(void* r) { delete static_cast<Rotator<float>*>(r); }

// Serialised flips (what chimera_index::save writes after the header).
int cref_rotator_flips(void* r, uint8_t* out, size_t cap) {
    char path[] = "/tmp/cref_flipsXXXXXX";
    int fd = mkstemp(path);
    if (fd < 0) return -1;
    close(fd);
    {
        std::ofstream os(path, std::ios::binary);
        static_cast<Rotator<float>*>(r)->save(os);
    }
    std::ifstream is(path, std::ios::binary | std::ios::ate);
    const size_t n = static_cast<size_t>(is.tellg());
    is.seekg(0);
    if (n > cap) { std::remove(path); return -1; }
    is.read(reinterpret_cast<char*>(out), static_cast<std::streamsize>(n));
    std::remove(path);
    return static_cast<int>(n);
}

void cref_rotate(void* r, const float* src, float* dst, size_t count, size_t dim,
                 size_t padded_dim) {
    auto* rot = static_cast<Rotator<float>*>(r);
    for (size_t i = 0; i < count; ++i) rot->rotate(src + i * dim, dst + i * padded_dim);
}

// ---- quantizer ---------------------------------------------------------------
// Buffers handed to the reference are 64-byte aligned so Eigen's packet
// reductions always start at element 0 (the reference's own std::vector
// buffers may start at any 16-byte offset).
void cref_encode(const float* rotated, size_t count, size_t dim, size_t ex_bits,
                 uint64_t* one_bit_codes, float* one_bit_factors,
                 uint8_t* full_codes, float* full_factors) {
    const size_t words = dim / 64;
    const size_t full_bytes = dim * (1 + ex_bits) / 8;
    float* buf = static_cast<float*>(aligned_alloc(64, ((dim * 4 + 63) / 64) * 64));
    for (size_t i = 0; i < count; ++i) {
        std::memcpy(buf, rotated + i * dim, dim * sizeof(float));
        Chimera::encode_one_bit(buf, dim, one_bit_codes + i * words, one_bit_factors + i);
        Chimera::encode_full_code(buf, dim, ex_bits, full_codes + i * full_bytes,
                                  full_factors + i);
    }
    free(buf);
}

double cref_best_rescale_factor(const float* o_abs, size_t dim, size_t ex_bits) {
    return Chimera::best_rescale_factor(o_abs, dim, ex_bits);
}

void cref_quantize_ex(const float* rotated, uint8_t* ex_code, size_t dim, size_t ex_bits) {
    float* buf = static_cast<float*>(aligned_alloc(64, ((dim * 4 + 63) / 64) * 64));
    std::memcpy(buf, rotated, dim * sizeof(float));
    Chimera::quantize_ex(buf, ex_code, dim, ex_bits);
    free(buf);
}

// ---- packing -----------------------------------------------------------------
void cref_pack(const uint8_t* raw, uint8_t* packed, size_t dim, size_t bits) {
    rabitqlib::quant::rabitq_impl::ex_bits::packing_rabitqplus_code(raw, packed, dim, bits);
}

void cref_unpack(const uint8_t* packed, float* out, size_t dim, size_t bits) {
    rabitqlib::select_excode_unpackfunc(bits)(packed, out, dim);
}

void cref_gemv_batch8(const float* queries, const float* decoded, float* out,
                      size_t n_queries, size_t dim) {
    alignas(64) float dec[1024];
    std::memcpy(dec, decoded, dim * sizeof(float));
    rabitqlib::gemv_batch8_avx512(queries, dec, out, n_queries, dim);
}

// ---- full-bit MaxSim -------------------------------------------------------
// Scores `count` documents (token ranges [doc_ptrs[d], doc_ptrs[d+1]) in
// token order) with the (1+ex_bits)-bit codes, exactly as
// compute_full_bit_scores does for one query: unpack -> 32-query GEMV ->
// max_t (ip - cbex_sumq[t]) * factor -> 512-bit add + reduce.
// Uses OpenMP over documents like the reference when threads > 1.
void cref_fullbit_doc_scores(const float* rotated_queries /*[32*128]*/,
                             const float* cbex_sumq /*[32]*/,
                             const uint8_t* full_codes, const float* full_factors,
                             const int64_t* doc_ptrs, const int32_t* docs, int count,
                             size_t ex_bits, float* out_scores, int threads) {
    constexpr size_t kDim = 128;
    constexpr size_t kQ = 32;
    const size_t stride = kDim * (1 + ex_bits) / 8;
    auto unpack = rabitqlib::select_excode_unpackfunc(1 + ex_bits);
    alignas(64) float cbex[kQ];
    for (size_t j = 0; j < kQ; ++j) cbex[j] = cbex_sumq[j];
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
    for (int i = 0; i < count; ++i) {
        const int64_t doc = docs[i];
        const size_t start = static_cast<size_t>(doc_ptrs[doc]);
        const size_t n_tok = static_cast<size_t>(doc_ptrs[doc + 1]) - start;
        alignas(64) float decoded[kDim];
        alignas(64) float full_ip[kQ];
        alignas(64) float max_ts[kQ];
        const __m512 neg_inf = _mm512_set1_ps(-std::numeric_limits<float>::infinity());
        for (size_t j = 0; j < kQ; j += 16) _mm512_store_ps(&max_ts[j], neg_inf);
        for (size_t t = 0; t < n_tok; ++t) {
            const size_t tid = start + t;
            unpack(full_codes + tid * stride, decoded, kDim);
            rabitqlib::gemv_batch8_avx512(rotated_queries, decoded, full_ip, kQ, kDim);
            const __m512 f = _mm512_set1_ps(full_factors[tid]);
            for (size_t j = 0; j < kQ; j += 16) {
                __m512 ip = _mm512_load_ps(&full_ip[j]);
                __m512 cb = _mm512_load_ps(&cbex[j]);
                __m512 comb = _mm512_mul_ps(_mm512_sub_ps(ip, cb), f);
                _mm512_store_ps(&max_ts[j], _mm512_max_ps(_mm512_load_ps(&max_ts[j]), comb));
            }
        }
        __m512 sum = _mm512_load_ps(&max_ts[0]);
        for (size_t j = 16; j < kQ; j += 16) sum = _mm512_add_ps(sum, _mm512_load_ps(&max_ts[j]));
        out_scores[i] = _mm512_reduce_add_ps(sum);
    }
}

// QueryState (cpp/src/chimera_index_internal.cuh:58-64).
void cref_query_state(const float* rotated, size_t padded_dim, size_t ex_bits, float* cb1,
                      float* cbex) {
    const float sumq = std::accumulate(rotated, rotated + padded_dim, 0.0f);
    *cb1 = sumq * ((1 << 1) - 1) / 2.0f;
    *cbex = sumq * ((1 << (ex_bits + 1)) - 1) / 2.0f;
}

// sample_centroids, cpp/src/build_index.cu:159-184: reservoir sample with
// std::mt19937_64(42) and std::uniform_int_distribution<size_t>(0, index).
void cref_sample_centroid_ids(size_t num_embeddings, size_t n_clusters, uint64_t* ids) {
    std::vector<size_t> sampled(n_clusters);
    std::iota(sampled.begin(), sampled.end(), size_t {0});
    std::mt19937_64 generator(42);
    for (size_t index = n_clusters; index < num_embeddings; ++index) {
        std::uniform_int_distribution<size_t> distribution(0, index);
        const size_t position = distribution(generator);
        if (position < n_clusters) sampled[position] = index;
    }
    for (size_t i = 0; i < n_clusters; ++i) ids[i] = sampled[i];
}

}  // extern "C"
