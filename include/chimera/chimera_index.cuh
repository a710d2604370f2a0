// Drop-in replacement for the reference's public C++ API
// (cpp/include/chimera/chimera_index.cuh:26-158): same namespace, class,
// SearchOptions fields and defaults, method signatures and exception types.
// The search runs on the B200 kernels of libchimera_b200 through the C ABI
// in chimera_b200.h; nothing here depends on cuVS, RAFT or RMM.
//
// Additive API (no reference counterpart): search_batch(), which runs many
// queries per GPU pass, and SearchOptions::batch.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace Chimera {

struct SearchOptions {
    int nprobe = 128;
    int k_refine = 3000;
    int k_full_bit = 300;
    int cagra_itopk_size = 150;  // accepted for drop-in compatibility; the probe is exact
    int num_chunks = 5;
    int batch = 64;              // queries per GPU pass in search_batch (additive)
};

inline void check_cuda(cudaError_t status, const char* operation = "CUDA operation") {
    if (status != cudaSuccess) {
        throw std::runtime_error(std::string(operation) + " failed: " + cudaGetErrorString(status));
    }
}

class chimera_index {
  public:
    chimera_index();
    ~chimera_index();

    void build(const std::vector<float>& embeddings, size_t dimension, const std::vector<int>& doc_lens,
               size_t n_clusters, size_t ex_bits, const SearchOptions& options = {});

    std::vector<size_t> search(const std::vector<float>& query, size_t k);
    std::vector<size_t> search(const float* query, size_t query_size, size_t k);

    // Batched search: `queries` holds num_queries row-major [32, d] queries.
    std::vector<std::vector<size_t>> search_batch(const float* queries, size_t num_queries, size_t k);

    void save(const std::string& index_dir) const;
    void load(const std::string& index_dir, const SearchOptions& options = {});

    chimera_index(const chimera_index&) = delete;
    chimera_index& operator=(const chimera_index&) = delete;

    struct Impl;

  private:
    std::unique_ptr<Impl> impl_;
};

}  // namespace Chimera
