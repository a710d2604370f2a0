// Host-side seeded draws of the index build, using the same standard-library
// engines and distributions as the reference so builds are reproducible
// across the two implementations:
//   * FhtKac sign flips: rabitqlib make_seeded_generator + fill_flip
//     (rotator.hpp:46-52, 184-189): std::mt19937 seeded through
//     std::seed_seq{lo32, hi32}, 64 bytes of uniform_int_distribution<int>(0,255).
//   * centroid sample: reservoir sampling with std::mt19937_64(42) and
//     uniform_int_distribution<size_t>(0, i) (build_index.cu:159-184).
#include <cstdint>
#include <numeric>
#include <random>
#include <vector>

extern "C" void chm_host_fhtkac_flips(uint64_t seed, uint8_t* out, size_t n) {
    std::seed_seq seq{static_cast<uint32_t>(seed & 0xFFFFFFFFu), static_cast<uint32_t>(seed >> 32)};
    std::mt19937 gen(seq);
    std::uniform_int_distribution<int> dist(0, 255);
    for (size_t i = 0; i < n; ++i) out[i] = static_cast<uint8_t>(dist(gen));
}

extern "C" void chm_host_sample_centroids(uint64_t num_embeddings, uint64_t n_clusters, uint64_t seed,
                                          uint64_t* ids) {
    std::vector<size_t> sampled(n_clusters);
    std::iota(sampled.begin(), sampled.end(), size_t{0});
    std::mt19937_64 generator(seed);
    for (size_t index = n_clusters; index < num_embeddings; ++index) {
        std::uniform_int_distribution<size_t> distribution(0, index);
        const size_t position = distribution(generator);
        if (position < n_clusters) sampled[position] = index;
    }
    for (size_t i = 0; i < n_clusters; ++i) ids[i] = sampled[i];
}
