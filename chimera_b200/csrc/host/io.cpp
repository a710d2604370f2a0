// Binary input readers; formats and error behaviour of cpp/src/io.cpp:53-109
// (std::runtime_error on a missing file, a short read, a non-positive header
// field or a size overflow).
#include "chimera/io.hpp"

#include <cstdint>
#include <fstream>
#include <limits>
#include <stdexcept>

namespace Chimera {
namespace {

std::ifstream open_or_throw(const std::string& f) {
    std::ifstream in(f, std::ios::binary);
    if (!in.is_open()) throw std::runtime_error("Failed to open input file: " + f);
    return in;
}

void read_exact(std::ifstream& in, void* dst, size_t bytes, const std::string& f) {
    if (bytes > static_cast<size_t>(std::numeric_limits<std::streamsize>::max()))
        throw std::runtime_error("Input payload is too large: " + f);
    in.read(static_cast<char*>(dst), static_cast<std::streamsize>(bytes));
    if (!in) throw std::runtime_error("Failed to read input file: " + f);
}

int32_t read_i32(std::ifstream& in, const std::string& f) {
    int32_t v = 0;
    read_exact(in, &v, sizeof(v), f);
    return v;
}

size_t mul_checked(size_t a, size_t b, const std::string& f) {
    if (a != 0 && b > std::numeric_limits<size_t>::max() / a)
        throw std::runtime_error("Input dimensions overflow size_t: " + f);
    return a * b;
}

}  // namespace

std::vector<float> load_data(size_t& num_embeddings, size_t& d, std::string filename) {
    auto in = open_or_throw(filename);
    const int32_t n = read_i32(in, filename), dim = read_i32(in, filename);
    if (n <= 0 || dim <= 0)
        throw std::runtime_error("Embedding header contains non-positive dimensions: " + filename);
    num_embeddings = static_cast<size_t>(n);
    d = static_cast<size_t>(dim);
    std::vector<float> out(mul_checked(num_embeddings, d, filename));
    read_exact(in, out.data(), mul_checked(out.size(), sizeof(float), filename), filename);
    return out;
}

std::vector<float> load_query(size_t& q_doclen, size_t& num_q, size_t& d, std::string filename) {
    auto in = open_or_throw(filename);
    const int32_t n = read_i32(in, filename), len = read_i32(in, filename), dim = read_i32(in, filename);
    if (n <= 0 || len <= 0 || dim <= 0)
        throw std::runtime_error("Query header contains non-positive dimensions: " + filename);
    num_q = static_cast<size_t>(n);
    q_doclen = static_cast<size_t>(len);
    d = static_cast<size_t>(dim);
    std::vector<float> out(mul_checked(mul_checked(num_q, q_doclen, filename), d, filename));
    read_exact(in, out.data(), mul_checked(out.size(), sizeof(float), filename), filename);
    return out;
}

std::vector<int> load_doclens(std::string filename) {
    auto in = open_or_throw(filename);
    const int32_t n = read_i32(in, filename);
    if (n <= 0) throw std::runtime_error("Document-length header contains a non-positive count: " + filename);
    std::vector<int> out(static_cast<size_t>(n));
    read_exact(in, out.data(), mul_checked(out.size(), sizeof(int), filename), filename);
    return out;
}

}  // namespace Chimera
