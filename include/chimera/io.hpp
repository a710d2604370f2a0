// Input readers with the reference's binary formats
// (cpp/include/chimera/io.hpp:9-13, cpp/src/io.cpp:53-109):
//   embeddings: int32 count, int32 dim, fp32[count * dim]
//   queries:    int32 count, int32 length, int32 dim, fp32[count * length * dim]
//   doclens:    int32 count, int32[count]
#pragma once

#include <cstddef>
#include <string>
#include <vector>

namespace Chimera {

std::vector<float> load_data(size_t& num_embeddings, size_t& d, std::string filename);
std::vector<float> load_query(size_t& q_doclen, size_t& num_q, size_t& d, std::string filename);
std::vector<int> load_doclens(std::string filename);

}  // namespace Chimera
