// pybind11 module `chimera` with the reference's surface
// (python/bindings.cpp:34-165): ChimeraIndex.build / load (static), search
// ([32, D] -> list[int], [Q, 32, D] -> list[list[int]]), save.  A 3-D query
// array runs as one batched GPU search instead of a Python-side loop.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <memory>
#include <stdexcept>
#include <vector>

#include "chimera/chimera_index.cuh"

namespace py = pybind11;
using Chimera::chimera_index;
using Chimera::SearchOptions;
using FloatArray = py::array_t<float, py::array::c_style>;

namespace {

SearchOptions make_options(int nprobe, int k_refine, int k_full_bit, int cagra_itopk_size, int num_chunks, int batch) {
    SearchOptions o;
    o.nprobe = nprobe;
    o.k_refine = k_refine;
    o.k_full_bit = k_full_bit;
    o.cagra_itopk_size = cagra_itopk_size;
    o.num_chunks = num_chunks;
    o.batch = batch;
    return o;
}

std::unique_ptr<chimera_index> build(const FloatArray& embeddings, const std::vector<int>& doc_lens, size_t n_clusters,
                                     size_t ex_bits, int nprobe, int k_refine, int k_full_bit, int cagra_itopk_size,
                                     int num_chunks, int batch) {
    if (embeddings.ndim() != 2)
        throw std::invalid_argument("embeddings must have shape [num_embeddings, dimension]");
    const size_t dim = static_cast<size_t>(embeddings.shape(1));
    std::vector<float> data(embeddings.data(), embeddings.data() + embeddings.size());
    auto index = std::make_unique<chimera_index>();
    {
        py::gil_scoped_release release;
        index->build(data, dim, doc_lens, n_clusters, ex_bits,
                     make_options(nprobe, k_refine, k_full_bit, cagra_itopk_size, num_chunks, batch));
    }
    return index;
}

std::unique_ptr<chimera_index> load(const std::string& dir, int nprobe, int k_refine, int k_full_bit,
                                    int cagra_itopk_size, int num_chunks, int batch) {
    auto index = std::make_unique<chimera_index>();
    {
        py::gil_scoped_release release;
        index->load(dir, make_options(nprobe, k_refine, k_full_bit, cagra_itopk_size, num_chunks, batch));
    }
    return index;
}

py::object search(chimera_index& index, const FloatArray& queries, size_t k) {
    if (queries.ndim() != 2 && queries.ndim() != 3)
        throw std::invalid_argument(
            "queries must have shape [query_length, dimension] or [num_queries, query_length, dimension]");
    const size_t nq = queries.ndim() == 3 ? static_cast<size_t>(queries.shape(0)) : 1;
    const size_t qlen = static_cast<size_t>(queries.shape(queries.ndim() - 2));
    const size_t dim = static_cast<size_t>(queries.shape(queries.ndim() - 1));
    const float* data = queries.data();
    if (queries.ndim() == 2) {
        std::vector<size_t> r;
        {
            py::gil_scoped_release release;
            r = index.search(data, qlen * dim, k);
        }
        return py::cast(std::move(r));
    }
    if (qlen != 32) throw std::invalid_argument("A Chimera query must have 32 tokens");
    std::vector<std::vector<size_t>> r;
    {
        py::gil_scoped_release release;
        if (nq > 0) {
            // the per-query shape check of chimera_index::search
            index.search(data, qlen * dim, k);
            r = index.search_batch(data, nq, k);
        }
    }
    return py::cast(std::move(r));
}

void save(const chimera_index& index, const std::string& dir) {
    py::gil_scoped_release release;
    index.save(dir);
}

}  // namespace

PYBIND11_MODULE(chimera, m) {
    const SearchOptions d;
    auto cls = py::class_<chimera_index>(m, "ChimeraIndex");
    cls.def_static("build", &build, py::arg("embeddings").noconvert(), py::arg("doc_lens"), py::arg("n_clusters"),
                   py::arg("ex_bits"), py::arg("nprobe") = d.nprobe, py::arg("k_refine") = d.k_refine,
                   py::arg("k_full_bit") = d.k_full_bit, py::arg("cagra_itopk_size") = d.cagra_itopk_size,
                   py::arg("num_chunks") = d.num_chunks, py::arg("batch") = d.batch)
        .def("search", &search, py::arg("queries").noconvert(), py::arg("k") = 100)
        .def("save", &save, py::arg("index_dir"))
        .def_static("load", &load, py::arg("index_dir"), py::arg("nprobe") = d.nprobe,
                    py::arg("k_refine") = d.k_refine, py::arg("k_full_bit") = d.k_full_bit,
                    py::arg("cagra_itopk_size") = d.cagra_itopk_size, py::arg("num_chunks") = d.num_chunks,
                    py::arg("batch") = d.batch);
}
