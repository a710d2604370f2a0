// CLI helpers with the reference's behaviour (cpp/apps/utils.cpp:52-290),
// including its quirks: read_gt_tsv exits(0) on an out-of-range rank and
// compute_recall divides by num_queries * k.
#include "cli.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <numeric>
#include <sstream>
#include <stdexcept>
#include <unordered_set>

namespace Chimera {
namespace {

std::string value_of(int argc, char** argv, int& i, const std::string& flag) {
    if (i + 1 >= argc) throw std::runtime_error("Missing value for " + flag);
    return argv[++i];
}

void check_options(const SearchOptions& o) {
    if (o.nprobe <= 0) throw std::runtime_error("--nprobe must be > 0");
    if (o.k_refine <= 0) throw std::runtime_error("--k-refine must be > 0");
    if (o.k_full_bit <= 0) throw std::runtime_error("--k-full-bit must be > 0");
    if (o.cagra_itopk_size <= 0) throw std::runtime_error("--cagra-itopk-size must be > 0");
    if (o.num_chunks <= 0) throw std::runtime_error("--num-chunks must be > 0");
    if (o.k_full_bit > o.k_refine) throw std::runtime_error("--k-full-bit must not exceed --k-refine");
}

}  // namespace

BuildCliArgs parse_build_args(int argc, char** argv) {
    if (argc == 1) throw HelpRequested{};
    BuildCliArgs a;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--help" || arg == "-h") throw HelpRequested{};
        if (arg == "--index" || arg == "-i") a.index_dir = value_of(argc, argv, i, arg);
        else if (arg == "--doclens" || arg == "-d") a.doclens_file = value_of(argc, argv, i, arg);
        else if (arg == "--data") a.data_file = value_of(argc, argv, i, arg);
        else if (arg == "--n-clusters") a.n_clusters = std::stoull(value_of(argc, argv, i, arg));
        else if (arg == "--ex-bits") a.ex_bits = std::stoull(value_of(argc, argv, i, arg));
        else throw std::runtime_error("Unknown argument: " + arg);
    }
    if (a.index_dir.empty() || a.doclens_file.empty() || a.data_file.empty() || a.n_clusters == 0 || a.ex_bits == 0)
        throw std::runtime_error("Missing required arguments.");
    return a;
}

SearchCliArgs parse_search_args(int argc, char** argv) {
    if (argc == 1) throw HelpRequested{};
    SearchCliArgs a;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--help" || arg == "-h") throw HelpRequested{};
        if (arg == "--query" || arg == "-q") a.query_file = value_of(argc, argv, i, arg);
        else if (arg == "--gt" || arg == "-g") a.gt_file = value_of(argc, argv, i, arg);
        else if (arg == "--index" || arg == "-i") a.index_dir = value_of(argc, argv, i, arg);
        else if (arg == "--k") a.k = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--nq") a.nq = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--warmup") a.warmup = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--nprobe") a.options.nprobe = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--k-refine") a.options.k_refine = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--k-full-bit") a.options.k_full_bit = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--cagra-itopk-size") a.options.cagra_itopk_size = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--num-chunks") a.options.num_chunks = std::stoi(value_of(argc, argv, i, arg));
        else if (arg == "--batch") a.batch = std::stoi(value_of(argc, argv, i, arg));
        else throw std::runtime_error("Unknown argument: " + arg);
    }
    if (a.query_file.empty() || a.gt_file.empty() || a.index_dir.empty())
        throw std::runtime_error("Missing required arguments.");
    if (!std::filesystem::is_directory(a.index_dir))
        throw std::runtime_error("--index must point to a Chimera index directory.");
    if (!std::filesystem::exists(std::filesystem::path(a.index_dir) / "doclens.bin"))
        throw std::runtime_error("Missing doclens.bin in --index.");
    if (a.k <= 0) throw std::runtime_error("--k must be > 0");
    if (a.warmup < 0) throw std::runtime_error("--warmup must be >= 0");
    if (a.batch < 0) throw std::runtime_error("--batch must be >= 0");
    check_options(a.options);
    if (a.batch > 0) a.options.batch = a.batch;
    return a;
}

void print_build_help(const char* program) {
    std::cout << "Usage: " << program
              << " --index <index_dir> --doclens <doclens> --data <data> --n-clusters <count> --ex-bits <count>\n\n"
              << "Arguments:\n"
              << "  --index, -i      Output index directory.\n"
              << "  --doclens, -d    Input document-length file.\n"
              << "  --data           Input token-embedding file.\n"
              << "  --n-clusters     Number of IVF centroids.\n"
              << "  --ex-bits        Residual quantization bits per dimension (1-7).\n";
}

void print_search_help(const char* program) {
    const SearchCliArgs d;
    std::cout << "Usage: " << program << "\n"
              << "  --query <query_embeddings.bin>\n"
              << "  --gt <groundtruth.tsv>\n"
              << "  --index <index_dir>\n"
              << "  [--k <top_k>]                   Final documents returned. Default: " << d.k << "\n"
              << "  [--nq <num_queries>]            Evaluation queries; -1 means all. Default: " << d.nq << "\n"
              << "  [--warmup <num_queries>]        Warmup queries. Default: " << d.warmup << "\n"
              << "  [--nprobe <num_probes>]         IVF clusters probed per query token. Default: "
              << d.options.nprobe << "\n"
              << "  [--k-refine <count>]            Candidates retained after refinement. Default: "
              << d.options.k_refine << "\n"
              << "  [--k-full-bit <count>]          Candidates scored with full-bit codes. Default: "
              << d.options.k_full_bit << "\n"
              << "  [--cagra-itopk-size <count>]    Accepted for compatibility (the probe is exact). Default: "
              << d.options.cagra_itopk_size << "\n"
              << "  [--num-chunks <count>]          Collaborative-scoring chunks. Default: " << d.options.num_chunks
              << "\n"
              << "  [--batch <count>]               Also time batched search of <count> queries per GPU pass.\n";
}

double percentile_ms(const std::vector<double>& s, double pct) {  // linear interpolation
    if (s.empty()) return 0.0;
    const double c = std::clamp(pct, 0.0, 100.0);
    const double pos = (c / 100.0) * static_cast<double>(s.size() - 1);
    const size_t lo = static_cast<size_t>(std::floor(pos)), hi = static_cast<size_t>(std::ceil(pos));
    const double w = pos - static_cast<double>(lo);
    return s[lo] * (1.0 - w) + s[hi] * w;
}

QueryLatencySummary summarize_query_latencies_ms(const std::vector<double>& lat) {
    QueryLatencySummary r;
    if (lat.empty()) return r;
    std::vector<double> s = lat;
    std::sort(s.begin(), s.end());
    r.mean_ms = std::accumulate(s.begin(), s.end(), 0.0) / static_cast<double>(s.size());
    double sq = 0.0;
    for (double x : s) sq += (x - r.mean_ms) * (x - r.mean_ms);
    r.stddev_ms = std::sqrt(sq / static_cast<double>(s.size()));
    r.min_ms = s.front();
    r.p50_ms = percentile_ms(s, 50.0);
    r.p90_ms = percentile_ms(s, 90.0);
    r.p95_ms = percentile_ms(s, 95.0);
    r.p99_ms = percentile_ms(s, 99.0);
    r.max_ms = s.back();
    return r;
}

std::vector<std::vector<size_t>> read_gt_tsv(int num_queries, int top_k, const std::string& gt_filename) {
    std::vector<std::vector<size_t>> gt(num_queries, std::vector<size_t>(top_k, static_cast<size_t>(-1)));
    std::ifstream file(gt_filename);
    if (!file.is_open()) {
        std::cerr << "Error: Could not open file " << gt_filename << std::endl;
        return gt;
    }
    std::string line;
    while (std::getline(file, line)) {
        std::stringstream ss(line);
        std::string seg;
        std::vector<std::string> f;
        while (std::getline(ss, seg, '\t')) f.push_back(seg);
        if (f.size() < 3) {
            std::cerr << "Warning: Skipping malformed line." << std::endl;
            continue;
        }
        const int qid = std::stoi(f[0]);
        const size_t item = std::stoull(f[1]);
        const int rank = std::stoi(f[2]);
        if (rank - 1 >= top_k || rank - 1 < 0) {
            std::cerr << "Warning: Rank " << rank << " exceeds top_k " << top_k << ". Skipping." << std::endl;
            std::exit(0);
        }
        if (qid >= 0 && qid < num_queries) gt[qid][rank - 1] = item;
    }
    return gt;
}

double compute_recall(const std::vector<std::vector<size_t>>& gt, const std::vector<std::vector<size_t>>& got,
                      int top_k) {
    if (top_k <= 0) return 0.0;
    const int nq = static_cast<int>(got.size());
    int hits = 0;
    for (int i = 0; i < nq; ++i) {
        const auto& r = got[i];
        const size_t cut = std::min(r.size(), static_cast<size_t>(top_k));
        const std::unordered_set<size_t> rs(r.begin(), r.begin() + cut);
        const int gc = std::min<int>(top_k, static_cast<int>(gt[i].size()));
        for (int j = 0; j < gc; ++j) hits += rs.count(gt[i][j]) != 0;
    }
    return static_cast<double>(hits) / (nq * top_k);
}

}  // namespace Chimera
