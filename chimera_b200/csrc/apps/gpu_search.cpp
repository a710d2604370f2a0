// gpu_search: same flags, warm-up, per-query timing loop and output lines as
// the reference CLI (cpp/apps/search.cpp:16-112).  `--batch B` (additive)
// also times batched search and prints one extra "[SEARCH] batched" line.
#include <algorithm>
#include <chrono>
#include <iomanip>
#include <iostream>

#include "chimera/chimera_index.cuh"
#include "chimera/io.hpp"
#include "cli.hpp"

using namespace Chimera;

namespace {
constexpr size_t kQlen = 32;

void report_recalls(const std::vector<std::vector<size_t>>& gt, const std::vector<std::vector<size_t>>& res, int k) {
    std::cout << "[SEARCH] recall@" << k << '=' << compute_recall(gt, res, k) << '\n';
    if (k == 100) std::cout << "[SEARCH] recall@10=" << compute_recall(gt, res, 10) << '\n';
}

void report_latency(const std::vector<double>& lat) {
    const auto s = summarize_query_latencies_ms(lat);
    std::cout << std::fixed << std::setprecision(3) << "[SEARCH] latency_ms" << " mean=" << s.mean_ms
              << " min=" << s.min_ms << " p50=" << s.p50_ms << " p90=" << s.p90_ms << " p95=" << s.p95_ms
              << " p99=" << s.p99_ms << " max=" << s.max_ms << " stddev=" << s.stddev_ms << '\n';
}
}  // namespace

int main(int argc, char** argv) {
    SearchCliArgs args;
    try {
        args = parse_search_args(argc, argv);
    } catch (const HelpRequested&) {
        print_search_help(argv[0]);
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "Argument error: " << e.what() << "\n\n";
        print_search_help(argv[0]);
        return 1;
    }
    size_t num_q = 0, d = 0, qlen = 0;
    std::vector<float> queries = load_query(qlen, num_q, d, args.query_file);
    auto gt = read_gt_tsv(static_cast<int>(num_q), 1000, args.gt_file);
    if (qlen != kQlen) {
        std::cerr << "Query length " << qlen << " does not match compiled Q_DOCLEN=" << kQlen << '\n';
        return 1;
    }
    const int warm = std::min<int>(args.warmup, static_cast<int>(num_q));
    const int run = args.nq < 0 ? static_cast<int>(num_q) : std::min<int>(args.nq, static_cast<int>(num_q));
    if (run == 0) {
        std::cerr << "No evaluation queries selected.\n";
        return 1;
    }
    std::vector<std::vector<size_t>> eval_gt(gt.begin(), gt.begin() + run);
    chimera_index index;
    index.load(args.index_dir, args.options);
    for (int i = 0; i < warm; ++i) index.search(&queries[i * kQlen * d], kQlen * d, args.k);
    std::vector<std::vector<size_t>> results(run);
    std::vector<double> lat(run);
    for (int i = 0; i < run; ++i) {
        const auto t0 = std::chrono::high_resolution_clock::now();
        results[i] = index.search(&queries[i * kQlen * d], kQlen * d, args.k);
        const auto t1 = std::chrono::high_resolution_clock::now();
        lat[i] = std::chrono::duration<double, std::milli>(t1 - t0).count();
    }
    report_latency(lat);
    report_recalls(eval_gt, results, args.k);
    if (args.batch > 0) {
        index.search_batch(queries.data(), std::min<size_t>(run, args.batch), args.k);  // warm-up
        const auto t0 = std::chrono::high_resolution_clock::now();
        auto batched = index.search_batch(queries.data(), run, args.k);
        const auto t1 = std::chrono::high_resolution_clock::now();
        const double s = std::chrono::duration<double>(t1 - t0).count();
        std::cout << std::fixed << std::setprecision(1) << "[SEARCH] batched qps=" << run / s
                  << " batch=" << args.batch << " queries=" << run << '\n';
        report_recalls(eval_gt, batched, args.k);
    }
    return 0;
}
