// gpu_build: same flags and behaviour as the reference CLI (cpp/apps/build.cpp:9-35).
#include <iostream>

#include "chimera/chimera_index.cuh"
#include "chimera/io.hpp"
#include "cli.hpp"

using namespace Chimera;

int main(int argc, char** argv) {
    BuildCliArgs args;
    try {
        args = parse_build_args(argc, argv);
    } catch (const HelpRequested&) {
        print_build_help(argv[0]);
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "Argument error: " << e.what() << "\n\n";
        print_build_help(argv[0]);
        return 1;
    }
    auto doc_lens = load_doclens(args.doclens_file);
    size_t n = 0, d = 0;
    auto emb = load_data(n, d, args.data_file);
    chimera_index index;
    index.build(emb, d, doc_lens, args.n_clusters, args.ex_bits);
    index.save(args.index_dir);
    return 0;
}
