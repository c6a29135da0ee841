// translate_ids: a graph or index from the reordered id space back to the original order,
// with the reference tool's options and behaviour (bucketDemo/buildBucket/src/translate_ids.cpp,
// translate_graph_ids.hpp:75-200):
//
//   translate_ids -g graph_new_ids.bin -p inverse_perm.bin -o final_graph.bin
//   translate_ids -g neighbors.npy     -p inverse_perm.bin -o neighbors_orig.npy
//
// Row inverse_perm[i] of the output is row i of the input with every id v replaced by
// inverse_perm[v] (on the GPU).  A .bin graph (int64 N, int32 K, uint32) must hold ids < N;
// a .npy (int64) keeps -1 padding.  inverse_perm.bin must hold exactly N uint32 forming a
// permutation.  Exit status 0 ok, 1 error ("FATAL: ...").
#include <chrono>
#include <cstdio>
#include <string>
#include <vector>

#include "args.hpp"
#include "gta.h"

namespace {

void check(int rc, const char* what)
{
    if (rc != GTA_OK) throw std::runtime_error(std::string(what) + ": " + gta_last_error());
}

bool ends_with(const std::string& s, const char* t)
{
    const std::string e(t);
    return s.size() >= e.size() && s.compare(s.size() - e.size(), e.size(), e) == 0;
}

int run(int argc, char** argv)
{
    const std::vector<cli::Opt> opts = {
        {"graph", 'g', false, "Graph in the reordered id space (.bin graph or .npy)", ""},
        {"inverse-perm", 'p', false, "inverse_perm.bin (inverse_perm[new_id] = old_id)", ""},
        {"output", 'o', false, "Output, same format, rows and ids in the original order", ""},
        {"out-buffer-mb", 0, false, "(accepted; the whole graph is translated in one pass)", "1024"},
    };
    cli::Args a("translate_ids (gta-b200)", opts);
    if (!a.parse(argc, argv)) return 0;
    const std::string gpath = a.required("graph");
    const std::string ppath = a.required("inverse-perm");
    const std::string opath = a.required("output");
    const auto t0 = std::chrono::steady_clock::now();
    const bool npy = ends_with(gpath, ".npy");
    int64_t n = 0;
    int32_t k = 0;
    if (npy) check(gta_read_npy_i64_header(gpath.c_str(), &n, &k), "read npy header");
    else check(gta_read_graph_header(gpath.c_str(), &n, &k), "read graph header");
    int64_t n_inv = 0;
    check(gta_read_u32_count(ppath.c_str(), &n_inv), "read inverse_perm");
    if (n_inv != n)
        throw std::runtime_error(ppath + " holds " + std::to_string(n_inv) + " ids, graph N=" + std::to_string(n));
    std::vector<uint32_t> inv(static_cast<size_t>(n));
    check(gta_read_u32(ppath.c_str(), inv.data()), "read inverse_perm");
    std::vector<int32_t> g(static_cast<size_t>(n) * k), out(g.size());
    if (npy) check(gta_read_npy_i64(gpath.c_str(), g.data()), "read npy");
    else check(gta_read_graph(gpath.c_str(), reinterpret_cast<uint32_t*>(g.data())), "read graph");
    check(gta_permute_graph(g.data(), n, k, inv.data(), 1, npy ? 1 : 0, out.data(), 0, nullptr), "translate");
    if (npy) check(gta_write_npy_i64(opath.c_str(), out.data(), n, k), "write npy");
    else check(gta_write_graph(opath.c_str(), reinterpret_cast<const uint32_t*>(out.data()), n, k), "write graph");
    std::printf("Wrote %s [%.3fs]\n", opath.c_str(),
                std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
    return 0;
}

}  // namespace

int main(int argc, char** argv)
{
    try {
        return run(argc, argv);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FATAL: %s\n", e.what());
        return 1;
    }
}
