// build_knng_gpu -- the reference's build_knng (tools/build_knng.cpp) with a
// GPU builder: same flags, same .knng v1 output, graphs bit-identical to
// knng::cpu::brute_force_knn.
//
//   build_knng_gpu --dataset PATH --k N [--metric l2|inner_product]
//                  [--algorithm brute_force_gpu|brute_force] [--output PATH]
//                  [--ground-truth PATH] [--device I] [--gpus N]
//
// .fvecs datasets are read as in the reference; .bvecs datasets (u8 rows) are
// read directly and feed the exact u8 tensor-core path. The header's
// algorithm_id is 1 for brute_force_gpu (the reference only defines 0 =
// brute_force, tools/build_knng.cpp:27); `--algorithm brute_force` writes 0,
// since the graph is the reference's brute-force graph bit for bit.
// --ground-truth additionally writes the graph as a ground-truth cache file
// (src/bench/ground_truth.cpp format) keyed by the dataset hash.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <exception>
#include <iostream>
#include <map>
#include <optional>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include "knng_files.hpp"
#include "knng_gpu.h"

namespace {

constexpr std::string_view kUsage =
    "Usage: build_knng_gpu --dataset PATH --k N [options]\n"
    "\n"
    "Required:\n"
    "  --dataset PATH        Path to a .fvecs or .bvecs dataset.\n"
    "  --k N                 Neighbors per point. Must satisfy 1 <= k <= n-1.\n"
    "\n"
    "Optional:\n"
    "  --metric M            l2 (default) | inner_product\n"
    "  --algorithm A         brute_force_gpu (default) | brute_force (same graph, algorithm_id 0)\n"
    "  --output PATH         Output .knng path (default: <dataset>.knng)\n"
    "  --ground-truth PATH   Also write a ground-truth cache file\n"
    "  --device I            CUDA device (default 0)\n"
    "  --gpus N              Build on GPUs 0..N-1 of this node (default 1)\n"
    "  --help                Print this message and exit\n";

struct Args {
    std::string dataset, output, ground_truth;
    std::uint64_t k = 0;
    std::string metric = "l2";
    std::string algorithm = "brute_force_gpu";
    int device = 0;
    int gpus = 1;
};

std::uint64_t parse_size(const std::string& s, const char* flag)
{
    if (s.empty()) throw std::invalid_argument(std::string{"empty value for "} + flag);
    std::size_t pos = 0;
    const unsigned long long v = std::stoull(s, &pos, 10);
    if (pos != s.size()) throw std::invalid_argument(std::string{"trailing garbage in value for "} + flag + ": '" + s + "'");
    return v;
}

// Every accepted flag, in the order its value is checked: the reference's
// flag names and error messages (tools/build_knng.cpp:100-179), plus
// --ground-truth, --device and --gpus.
struct FlagSpec {
    const char* name;
    bool required;
    void (*apply)(Args&, const std::string&);
};

const FlagSpec kFlags[] = {
    {"dataset", true, [](Args& a, const std::string& v) { a.dataset = v; }},
    {"k", true, [](Args& a, const std::string& v) { a.k = parse_size(v, "--k"); }},
    {"metric", false, [](Args& a, const std::string& v) { a.metric = v; }},
    {"algorithm", false, [](Args& a, const std::string& v) { a.algorithm = v; }},
    {"output", false, [](Args& a, const std::string& v) { a.output = v; }},
    {"ground-truth", false, [](Args& a, const std::string& v) { a.ground_truth = v; }},
    {"device", false, [](Args& a, const std::string& v) { a.device = static_cast<int>(parse_size(v, "--device")); }},
    {"gpus", false, [](Args& a, const std::string& v) { a.gpus = static_cast<int>(parse_size(v, "--gpus")); }},
};

const FlagSpec* find_flag(const std::string& name)
{
    for (const FlagSpec& f : kFlags)
        if (name == f.name) return &f;
    return nullptr;
}

// argv -> Args in three steps: split into (--name, value) pairs, apply the
// spec table (a repeated flag keeps its last value), then check the values
// against each other. nullopt: --help.
std::optional<Args> parse_args(int argc, char** argv)
{
    std::vector<std::pair<std::string, std::string>> given;
    for (int i = 1; i < argc; i += 2) {
        const std::string tok = argv[i];
        if (tok == "--help" || tok == "-h") return std::nullopt;
        if (tok.rfind("--", 0) != 0) throw std::invalid_argument("unexpected positional argument: '" + tok + "'");
        if (i + 1 >= argc) throw std::invalid_argument("flag '" + tok + "' requires a value");
        given.emplace_back(tok.substr(2), argv[i + 1]);
    }
    Args a;
    for (const FlagSpec& f : kFlags) {
        const std::string* value = nullptr;
        for (const auto& [name, v] : given)
            if (name == f.name) value = &v;
        if (value)
            f.apply(a, *value);
        else if (f.required)
            throw std::invalid_argument(std::string{"missing required flag --"} + f.name);
    }
    std::string unknown;  // the alphabetically first unknown flag is reported
    for (const auto& [name, v] : given)
        if (!find_flag(name) && (unknown.empty() || name < unknown)) unknown = name;
    if (!unknown.empty()) throw std::invalid_argument("unknown flag --" + unknown);
    if (a.k == 0) throw std::invalid_argument("--k must be > 0");
    if (a.output.empty()) a.output = a.dataset + ".knng";
    if (a.metric != "l2" && a.metric != "inner_product")
        throw std::invalid_argument("--metric must be 'l2' or 'inner_product', got '" + a.metric + "'");
    if (a.algorithm != "brute_force_gpu" && a.algorithm != "brute_force")
        throw std::invalid_argument("--algorithm must be 'brute_force_gpu' or 'brute_force', got '" + a.algorithm + "'");
    if (a.gpus < 1) throw std::invalid_argument("--gpus must be > 0");
    return a;
}

bool ends_with(const std::string& s, const std::string& suffix)
{
    return s.size() >= suffix.size() && s.compare(s.size() - suffix.size(), suffix.size(), suffix) == 0;
}

}  // namespace

int main(int argc, char** argv)
{
    Args args;
    try {
        auto parsed = parse_args(argc, argv);
        if (!parsed) {
            std::cout << kUsage;
            return 0;
        }
        args = *parsed;
    } catch (const std::exception& e) {
        std::cerr << "build_knng_gpu: " << e.what() << "\n\n" << kUsage;
        return 2;
    }
    try {
        std::cerr << "build_knng_gpu: loading " << args.dataset << '\n';
        // .bvecs rows stay bytes all the way to the device (u8 ingest, no
        // float round trip); .fvecs rows go through the fp32 entry point.
        std::vector<float> x;
        std::vector<std::uint8_t> raw;
        const bool bytes = ends_with(args.dataset, ".bvecs");
        std::uint64_t n = 0, d = 0;
        if (bytes)
            knng_files::read_vecs<std::uint8_t>(args.dataset, raw, n, d);
        else
            knng_files::read_vecs<float>(args.dataset, x, n, d);
        std::cerr << "build_knng_gpu: loaded n=" << n << " d=" << d << '\n';
        if (args.gpus == 1 && cudaSetDevice(args.device) != cudaSuccess)
            throw std::runtime_error("cudaSetDevice failed");
        const std::uint32_t metric = args.metric == "l2" ? KNNG_METRIC_L2_SQUARED : KNNG_METRIC_NEGATIVE_INNER_PRODUCT;
        std::cerr << "build_knng_gpu: building k=" << args.k << " metric=" << args.metric
                  << " algorithm=" << args.algorithm << '\n';
        knng_files::Graph g;
        g.n = n;
        g.k = args.k;
        g.ids.resize(n * args.k);
        g.dists.resize(n * args.k);
        knng_gpu_stats stats{};
        knng_gpu_status st;
        if (args.gpus > 1) {
            // Devices 0..gpus-1 from this process (NCCL inside the library).
            if (bytes) x.assign(raw.begin(), raw.end());
            st = knng_gpu_brute_force_multi(x.data(), n, d, args.k, static_cast<int>(metric), args.gpus, 0,
                                            g.ids.data(), g.dists.data(), &stats);
        } else {
            st = bytes ? knng_gpu_brute_force_u8(raw.data(), n, d, d, args.k, static_cast<int>(metric), g.ids.data(),
                                                 g.dists.data(), &stats)
                       : knng_gpu_brute_force(x.data(), n, d, args.k, static_cast<int>(metric), g.ids.data(),
                                              g.dists.data(), &stats);
        }
        if (st != KNNG_GPU_OK) throw std::runtime_error(knng_gpu_last_error());
        std::cerr << "build_knng_gpu: device time " << stats.total_ms << " ms (path "
                  << (stats.path == KNNG_PATH_U8_TENSOR ? "u8 tensor" : "fp32 tensor") << ")\n";
        std::cerr << "build_knng_gpu: writing " << args.output << '\n';
        knng_files::write_knng(args.output, g, metric, args.algorithm == "brute_force" ? 0u : 1u);
        if (!args.ground_truth.empty()) {
            const std::uint64_t hash =
                bytes ? knng_files::dataset_hash_u8(raw.data(), n, d) : knng_files::dataset_hash(x.data(), n, d);
            knng_files::save_ground_truth(args.ground_truth, g, hash, metric);
            std::cerr << "build_knng_gpu: wrote ground truth " << args.ground_truth << '\n';
        }
        std::cerr << "build_knng_gpu: done\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "build_knng_gpu: " << e.what() << '\n';
        return 1;
    }
}
