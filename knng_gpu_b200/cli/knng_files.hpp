// knng_files.hpp -- the file formats around the brute-force path, in plain
// C++17 (no dependency on the reference's headers):
//   * .fvecs / .ivecs / .bvecs records (include/knng/io/fvecs.hpp:9-30):
//     per record a little-endian int32 dim, then dim elements; n recovered
//     from the file size; every record's dim must match the first.
//   * .knng v1 graph files (tools/build_knng.cpp:13-33): 64-byte header
//     "KNNGRAPH", version 1, index width 4, distance width 4, metric id,
//     algorithm id, n, k, 20 reserved bytes; then n*k uint32 ids and n*k
//     float32 distances.
//   * ground-truth cache files (src/bench/ground_truth.cpp:36-40, 165-234):
//     "KNNGRDTR", version 1, widths, metric id, FNV-1a 64 dataset hash, n, k,
//     16 reserved bytes, ids, distances; written to <path>.tmp and renamed.
//   * dataset_hash: FNV-1a 64 over (u64 n, u64 d, fp32 payload)
//     (src/bench/ground_truth.cpp:45-56, 90-101).
#pragma once

#include <array>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace knng_files {

template <class Element>
void read_vecs(const std::string& path, std::vector<Element>& out, std::uint64_t& n, std::uint64_t& d)
{
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("knng::io: could not open '" + path + "'");
    std::fseek(f, 0, SEEK_END);
    const long long total = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    auto fail = [&](const std::string& msg) {
        std::fclose(f);
        throw std::runtime_error(msg);
    };
    if (total < 4) fail("knng::io: file too small to hold a single record: '" + path + "'");
    std::int32_t dim0 = 0;
    if (std::fread(&dim0, 4, 1, f) != 1) fail("knng::io: read failed: '" + path + "'");
    if (dim0 <= 0) fail("knng::io: invalid dim prefix " + std::to_string(dim0) + " in '" + path + "'");
    const std::uint64_t rec = 4 + static_cast<std::uint64_t>(dim0) * sizeof(Element);
    if (static_cast<std::uint64_t>(total) % rec != 0)
        fail("knng::io: file size " + std::to_string(total) + " is not a multiple of record size " +
             std::to_string(rec) + " for '" + path + "'");
    n = static_cast<std::uint64_t>(total) / rec;
    d = static_cast<std::uint64_t>(dim0);
    out.resize(n * d);
    std::fseek(f, 0, SEEK_SET);
    std::vector<unsigned char> buf(rec);
    for (std::uint64_t i = 0; i < n; ++i) {
        if (std::fread(buf.data(), 1, rec, f) != rec) fail("knng::io: read failed: '" + path + "'");
        std::int32_t dim = 0;
        std::memcpy(&dim, buf.data(), 4);
        if (dim != dim0)
            fail("knng::io: record " + std::to_string(i) + " has dim " + std::to_string(dim) +
                 " but the first record has dim " + std::to_string(dim0) + " in '" + path + "'");
        std::memcpy(out.data() + i * d, buf.data() + 4, d * sizeof(Element));
    }
    std::fclose(f);
}

inline std::uint64_t fnv1a64(std::uint64_t state, const void* bytes, std::uint64_t n)
{
    const auto* p = static_cast<const unsigned char*>(bytes);
    for (std::uint64_t i = 0; i < n; ++i) {
        state ^= p[i];
        state *= 1099511628211ull;
    }
    return state;
}

inline std::uint64_t dataset_hash(const float* x, std::uint64_t n, std::uint64_t d)
{
    std::uint64_t s = 14695981039346656037ull;
    s = fnv1a64(s, &n, 8);
    s = fnv1a64(s, &d, 8);
    if (n * d) s = fnv1a64(s, x, n * d * 4);
    return s;
}

// The same hash for u8 rows, over the bytes of their float values (what the
// reference hashes after loading .bvecs as floats), without a float copy.
inline std::uint64_t dataset_hash_u8(const std::uint8_t* x, std::uint64_t n, std::uint64_t d)
{
    std::uint64_t s = 14695981039346656037ull;
    s = fnv1a64(s, &n, 8);
    s = fnv1a64(s, &d, 8);
    for (std::uint64_t i = 0; i < n * d; ++i) {
        const float f = static_cast<float>(x[i]);
        s = fnv1a64(s, &f, 4);
    }
    return s;
}

struct Graph {
    std::uint64_t n = 0, k = 0;
    std::vector<std::uint32_t> ids;
    std::vector<float> dists;
};

inline void write_all(std::FILE* f, const void* p, std::size_t bytes, const std::string& path)
{
    if (bytes && std::fwrite(p, 1, bytes, f) != bytes) {
        std::fclose(f);
        throw std::runtime_error("write to '" + path + "' failed");
    }
}

// .knng v1 (tools/build_knng.cpp:196-233).
inline void write_knng(const std::string& path, const Graph& g, std::uint32_t metric, std::uint32_t algorithm)
{
    std::FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) throw std::runtime_error("could not open output for writing: '" + path + "'");
    const char magic[8] = {'K', 'N', 'N', 'G', 'R', 'A', 'P', 'H'};
    const std::uint32_t version = 1, iw = 4, dw = 4;
    const std::array<char, 20> reserved{};
    write_all(f, magic, 8, path);
    write_all(f, &version, 4, path);
    write_all(f, &iw, 4, path);
    write_all(f, &dw, 4, path);
    write_all(f, &metric, 4, path);
    write_all(f, &algorithm, 4, path);
    write_all(f, &g.n, 8, path);
    write_all(f, &g.k, 8, path);
    write_all(f, reserved.data(), reserved.size(), path);
    write_all(f, g.ids.data(), g.ids.size() * 4, path);
    write_all(f, g.dists.data(), g.dists.size() * 4, path);
    std::fclose(f);
}

// Ground-truth cache (src/bench/ground_truth.cpp:165-234): tmp file + rename.
inline void save_ground_truth(const std::string& path, const Graph& g, std::uint64_t hash, std::uint32_t metric)
{
    const std::string tmp = path + ".tmp";
    std::FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) throw std::runtime_error("knng::bench::save_ground_truth: could not open '" + tmp + "' for writing");
    const char magic[8] = {'K', 'N', 'N', 'G', 'R', 'D', 'T', 'R'};
    const std::uint32_t version = 1, iw = 4, dw = 4;
    const std::array<char, 16> reserved{};
    write_all(f, magic, 8, tmp);
    write_all(f, &version, 4, tmp);
    write_all(f, &iw, 4, tmp);
    write_all(f, &dw, 4, tmp);
    write_all(f, &metric, 4, tmp);
    write_all(f, &hash, 8, tmp);
    write_all(f, &g.n, 8, tmp);
    write_all(f, &g.k, 8, tmp);
    write_all(f, reserved.data(), reserved.size(), tmp);
    write_all(f, g.ids.data(), g.ids.size() * 4, tmp);
    write_all(f, g.dists.data(), g.dists.size() * 4, tmp);
    std::fclose(f);
    if (std::rename(tmp.c_str(), path.c_str()) != 0)
        throw std::runtime_error("knng::bench::save_ground_truth: rename of '" + tmp + "' failed");
}

}  // namespace knng_files
