// test_residency.cpp — the row log of FlatIndexMemory and the device
// residency built on it (include/heteromm/residency.h).
//
// Without arguments (CPU only): the log's entries, their generation chain, its
// bound, and that set_data and copies break the chain.
//
// With --gpu: GPU steps after inserts, pops and erases (one at a time and
// mixed, at random positions) agree with the CPU arm and upload only the
// appended rows and the query; a log longer than its bound, a copy and
// set_data fall back to a full upload and still agree; make_resident /
// release / is_resident; held copies of GPU_MEM-tagged memories outlive
// cycling through more memories than the cache holds; a KV cache made
// resident is not uploaded again by the attention step.  Times of a full
// upload and of an append at 65,536 x 128 are printed.
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "heteromm/dev/steps/apply_memory.h"
#include "heteromm/dev/steps/compute_score.h"
#include "heteromm/dev/steps/fused_steps/template.h"
#include "heteromm/dev/steps/memory_retrieval.h"
#include "heteromm/residency.h"

using namespace heteromm;
using data_type::FlatIndexMemory;
using Rows = std::vector<std::vector<float>>;

static int g_fail = 0;
#define CHECK(cond)                                                      \
    do {                                                                 \
        if (!(cond)) {                                                   \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); \
            ++g_fail;                                                    \
        }                                                                \
    } while (0)

static std::mt19937 g_rng(7);
static std::vector<float> vec(size_t d) {
    std::normal_distribution<float> nd(0.0f, 1.0f);
    std::vector<float> v(d);
    for (auto& x : v) x = nd(g_rng);
    return v;
}
static Rows matrix(size_t n, size_t d) {
    Rows r(n);
    for (auto& row : r) row = vec(d);
    return r;
}

static void test_log_cpu() {
    FlatIndexMemory<float> m(matrix(10, 4));
    CHECK(m.row_deltas().empty());
    const uint64_t g0 = m.generation();
    const std::vector<float> row = vec(4);
    m.insert_memory(row);
    m.delete_memory(3);
    m.pop_last_memory();
    const auto& log = m.row_deltas();
    CHECK(log.size() == 3);
    CHECK(log[0].kind == FlatIndexMemory<float>::RowDelta::Append && log[0].index == 10 &&
          log[0].row == row && log[0].from == g0);
    CHECK(log[1].kind == FlatIndexMemory<float>::RowDelta::Erase && log[1].index == 3);
    CHECK(log[2].kind == FlatIndexMemory<float>::RowDelta::PopLast && log[2].index == 9);
    CHECK(log[0].to == log[1].from && log[1].to == log[2].from && log[2].to == m.generation());
    CHECK(m.get_num_entries() == 9);

    FlatIndexMemory<float> copy = m;   // a generation of its own: the inherited log never ends at it
    CHECK(copy.row_deltas().size() == 3 && copy.row_deltas().back().to != copy.generation());
    copy.insert_memory(row);
    CHECK(copy.row_deltas().back().from == copy.row_deltas()[3].from &&
          copy.row_deltas()[2].to != copy.row_deltas()[3].from);

    for (size_t i = 0; i < FlatIndexMemory<float>::kMaxRowDeltas + 10; ++i) m.insert_memory(row);
    CHECK(m.row_deltas().size() == FlatIndexMemory<float>::kMaxRowDeltas);
    CHECK(m.row_deltas().back().to == m.generation());
    m.set_data(matrix(5, 4));
    CHECK(m.row_deltas().empty() && m.get_num_entries() == 5);
}

// GPU and CPU arms of the fused inner-product top-k and of the scores agree;
// returns the host->device bytes the two GPU calls moved.
static uint64_t agree(const FlatIndexMemory<float>& m, const data_type::VectorQuery<float>& q,
                      const char* what) {
    data_type::TopKIndex cpu, gpu;
    data_type::VectorScore<float> sc_cpu, sc_gpu;
    step::InnerProductTopKRetrieval s(25);
    s.execute(m, q, cpu);
    step::InnerProductCompute c;
    c.execute(m, q, sc_cpu);
    const uint64_t b0 = gpu::h2d_bytes();
    s.set_kernel(step::KernelType::GPU);
    s.execute(m, q, gpu);
    c.set_current_kernel(step::KernelType::GPU);
    c.execute(m, q, sc_gpu);
    const uint64_t moved = gpu::h2d_bytes() - b0;
    if (cpu.export_data() != gpu.export_data() || sc_cpu.export_data() != sc_gpu.export_data()) {
        std::printf("FAIL: GPU differs from CPU after %s\n", what);
        ++g_fail;
    }
    return moved;
}

static void test_gpu() {
    const size_t d = 64;
    const data_type::VectorQuery<float> q(vec(d));
    const uint64_t qb = 2 * d * sizeof(float);   // the query, uploaded by each of the two steps
    FlatIndexMemory<float> m(matrix(3000, d));
    CHECK(!gpu::is_resident(m));
    CHECK(agree(m, q, "first use") == qb + 3000 * d * sizeof(float));
    CHECK(gpu::is_resident(m) && gpu::is_resident(m, d));
    CHECK(agree(m, q, "reuse") == qb);

    std::vector<float> big = vec(d);
    for (auto& x : big) x *= 50.0f;   // a row that wins
    m.insert_memory(big);
    CHECK(agree(m, q, "insert_memory") == qb + d * sizeof(float));
    for (int i = 0; i < 5; ++i) m.insert_memory(vec(d));
    CHECK(agree(m, q, "five inserts") == qb + 5 * d * sizeof(float));   // one copy of the run
    m.delete_memory(3000);   // the winning row
    CHECK(agree(m, q, "delete_memory of the winner") == qb);
    m.delete_memory(0);
    m.pop_last_memory();
    CHECK(agree(m, q, "delete_memory(0) + pop_last_memory") == qb);

    std::uniform_int_distribution<int> op(0, 9);
    for (int round = 0; round < 20; ++round) {   // mixed changes at random positions
        size_t appended = 0;
        for (int i = 0; i < 40; ++i) {
            const int o = op(g_rng);
            if (o < 5) {
                m.insert_memory(vec(d));
                ++appended;
            } else if (o < 8) {
                m.delete_memory(std::uniform_int_distribution<size_t>(0, m.get_num_entries() - 1)(g_rng));
            } else {
                m.pop_last_memory();
            }
        }
        const uint64_t moved = agree(m, q, "mixed changes");
        CHECK(moved <= qb + appended * d * sizeof(float));
    }

    // beyond the log's bound: a full upload, still right
    for (size_t i = 0; i < FlatIndexMemory<float>::kMaxRowDeltas + 1; ++i) m.insert_memory(vec(d));
    CHECK(agree(m, q, "a log past its bound") == qb + m.get_num_entries() * d * sizeof(float));
    // a modified copy and set_data: full uploads
    FlatIndexMemory<float> copy = m;
    copy.insert_memory(big);
    CHECK(agree(copy, q, "a modified copy") == qb + copy.get_num_entries() * d * sizeof(float));
    CHECK(agree(m, q, "its original") == qb);
    m.set_data(matrix(777, d));
    CHECK(agree(m, q, "set_data") == qb + 777 * d * sizeof(float));

    // make_resident / release
    FlatIndexMemory<float> r(matrix(2000, d));
    gpu::make_resident(r);
    CHECK(gpu::is_resident(r));
    CHECK(agree(r, q, "after make_resident") == qb);
    gpu::release(r);
    CHECK(!gpu::is_resident(r));

    // a GPU_MEM-tagged memory is held while more memories than the cache holds pass through
    FlatIndexMemory<float> pinned(matrix(1000, d));
    pinned.set_device(data_type::DataLocation::GPU_MEM);
    gpu::make_resident(pinned);
    std::vector<FlatIndexMemory<float>> others;
    for (int i = 0; i < 12; ++i) others.emplace_back(matrix(500 + i, d));
    for (auto& o : others) agree(o, q, "cycling memories");
    CHECK(gpu::is_resident(pinned));
    CHECK(agree(pinned, q, "held memory") == qb);
    FlatIndexMemory<float> untagged(matrix(1000, d));
    gpu::make_resident(untagged);
    for (auto& o : others) agree(o, q, "cycling memories");
    CHECK(!gpu::is_resident(untagged));   // replaced like any other copy
    gpu::release(pinned);

    // a resident KV cache: the attention step uploads only the query and the block ids
    const size_t L = 4096, D = 128;
    data_type::KVCacheData<float> kv(data_type::KVCache<float>{matrix(L, D), matrix(L, D)});
    gpu::make_resident(kv);
    step::BlockSparseAttention att(64);
    att.set_current_kernel(step::KernelType::GPU);
    data_type::TopKIndex blocks(std::vector<int>{5, 1, 63, 20});
    data_type::VectorInputOutputData<float> in(vec(D)), out_gpu, out_cpu;
    uint64_t b0 = gpu::h2d_bytes();
    att.execute(kv, blocks, in, out_gpu);
    CHECK(gpu::h2d_bytes() - b0 == D * sizeof(float) + 4 * sizeof(int));
    step::BlockSparseAttention att_cpu(64);
    att_cpu.execute(kv, blocks, in, out_cpu);
    const auto& a = out_gpu.data_ref();
    const auto& b = out_cpu.data_ref();
    bool close = a.size() == b.size();
    for (size_t i = 0; close && i < a.size(); ++i)
        close = std::fabs(a[i] - b[i]) <= 2e-6f + 2e-5f * std::fabs(b[i]);
    CHECK(close);

    // times at the flat-retrieval shape of config 1
    FlatIndexMemory<float> mem(matrix(65536, 128));
    const data_type::VectorQuery<float> q128(vec(128));
    step::InnerProductTopKRetrieval s(64);
    s.set_kernel(step::KernelType::GPU);
    data_type::TopKIndex out;
    auto ms = [&]() {
        const auto t0 = std::chrono::steady_clock::now();
        s.execute(mem, q128, out);
        return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    };
    const double first = ms();
    const double again = ms();
    double append = 0.0;
    for (int i = 0; i < 10; ++i) {
        mem.insert_memory(vec(128));
        append += ms() / 10;
    }
    double erase = 0.0;
    for (int i = 0; i < 10; ++i) {
        mem.delete_memory(1000 + i);
        erase += ms() / 10;
    }
    std::printf("InnerProductTopKRetrieval GPU, 65536 x 128: first call %.3f ms, unchanged %.3f ms, "
                "after one insert_memory %.3f ms, after one delete_memory %.3f ms\n",
                first, again, append, erase);
}

int main(int argc, char** argv) {
    const bool gpu = argc > 1 && std::strcmp(argv[1], "--gpu") == 0;
    try {
        test_log_cpu();
        if (gpu) test_gpu();
    } catch (const std::exception& e) {
        std::printf("FAIL: uncaught exception: %s\n", e.what());
        ++g_fail;
    }
    std::printf("%s: %d failure(s)\n", g_fail ? "FAILED" : "PASSED", g_fail);
    return g_fail ? 1 : 0;
}
