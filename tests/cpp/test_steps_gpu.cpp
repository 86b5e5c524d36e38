// GPU arms of the C++ step API against their CPU arms (same inputs, same
// step objects, KernelType::GPU vs KernelType::CPU).  Exits nonzero on the
// first mismatch.  Built and run by tests/test_step_api_gpu.py.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <stdexcept>
#include <unordered_map>
#include <utility>
#include <vector>

#include "heteromm/dev/steps/apply_memory.h"
#include "heteromm/dev/steps/build_memory.h"
#include "heteromm/dev/steps/compute_score.h"
#include "heteromm/dev/steps/fused_steps/template.h"
#include "heteromm/dev/steps/memory_retrieval.h"

using namespace heteromm;
using step::KernelType;

static int failures = 0;
#define EXPECT(cond, ...)                                 \
    do {                                                  \
        if (!(cond)) {                                    \
            std::printf("FAIL %s:%d: ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);                     \
            std::printf("\n");                            \
            ++failures;                                   \
        }                                                 \
    } while (0)

static std::vector<std::vector<float>> matrix(std::mt19937& g, size_t r, size_t c) {
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<std::vector<float>> m(r, std::vector<float>(c));
    for (auto& row : m)
        for (auto& v : row) v = nd(g);
    return m;
}

static std::vector<float> vec(std::mt19937& g, size_t n) { return matrix(g, 1, n)[0]; }

int main() {
    std::mt19937 g(1234);

    {   // InnerProductCompute: bit-exact fp32 scores
        data_type::FlatIndexMemory<float> mem(matrix(g, 3000, 96));
        data_type::VectorQuery<float> q(vec(g, 96));
        data_type::VectorScore<float> cpu, gpu;
        step::InnerProductCompute s;
        s.execute(mem, q, cpu);
        s.set_current_kernel(KernelType::GPU);
        s.execute(mem, q, gpu);
        EXPECT(cpu.export_data() == gpu.export_data(), "InnerProductCompute scores differ");
    }
    {   // TopKRetrieval with ties and k > n
        std::vector<float> sc = vec(g, 5000);
        for (size_t i = 0; i < sc.size(); i += 7) sc[i] = 1.5f;   // many exact ties
        data_type::VectorScore<float> score(sc);
        data_type::VectorScore<float> small(std::vector<float>(sc.begin(), sc.begin() + 3000));
        // k up to the device limit (4096), and k above n (all of n)
        for (auto kc : {std::make_pair(1u, &score), std::make_pair(17u, &score),
                        std::make_pair(300u, &score), std::make_pair(4096u, &score),
                        std::make_pair(6000u, &small)}) {
            data_type::TopKIndex cpu, gpu;
            step::TopKRetrieval s(kc.first);
            s.execute(*kc.second, cpu);
            s.set_current_kernel(KernelType::GPU);
            s.execute(*kc.second, gpu);
            EXPECT(cpu.export_data() == gpu.export_data(), "TopKRetrieval(k=%u) differs", kc.first);
        }
    }
    {   // ThresholdRetrieval: bitmap and selected list
        data_type::VectorScore<float> score(vec(g, 1000));
        data_type::ThresholdBitmapIndex cpu, gpu;
        step::ThresholdRetrieval s(0.5f);
        s.execute(score, cpu);
        s.set_current_kernel(KernelType::GPU);
        s.execute(score, gpu);
        EXPECT(cpu.export_data() == gpu.export_data(), "ThresholdRetrieval bitmap differs");
        EXPECT(cpu.get_selected_indices() == gpu.get_selected_indices(),
               "ThresholdRetrieval selection differs");
        EXPECT(gpu.get_total_length() == 1000, "ThresholdRetrieval total length");
    }
    {   // fused inner product + top-k
        data_type::FlatIndexMemory<float> mem(matrix(g, 4000, 64));
        data_type::VectorQuery<float> q(vec(g, 64));
        data_type::TopKIndex cpu, gpu;
        step::InnerProductTopKRetrieval s(10);
        s.execute(mem, q, cpu);
        s.set_kernel(KernelType::GPU);
        s.execute(mem, q, gpu);
        EXPECT(cpu.export_data() == gpu.export_data(), "InnerProductTopKRetrieval differs");
    }
    {   // PagedKVIndexBuilder: bit-exact page summaries, ragged last page
        data_type::KVCache<float> kv;
        kv.keys = matrix(g, 333, 64);
        kv.values = kv.keys;
        data_type::KVCacheData<float> raw(kv);
        data_type::FlatIndexMemory<float> cpu, gpu;
        step::PagedKVIndexBuilder s(matrix(g, 24, 64), 7);
        s.execute(raw, cpu);
        s.set_current_kernel(KernelType::GPU);
        s.execute(raw, gpu);
        EXPECT(cpu.export_data() == gpu.export_data(), "PagedKVIndexBuilder differs");
        EXPECT(gpu.export_data().size() == 48, "PagedKVIndexBuilder page count");
    }
    {   // BlockSparseAttention: fp32 tolerance (device expf, summation order)
        data_type::KVCache<float> kv;
        kv.keys = matrix(g, 500, 128);
        kv.values = matrix(g, 500, 128);
        data_type::KVCacheData<float> data(kv);
        data_type::TopKIndex blocks(std::vector<int>{3, 62, 0, 17, 100});   // 62: ragged, 100: past the end
        data_type::VectorInputOutputData<float> in(vec(g, 128)), cpu, gpu;
        step::BlockSparseAttention s(8);
        s.execute(data, blocks, in, cpu);
        s.set_current_kernel(KernelType::GPU);
        s.execute(data, blocks, in, gpu);
        const auto a = cpu.export_data(), b = gpu.export_data();
        EXPECT(a.size() == b.size(), "BlockSparseAttention size");
        for (size_t i = 0; i < a.size() && i < b.size(); ++i)
            EXPECT(std::fabs(a[i] - b[i]) <= 2e-6f + 2e-5f * std::fabs(a[i]),
                   "BlockSparseAttention[%zu] %g vs %g", i, a[i], b[i]);
        bool threw = false;   // a negative block id is reported, not followed
        try {
            data_type::TopKIndex bad(std::vector<int>{1, -2});
            s.execute(data, bad, in, gpu);
        } catch (const std::runtime_error&) {
            threw = true;
        }
        EXPECT(threw, "BlockSparseAttention with a negative block id did not throw");
    }
    {   // FusedBM25Retrieval: queries of at most two tokens (order-free sums)
        data_type::BM25IndexMemory mem;
        std::uniform_int_distribution<int> tok(0, 199), len(3, 40), tf(1, 4);
        for (int d = 0; d < 3000; ++d) {
            std::unordered_map<int, int> doc;
            for (int i = len(g); i > 0; --i) doc[tok(g) * 3 + 5] += tf(g);   // sparse token ids
            mem.insert_document(doc);
        }
        for (int t = 0; t < 20; ++t) {
            data_type::BM25QueryType qm;
            qm[tok(g) * 3 + 5] = 1;
            if (t % 2) qm[tok(g) * 3 + 5] = 2;
            if (t == 19) qm[-7] = 1;   // unknown token: ignored
            data_type::BM25Query q(qm);
            data_type::TopKIndex cpu, gpu;
            step::FusedBM25Retrieval s;
            s.execute(mem, q, cpu);
            s.set_kernel(KernelType::GPU);
            s.execute(mem, q, gpu);
            EXPECT(cpu.export_data() == gpu.export_data(), "FusedBM25Retrieval query %d differs", t);
        }
    }
    {   // device copies of unchanged memories are reused; every change is seen
        data_type::FlatIndexMemory<float> mem(matrix(g, 2000, 32));
        data_type::VectorQuery<float> q(vec(g, 32));
        auto agree = [&](data_type::FlatIndexMemory<float>& m, const char* what) {
            data_type::TopKIndex cpu, gpu;
            data_type::VectorScore<float> sc_cpu, sc_gpu;
            step::InnerProductTopKRetrieval s(20);
            s.execute(m, q, cpu);
            s.set_kernel(KernelType::GPU);
            s.execute(m, q, gpu);
            step::InnerProductCompute c;
            c.execute(m, q, sc_cpu);
            c.set_current_kernel(KernelType::GPU);
            c.execute(m, q, sc_gpu);
            EXPECT(cpu.export_data() == gpu.export_data(), "cached top-k after %s", what);
            EXPECT(sc_cpu.export_data() == sc_gpu.export_data(), "cached scores after %s", what);
        };
        agree(mem, "first use");
        agree(mem, "reuse");
        std::vector<float> big = vec(g, 32);
        for (auto& v : big) v *= 100.0f;   // a row that wins every query
        mem.insert_memory(big);
        agree(mem, "insert_memory");
        mem.delete_memory(0);
        agree(mem, "delete_memory");
        mem.pop_last_memory();
        agree(mem, "pop_last_memory");
        mem.set_data(matrix(g, 1500, 32));
        agree(mem, "set_data");
        data_type::FlatIndexMemory<float> copy = mem;
        copy.insert_memory(big);
        agree(copy, "a modified copy");
        agree(mem, "its unchanged original");
        // more memories in turn than the cache holds
        std::vector<data_type::FlatIndexMemory<float>> many;
        for (int i = 0; i < 6; ++i) many.emplace_back(matrix(g, 300 + i, 32));
        for (int r = 0; r < 2; ++r)
            for (auto& m : many) agree(m, "cycling memories");
    }
    {   // the cost the cache saves, at the flat-retrieval shape of config 1
        data_type::FlatIndexMemory<float> mem(matrix(g, 65536, 128));
        data_type::VectorQuery<float> q(vec(g, 128));
        step::InnerProductTopKRetrieval s(64);
        s.set_kernel(KernelType::GPU);
        data_type::TopKIndex out;
        auto ms = [&]() {
            const auto t0 = std::chrono::steady_clock::now();
            s.execute(mem, q, out);
            return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        };
        const double first = ms();
        double again = 0.0;
        for (int i = 0; i < 10; ++i) again += ms() / 10;
        std::printf("InnerProductTopKRetrieval GPU, 65536 x 128: first call %.3f ms, "
                    "unchanged memory %.3f ms per call\n", first, again);
    }
    std::printf("%s (%d failures)\n", failures ? "FAILED" : "PASSED", failures);
    return failures ? 1 : 0;
}
