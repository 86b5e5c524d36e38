// test_deploy.cpp — the deploy layer (include/heteromm/deploy) against the
// step API it orchestrates.
//
// Without arguments (CPU only): the JSON reader, ScheduleConfig rule matching
// on a schedule shaped like the reference's deploy/schedule.json, the
// PagedAttention pipeline on CPU kernels (equal to the four steps composed by
// hand), run_functional_tests, FPGA-scheduled steps (the reference's stubs:
// outputs left empty), missing steps, and the projection-weight generator
// pinned to values computed independently in float32.
//
// With --gpu: the same pipeline scheduled on the GPU.  build_memory equals the
// CPU build bit for bit; the device-resident manage_memory_and_apply equals the
// step-by-step GPU route bit for bit and the CPU pipeline within the attention
// tolerance (rtol 2e-5, atol 2e-6); after the first call only the two query
// vectors cross to the device; a changed KV cache is re-read; a subclassed step
// turns the device pass off; per-call times of the three routes are printed.
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "heteromm/deploy/device_chain.h"
#include "heteromm/deploy/paged_attention.h"

using namespace heteromm;
using deploy::ExecutionResult;
using deploy::PagedAttention;
using deploy::ScheduleConfig;
using Rows = std::vector<std::vector<float>>;

static int g_fail = 0;
#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);         \
            ++g_fail;                                                            \
        }                                                                        \
    } while (0)

template <typename F>
static bool throws(F&& f) {
    try {
        f();
    } catch (const std::exception&) {
        return true;
    }
    return false;
}

static Rows random_rows(size_t n, size_t d, uint32_t seed) {
    std::mt19937 gen(seed);
    std::normal_distribution<float> nd(0.0f, 1.0f);
    Rows r(n, std::vector<float>(d));
    for (auto& row : r)
        for (auto& x : row) x = nd(gen);
    return r;
}

static std::vector<float> random_vec(size_t d, uint32_t seed) { return random_rows(1, d, seed)[0]; }

static bool close(const std::vector<float>& a, const std::vector<float>& b, float rtol, float atol) {
    if (a.size() != b.size()) return false;
    for (size_t i = 0; i < a.size(); ++i)
        if (!(std::fabs(a[i] - b[i]) <= atol + rtol * std::fabs(b[i]))) return false;
    return true;
}

static uint32_t bits(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    return u;
}

// A schedule in the reference's format: small contexts on the FPGA, the rest
// on the GPU.
static const char* kMixedSchedule = R"({
  "build_memory": [ {"retrieved_data": 4096, "config": "fpga"},
                    {"retrieved_data": -1, "config": "gpu"} ],
  "manage_memory_and_apply": [
    {"retrieved_data": 4096, "memory": 4096, "query": 1, "output": 1,
     "config": ["fpga", "fpga", "gpu"]},
    {"retrieved_data": -1, "memory": -1, "query": 1, "output": 1,
     "config": ["gpu", "gpu", "gpu"]} ],
  "build_and_apply_memory": [
    {"retrieved_data": 4096, "query": 1, "output": 1, "config": ["gpu", "fpga", "fpga", "gpu"]},
    {"retrieved_data": -1, "query": 1, "output": 1, "config": ["gpu", "gpu", "gpu", "gpu"]} ]
})";

static ScheduleConfig all_on(const std::string& k) {
    const std::string q = "\"" + k + "\"";
    return ScheduleConfig::load_from_string(
        "{\"build_memory\": [{\"retrieved_data\": -1, \"config\": " + q + "}],"
        " \"manage_memory_and_apply\": [{\"retrieved_data\": -1, \"memory\": -1, \"query\": 1,"
        " \"output\": 1, \"config\": [" + q + "," + q + "," + q + "]}],"
        " \"build_and_apply_memory\": [{\"retrieved_data\": -1, \"query\": 1, \"output\": 1,"
        " \"config\": [" + q + "," + q + "," + q + "," + q + "]}]}");
}

// The four steps composed by hand on one kernel type.
static std::vector<float> by_hand(const data_type::KVCacheData<float>& kv, const Rows& w,
                                  size_t page, size_t k, const std::vector<float>& qv,
                                  const std::vector<float>& in, step::KernelType kt,
                                  data_type::FlatIndexMemory<float>* built = nullptr) {
    step::PagedKVIndexBuilder b(w, (int)page);
    step::InnerProductCompute s;
    step::TopKRetrieval r(k);
    step::BlockSparseAttention a(page);
    b.set_current_kernel(kt);
    s.set_current_kernel(kt);
    r.set_current_kernel(kt);
    a.set_current_kernel(kt);
    data_type::FlatIndexMemory<float> mem;
    b.execute(kv, mem);
    data_type::VectorScore<float> sc;
    s.execute(mem, data_type::VectorQuery<float>(qv), sc);
    data_type::TopKIndex idx;
    r.execute(sc, idx);
    data_type::VectorInputOutputData<float> out;
    a.execute(kv, idx, data_type::VectorInputOutputData<float>(in), out);
    if (built) *built = mem;
    return out.export_data();
}

static void test_json() {
    using deploy::json;
    const json j = json::parse(
        " {\"a\": [1, -2, 3.5e2, true, false, null, \"x\\u00e9\\n\\\"\"], \"b\": {\"c\": 0},"
        " \"a2\": [], \"b\": {\"c\": 7}} ");
    CHECK(j.is_object());
    CHECK(j["a"].size() == 7);
    CHECK(j["a"][0].get<int>() == 1);
    CHECK(j["a"][1].get<int>() == -2);
    CHECK(j["a"][2].get<double>() == 350.0);
    CHECK(j["a"][3].get<bool>() && !j["a"][4].get<bool>());
    CHECK(j["a"][5].is_null());
    CHECK(j["a"][6].get<std::string>() == "x\xc3\xa9\n\"");
    CHECK(j["b"]["c"].get<int>() == 7);   // the later duplicate wins
    CHECK(j["a2"].size() == 0 && j.contains("a2") && !j.contains("zz"));
    CHECK(json::parse("\"\\ud83d\\ude00\"").get<std::string>() == "\xf0\x9f\x98\x80");
    CHECK(throws([&] { j["a"][2].get<int>(); }));      // 350.0 is not an integer literal
    CHECK(throws([&] { j["zz"]; }));
    CHECK(throws([&] { json::parse("3000000000").get<int>(); }));
    for (const char* bad : {"", "{", "[1,]", "{\"a\" 1}", "{\"a\":1,}", "tru", "01", "1.", "-",
                            "\"abc", "\"\\q\"", "\"\\ud800\"", "\"\\udc00\"", "\"a\x01\"", "{} x",
                            "[1 2]", "{1: 2}"})
        CHECK(throws([&] { json::parse(bad); }));
    CHECK(throws([&] { json::parse(std::string(300, '[') + std::string(300, ']')); }));
    CHECK(!throws([&] { json::parse(std::string(200, '[') + std::string(200, ']')); }));
}

static void test_schedule() {
    const ScheduleConfig s = ScheduleConfig::load_from_string(kMixedSchedule);
    CHECK(s.build_memory_rules.size() == 2);
    CHECK(s.get_build_memory_config(4096) == "fpga");
    CHECK(s.get_build_memory_config(4097) == "gpu");
    CHECK((s.get_manage_memory_and_apply_config(100, 100) ==
           std::vector<std::string>{"fpga", "fpga", "gpu"}));
    CHECK((s.get_manage_memory_and_apply_config(100, 5000) ==
           std::vector<std::string>{"gpu", "gpu", "gpu"}));   // memory over the first bound
    CHECK((s.get_manage_memory_and_apply_config(5000, 100) ==
           std::vector<std::string>{"gpu", "gpu", "gpu"}));
    CHECK((s.get_build_and_apply_memory_config(10) ==
           std::vector<std::string>{"gpu", "fpga", "fpga", "gpu"}));
    const ScheduleConfig bounded = ScheduleConfig::load_from_string(
        "{\"build_memory\": [{\"retrieved_data\": 10, \"config\": \"cpu\"}]}");
    CHECK(throws([&] { bounded.get_build_memory_config(11); }));   // no rule matches
    CHECK(throws([&] { bounded.get_manage_memory_and_apply_config(1, 1); }));
    CHECK(throws([&] {   // a rule without its sizes
        ScheduleConfig::load_from_string("{\"build_memory\": [{\"config\": \"gpu\"}]}");
    }));
    CHECK(throws([&] {   // two kernels for three steps
        ScheduleConfig::load_from_string(
            "{\"manage_memory_and_apply\": [{\"retrieved_data\": -1, \"memory\": -1, \"query\": 1,"
            " \"output\": 1, \"config\": [\"gpu\", \"gpu\"]}]}");
    }));
    CHECK(throws([&] { ScheduleConfig::load_from_file("/nonexistent/schedule.json"); }));
    CHECK(throws([&] { PagedAttention p("/nonexistent/schedule.json"); }));
}

static void test_projection_weight() {
    const Rows w = deploy::create_random_projection_weight(64, 32, 7);
    CHECK(w.size() == 32 && w[0].size() == 64);
    // float32 values of the same generator computed independently
    CHECK(bits(w[0][0]) == 1013287476u);
    CHECK(bits(w[0][1]) == 3169671731u);
    CHECK(bits(w[0][63]) == 1018269445u);
    CHECK(bits(w[1][0]) == 1013476662u);
    CHECK(bits(w[31][63]) == 3172961025u);
    CHECK(deploy::create_random_projection_weight(64, 32, 7) == w);
    CHECK(deploy::create_random_projection_weight(64, 32, 8) != w);
}

// A manager that provides no steps.
class Bare : public deploy::MemoryManager<data_type::KVCacheData<float>, data_type::FlatIndexMemory<float>,
                                          data_type::VectorQuery<float>, data_type::VectorScore<float>,
                                          data_type::TopKIndex,
                                          data_type::VectorInputOutputData<float>,
                                          data_type::VectorInputOutputData<float>> {
public:
    int ret_data_size(const data_type::KVCacheData<float>& d) override {
        return (int)d.get_context_length();
    }
    int memory_size(const data_type::FlatIndexMemory<float>& m) override {
        return (int)m.get_num_entries();
    }
};

static void test_cpu_pipeline() {
    const size_t L = 1000, D = 64, page = 16, k = 8;
    data_type::KVCacheData<float> kv(data_type::KVCache<float>{random_rows(L, D, 1), random_rows(L, D, 2)});
    const Rows w = deploy::create_random_projection_weight(D, 32, 3);
    const std::vector<float> qv = random_vec(32, 4), in = random_vec(D, 5);
    data_type::FlatIndexMemory<float> want_mem;
    const std::vector<float> want = by_hand(kv, w, page, k, qv, in, step::KernelType::CPU, &want_mem);

    auto pa = deploy::create_paged_attention().with_projection_weight(w).with_page_size(page).with_top_k(k).build();
    data_type::FlatIndexMemory<float> mem;
    ExecutionResult r = pa->build_memory(kv, mem);   // no schedule: the configured CPU kernels
    CHECK(r.success && r.build_memory_time_ms >= 0.0);
    CHECK(mem.is_equal(want_mem));
    CHECK(mem.get_num_entries() == (L + page - 1) / page);   // set_data keeps the count
    CHECK(pa->memory_size(mem) == 63 && pa->ret_data_size(kv) == 1000);

    data_type::VectorInputOutputData<float> out;
    r = pa->manage_memory_and_apply(kv, mem, data_type::VectorQuery<float>(qv),
                                    data_type::VectorInputOutputData<float>(in), out);
    CHECK(r.success);
    CHECK(out.export_data() == want);
    CHECK(r.total_time_ms == r.compute_score_time_ms + r.retrieval_time_ms + r.apply_memory_time_ms);

    data_type::VectorInputOutputData<float> out2;
    r = pa->build_and_apply_memory(kv, data_type::VectorQuery<float>(qv),
                                   data_type::VectorInputOutputData<float>(in), out2);
    CHECK(r.success && out2.export_data() == want);

    // functional tests: expected outputs from the CPU arms pass, a changed one fails
    data_type::VectorScore<float> sc;
    step::InnerProductCompute().execute(want_mem, data_type::VectorQuery<float>(qv), sc);
    data_type::TopKIndex idx;
    step::TopKRetrieval(k).execute(sc, idx);
    data_type::VectorInputOutputData<float> want_out(want);
    data_type::FlatIndexMemory<float> m2 = want_mem;
    CHECK(pa->run_functional_tests(kv, m2, data_type::VectorQuery<float>(qv), sc, idx,
                                   data_type::VectorInputOutputData<float>(in), want_out));
    std::vector<float> bad = want;
    bad[0] += 1.0f;
    data_type::VectorInputOutputData<float> bad_out(bad);
    CHECK(!pa->run_functional_tests(kv, m2, data_type::VectorQuery<float>(qv), sc, idx,
                                    data_type::VectorInputOutputData<float>(in), bad_out));

    // setters rebuild the steps they affect
    pa->set_top_k(3);
    pa->manage_memory_and_apply(kv, mem, data_type::VectorQuery<float>(qv),
                                data_type::VectorInputOutputData<float>(in), out);
    CHECK(out.export_data() == by_hand(kv, w, page, 3, qv, in, step::KernelType::CPU));

    // an explicit CPU schedule gives the same
    pa->set_top_k(k);
    pa->set_schedule_config(all_on("cpu"));
    pa->manage_memory_and_apply(kv, mem, data_type::VectorQuery<float>(qv),
                                data_type::VectorInputOutputData<float>(in), out);
    CHECK(out.export_data() == want);

    // FPGA-scheduled steps are stubs: a small context builds no memory and
    // selects no block, so the GPU attention returns zeros
    pa->set_schedule_config(ScheduleConfig::load_from_string(kMixedSchedule));
    data_type::FlatIndexMemory<float> fmem;
    CHECK(pa->build_memory(kv, fmem).success);
    CHECK(fmem.get_num_entries() == 0 && pa->get_kernel_config().build_memory == step::KernelType::FPGA);
    pa->manage_memory_and_apply(kv, mem, data_type::VectorQuery<float>(qv),
                                data_type::VectorInputOutputData<float>(in), out);
    CHECK(pa->get_kernel_config().compute_score == step::KernelType::FPGA);
    CHECK(pa->get_kernel_config().apply_memory == step::KernelType::GPU);
    CHECK(out.export_data() == std::vector<float>(D, 0.0f));

    // a manager without steps fails by status, as the reference's does
    Bare bare;
    data_type::FlatIndexMemory<float> bm;
    r = bare.build_memory(kv, bm);
    CHECK(!r.success && r.error_message == "BuildMemory step not configured");
    r = bare.manage_memory_and_apply(kv, mem, data_type::VectorQuery<float>(qv),
                                     data_type::VectorInputOutputData<float>(in), out);
    CHECK(!r.success && r.error_message == "ComputeScore step not configured");
}

// An attention step whose GPU arm is its own: the device pass must not bypass it.
class CountingAttention : public step::BlockSparseAttention {
public:
    explicit CountingAttention(size_t page) : step::BlockSparseAttention(page) {}
    int gpu_calls = 0;

protected:
    void run_gpu_kernel(const data_type::KVCacheData<float>& kv, const data_type::TopKIndex& idx,
                        const data_type::VectorInputOutputData<float>& in,
                        data_type::VectorInputOutputData<float>& out) override {
        ++gpu_calls;
        step::BlockSparseAttention::run_gpu_kernel(kv, idx, in, out);
    }
};

template <typename F>
static double ms_per_call(int reps, F&& f) {
    f();
    const auto t0 = std::chrono::high_resolution_clock::now();
    for (int i = 0; i < reps; ++i) f();
    return std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t0)
               .count() / reps;
}

static void test_gpu_pipeline() {
    // one (batch, head) of the paged decode workload: 32,768 tokens x 128, 64-token
    // summaries (identity projection), top-64 of 512 blocks
    const size_t L = 32768, D = 128, page = 64, k = 64;
    data_type::KVCacheData<float> kv(data_type::KVCache<float>{random_rows(L, D, 11), random_rows(L, D, 12)});
    Rows eye(D, std::vector<float>(D, 0.0f));
    for (size_t i = 0; i < D; ++i) eye[i][i] = 1.0f;
    const std::vector<float> qv = random_vec(D, 13), in = random_vec(D, 14);
    data_type::FlatIndexMemory<float> cpu_mem;
    const std::vector<float> want = by_hand(kv, eye, page, k, qv, in, step::KernelType::CPU, &cpu_mem);

    PagedAttention pa("", eye, page, k);
    pa.set_schedule_config(all_on("gpu"));
    data_type::FlatIndexMemory<float> mem;
    CHECK(pa.build_memory(kv, mem).success);
    CHECK(pa.get_kernel_config().build_memory == step::KernelType::GPU);
    CHECK(mem.is_equal(cpu_mem));   // bit-exact summaries

    const data_type::VectorQuery<float> q(qv);
    const data_type::VectorInputOutputData<float> input(in);
    data_type::VectorInputOutputData<float> chain_out, step_out;
    uint64_t b0 = gpu::h2d_bytes();
    ExecutionResult r = pa.manage_memory_and_apply(kv, mem, q, input, chain_out);
    CHECK(r.success && r.retrieval_time_ms == 0.0 && r.apply_memory_time_ms > 0.0);
    const uint64_t first = gpu::h2d_bytes() - b0;   // values (the keys and summaries are resident)
    b0 = gpu::h2d_bytes();
    pa.manage_memory_and_apply(kv, mem, q, input, chain_out);
    const uint64_t second = gpu::h2d_bytes() - b0;
    std::printf("h2d bytes: first call %llu, next call %llu\n", (unsigned long long)first,
                (unsigned long long)second);
    CHECK(first == (L * D + 2 * D) * sizeof(float));
    CHECK(second == 2 * D * sizeof(float));
    CHECK(close(chain_out.export_data(), want, 2e-5f, 2e-6f));

    pa.set_device_chain(false);
    pa.manage_memory_and_apply(kv, mem, q, input, step_out);
    CHECK(step_out.export_data() == chain_out.export_data());   // same kernels, same inputs
    CHECK(by_hand(kv, eye, page, k, qv, in, step::KernelType::GPU) == chain_out.export_data());
    pa.set_device_chain(true);

    // build_and_apply_memory on the GPU, and the degenerate selections
    data_type::VectorInputOutputData<float> ba;
    CHECK(pa.build_and_apply_memory(kv, q, input, ba).success);
    CHECK(ba.export_data() == chain_out.export_data());
    pa.set_top_k(0);
    pa.manage_memory_and_apply(kv, mem, q, input, ba);
    CHECK(ba.export_data() == std::vector<float>(D, 0.0f));
    pa.set_top_k(k);
    data_type::FlatIndexMemory<float> empty;
    pa.manage_memory_and_apply(kv, empty, q, input, ba);
    CHECK(ba.export_data() == std::vector<float>(D, 0.0f));

    // a changed KV cache is read again
    data_type::KVCacheData<float> kv2 = kv;
    data_type::KVCache<float> c = kv2.export_data();
    for (auto& row : c.values) row[5] += 3.0f;
    kv2.set_data(c);
    data_type::VectorInputOutputData<float> o2;
    pa.manage_memory_and_apply(kv2, mem, q, input, o2);
    const std::vector<float> want2 = by_hand(kv2, eye, page, k, qv, in, step::KernelType::CPU);
    CHECK(close(o2.export_data(), want2, 2e-5f, 2e-6f));
    CHECK(o2.export_data()[5] != chain_out.export_data()[5]);

    // mismatched keys and values are reported on both routes
    data_type::KVCacheData<float> ragged(data_type::KVCache<float>{random_rows(256, D, 15), random_rows(200, D, 16)});
    data_type::FlatIndexMemory<float> rmem;
    pa.build_memory(ragged, rmem);
    CHECK(throws([&] { pa.manage_memory_and_apply(ragged, rmem, q, input, ba); }));
    pa.set_device_chain(false);
    CHECK(throws([&] { pa.manage_memory_and_apply(ragged, rmem, q, input, ba); }));
    pa.set_device_chain(true);

    // a subclassed step keeps the step-by-step route
    auto counting = std::make_shared<CountingAttention>(page);
    pa.set_apply_memory_step(counting);
    pa.manage_memory_and_apply(kv, mem, q, input, ba);
    CHECK(counting->gpu_calls == 1 && ba.export_data() == chain_out.export_data());
    pa.set_page_size(page);   // back to the stock step

    // per-call host time of the three routes
    PagedAttention cpu("", eye, page, k);
    cpu.set_schedule_config(all_on("cpu"));
    data_type::VectorInputOutputData<float> o;
    const double t_cpu = ms_per_call(3, [&] { cpu.manage_memory_and_apply(kv, mem, q, input, o); });
    pa.set_device_chain(false);
    const double t_steps = ms_per_call(20, [&] { pa.manage_memory_and_apply(kv, mem, q, input, o); });
    pa.set_device_chain(true);
    const double t_chain = ms_per_call(200, [&] { pa.manage_memory_and_apply(kv, mem, q, input, o); });
    std::printf("manage_memory_and_apply per call (L=%zu, D=%zu, %zu blocks, top-%zu): "
                "cpu %.3f ms, gpu steps %.3f ms, gpu device pass %.4f ms\n",
                L, D, (L + page - 1) / page, k, t_cpu, t_steps, t_chain);
}

int main(int argc, char** argv) {
    const bool gpu = argc > 1 && std::strcmp(argv[1], "--gpu") == 0;
    try {
        test_json();
        test_schedule();
        test_projection_weight();
        test_cpu_pipeline();
        if (gpu) test_gpu_pipeline();
    } catch (const std::exception& e) {
        std::printf("FAIL: uncaught exception: %s\n", e.what());
        ++g_fail;
    }
    std::printf("%s: %d failure(s)\n", g_fail ? "FAILED" : "PASSED", g_fail);
    return g_fail ? 1 : 0;
}
