// residency.cpp — make_resident / release / is_resident / h2d_bytes
// (include/heteromm/residency.h) over the per-thread device mirrors of
// device.h.
#include "device.h"
#include "heteromm/residency.h"

namespace heteromm {
namespace gpu {

namespace {
bool tagged_gpu(data_type::DataLocation loc) { return loc == data_type::DataLocation::GPU_MEM; }

void drop(uint64_t gen, int tag) {
    for (auto& x : mirror_table().m)
        if (x.gen == gen && x.tag == tag) {
            x.gen = 0;
            x.held = false;
        }
}
}  // namespace

void make_resident(const data_type::FlatIndexMemory<float>& memory) {
    const auto& rows = memory.data_ref();
    if (rows.empty() || rows[0].empty()) return;
    device_flat_rows(memory, rows[0].size(), "make_resident");
}

void make_resident(const data_type::KVCacheData<float>& kv) {
    const auto& c = kv.data_ref();
    const bool held = tagged_gpu(kv.get_device());
    if (!c.keys.empty() && !c.keys[0].empty())
        device_rows(c.keys, kv.generation(), kKeys, c.keys[0].size(), "make_resident keys", held);
    if (!c.values.empty() && !c.values[0].empty())
        device_rows(c.values, kv.generation(), kValues, c.values[0].size(),
                    "make_resident values", held);
}

void release(const data_type::FlatIndexMemory<float>& memory) {
    drop(memory.generation(), kRows);
}

void release(const data_type::KVCacheData<float>& kv) {
    drop(kv.generation(), kKeys);
    drop(kv.generation(), kValues);
}

bool is_resident(const data_type::FlatIndexMemory<float>& memory, size_t d) {
    const auto& rows = memory.data_ref();
    if (rows.empty()) return false;
    if (d == 0) d = rows[0].size();
    for (const auto& x : mirror_table().m)
        if (x.gen != 0 && x.gen == memory.generation() && x.tag == kRows && x.n == rows.size() &&
            x.d == d)
            return true;
    return false;
}

uint64_t h2d_bytes() { return h2d_counter(); }

}  // namespace gpu
}  // namespace heteromm
