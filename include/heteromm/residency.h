// residency.h — device residency of the step API's data (B200 build),
// exported by libheteromm_steps.so.
//
// The reference's data types carry a DataLocation tag (types/base_types.h:26-30,
// 57-59: SYS_DRAM, GPU_MEM, FPGA_MEM) that nothing acts on.  Here the GPU arms
// of the steps keep device copies ("mirrors") of the rows they read, per
// thread and GPU, keyed by each object's generation, and act on the tag:
//   - a copy of an object tagged GPU_MEM is held: it is replaced only after
//     every copy that is not;
//   - make_resident() takes the copy now, so the first GPU step on the object
//     does no upload; release() drops it;
//   - after insert_memory / pop_last_memory / delete_memory on a
//     FlatIndexMemory, the next GPU step brings the old copy up to date on the
//     device (appended rows copied up, erased rows closed up) from the
//     memory's row log instead of uploading the memory again.
// Full uploads pack the rows into pinned chunks, overlapped with the copies.
// All of it is per calling thread and current GPU, as the adapters' scratch is.
#ifndef HETEROMM_B200_RESIDENCY_H_
#define HETEROMM_B200_RESIDENCY_H_

#include <cstddef>
#include <cstdint>

#include "dev/types/memory.h"
#include "dev/types/retrieved_data.h"

namespace heteromm {
namespace gpu {

// Copies the memory's rows (all columns) to this thread's device mirrors now,
// unless a copy of its current contents is there already; the copy is held
// when the memory is tagged DataLocation::GPU_MEM.
void make_resident(const data_type::FlatIndexMemory<float>& memory);
// The same for a KV cache's keys and values.
void make_resident(const data_type::KVCacheData<float>& kv);

// Drops this thread's device copies of the object's current contents.
void release(const data_type::FlatIndexMemory<float>& memory);
void release(const data_type::KVCacheData<float>& kv);

// Whether this thread holds a device copy of the memory's current rows: the
// first d columns (d = 0: all of them).
bool is_resident(const data_type::FlatIndexMemory<float>& memory, size_t d = 0);

// Bytes the calling thread has copied host -> device through the step
// adapters, the deploy layer and these calls so far (a monotone counter).
uint64_t h2d_bytes();

}  // namespace gpu
}  // namespace heteromm

#endif  // HETEROMM_B200_RESIDENCY_H_
