// device_chain.h — device-resident passes of the deploy layer (B200 build),
// exported by libheteromm_steps.so.
//
// paged_attention_chain runs the PagedAttention pipeline's InnerProductCompute
// -> TopKRetrieval -> BlockSparseAttention (reference deploy/paged_attention.h:
// 146-175) with scores and block ids kept on the device: one fused score +
// top-k launch (hmm_ip_topk_f32) writes the block ids where the attention
// (hmm_block_sparse_attention_f32) reads them.  The page summaries and the KV
// cache come from this thread's device mirrors, keyed by the objects'
// generations, so an unchanged memory or KV cache is uploaded once; the
// summaries a GPU PagedKVIndexBuilder produced are already mirrored.  Per call
// only the two query vectors go up and the output comes back.
//
// Results are those of the three steps' GPU arms run one after another: the
// same block ids (bit-exact with the CPU arms) and the same attention output.
#ifndef HETEROMM_B200_DEPLOY_DEVICE_CHAIN_H_
#define HETEROMM_B200_DEPLOY_DEVICE_CHAIN_H_

#include <cstddef>
#include <cstdint>
#include <vector>

#include "../dev/types/memory.h"
#include "../dev/types/retrieved_data.h"
#include "../residency.h"

namespace heteromm {
namespace gpu {

// Device times of one chain call, from CUDA events on the launching stream.
struct ChainTimes {
    double score_topk_ms = 0.0;   // query upload + fused score / top-k
    double apply_ms = 0.0;        // KV mirror check, attention, output download
};

// The attention output [input.size()] of `input` over the tokens of the
// min(k, memory rows) blocks of `page_size` tokens whose summaries score
// highest against `query` (best first, ties to the lower block).  Zeros when no
// block is selected, the KV cache is empty or page_size is 0.  Throws
// std::invalid_argument when memory rows are shorter than the query, KV rows
// shorter than the input, or keys and values differ in length;
// std::runtime_error with the library's message when a kernel fails.
std::vector<float> paged_attention_chain(const data_type::KVCacheData<float>& kv,
                                         const data_type::FlatIndexMemory<float>& memory,
                                         const std::vector<float>& query, size_t k,
                                         const std::vector<float>& input, size_t page_size,
                                         ChainTimes* times = nullptr);

}  // namespace gpu
}  // namespace heteromm

#endif  // HETEROMM_B200_DEPLOY_DEVICE_CHAIN_H_
