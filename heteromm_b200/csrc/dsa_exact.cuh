// dsa_exact.cuh — what the FP8 DSA indexer's scoring pass (dsa.cu) and its
// exact selection (dsa_exact.cu) share: the device buffers of one call and the
// host steps of the selection, in call order.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "heteromm_cuda.h"

namespace hmm {

// Device buffers of one indexer call, carved from the caller's workspace.
struct DsaExactBufs {
    int* status;            // status words, then the flagged tokens
    float* norms;           // [L] ||k_j||_2 rounded up (real units)
    uint8_t* skeys;         // [S][128] the sampled keys
    float* sscores;         // [T][S] approximate scores of the sampled keys
    float* tok_e;           // [T] E_t = C_TOL * ||u_t||_2 rounded up
    float* tok_tau;         // [T] the token's threshold (-inf: every visible key)
    uint32_t* bitmap;       // [T][W] keys with s~ + E_t ||k_j|| >= tau (bit j of word j / 32)
    int S;                  // sampled keys (0: every token takes all its visible keys)
    int W;                  // bitmap words per token: ceil(L / 32)
};

size_t dsa_exact_ws_bytes(int64_t T, int64_t L);

// Clears the status words and the counters, computes the key norms and checks
// the keys for NaN encodings, and gathers the sampled keys.
hmm_status_t dsa_exact_prepare(const uint8_t* keys, int64_t T, int64_t L, int64_t topk,
                               void* ws, cudaStream_t st, DsaExactBufs* b);

// Per token: E_t and the threshold tau from the sampled keys' scores.
hmm_status_t dsa_exact_thresholds(const uint8_t* q, const float* w, int64_t T, int64_t H,
                                  int64_t L, int64_t pos0, int64_t topk, const DsaExactBufs& b,
                                  cudaStream_t st);

// Candidates from the bitmap, their exact scores, the exact top-k; then the
// host reads the status words and recomputes flagged tokens from exact rows.
hmm_status_t dsa_exact_select(const uint8_t* q, const uint8_t* keys, const float* w, int64_t T,
                              int64_t H, int64_t L, int64_t pos0, int64_t topk,
                              const DsaExactBufs& b, int32_t* out_idx, float* out_sc, void* ws,
                              cudaStream_t st);

}  // namespace hmm
