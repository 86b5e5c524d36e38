// Stand-in for the one piece of Xilinx ap_int<16> the reference indexer
// functions use: construction from an integer and to_int().  Test
// infrastructure for oracle/build_ref.sh only.
#ifndef HMM_REF_AP_INT_H_
#define HMM_REF_AP_INT_H_
#include <algorithm>
#include <cstdint>
#include <utility>
#include <vector>

template <int W>
struct ap_int {
    int64_t v = 0;
    ap_int() = default;
    ap_int(int64_t x) : v(x) {}
    int64_t to_int() const { return v; }
};
#endif
