#!/usr/bin/env bash
# Builds the reference's own CPU code for the hot path into oracle/_ref/.
#
# Test infrastructure only: the outputs are the checker that pins the oracle
# (tests/test_oracle_pins.py, tests/golden/make_golden.py) and the CPU arm of
# `bench.py --impl reference`.  Nothing in the product links them.
#
# Sources are compiled from the reference checkout.  Two one-line defects stop
# the reference's headers from compiling as shipped, so the headers are copied
# to a scratch directory under /tmp and patched there (the reference itself is
# read-only and nothing is copied into this repository):
#   1. steps/util.h:30  `KernelType string_to_kernel_type(...)` is a non-inline
#      function defined in a header -> duplicate symbol at link time; add
#      `inline`.
#   2. types/memory.h:240  BM25IndexMemory lacks the `content_type` alias that
#      the static_assert in steps/build_memory.h:46-49 requires; add it.
# The indexer references (DSA, LServe, SeerAttention) live inside HLS
# testbenches that need TAPA/ap_int headers which are not available; the
# reference functions themselves use only std:: containers and
# `ap_int<16>::to_int()`, so their exact line ranges are compiled together
# with a small stand-in for ap_int<16> and the reference's own constexpr
# constants.  The BM25 CPU kernel (bm25_fpga_retrieval.cpp:138-205) is
# compiled the same way as a free function, with its ambiguous
# `TopKIndex({})` spelled `TopKIndex(std::vector<int>{})`.
#
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]
#   (default: $HMM_REFERENCE_ROOT, else a directory named "reference" beside the
#   repository)
set -euo pipefail

HERE=$(cd "$(dirname "$0")" && pwd)
REF=${1:-${HMM_REFERENCE_ROOT:-$(cd "$HERE/../.." && pwd)/reference}}
OUT="$HERE/_ref"
DEV="$REF/toolchain/frontend/dev"
KER="$REF/kernels"

if [ ! -d "$DEV" ]; then
    echo "build_ref.sh: reference checkout not found at $REF" >&2
    exit 2
fi

SCRATCH=$(mktemp -d /tmp/hmm_ref_build.XXXXXX)
trap 'rm -rf "$SCRATCH"' EXIT
mkdir -p "$OUT" "$SCRATCH/dev"

cp -r "$DEV/types" "$DEV/steps" "$DEV/unittest" "$SCRATCH/dev/"

# patch 1: inline the header-defined function (steps/util.h:30)
sed -i 's/^KernelType string_to_kernel_type(/inline KernelType string_to_kernel_type(/' \
    "$SCRATCH/dev/steps/util.h"
grep -q '^inline KernelType string_to_kernel_type(' "$SCRATCH/dev/steps/util.h"
# patch 2: content_type alias for BM25IndexMemory (types/memory.h:240)
sed -i 's/^class BM25IndexMemory : public Memory<BM25IndexData> {$/&\npublic:\n    using content_type = BM25IndexData;/' \
    "$SCRATCH/dev/types/memory.h"
grep -q 'using content_type = BM25IndexData;' "$SCRATCH/dev/types/memory.h"

CXX=/usr/bin/g++

# ---- the reference's 5 doctest unit-test binaries (unittest/Makefile:3-39 flags)
for t in innerproduct:inner_product_compute topk_retrieval:topk_retrieval \
         threshold_retrieval:threshold_retrieval \
         paged_kv_index_builder:paged_kv_index_builder \
         block_sparse_attention:block_sparse_attention; do
    test=${t%%:*}; kern=${t##*:}
    (cd "$SCRATCH/dev/unittest" && $CXX -std=c++17 -Wall -Wextra -I.. -o "$OUT/test_$test" \
        "test_$test.cpp" "../steps/example_kernel/$kern.cpp" 2> "$SCRATCH/warn_$test.txt")
done

# ---- indexer reference functions, compiled from their exact line ranges
extract() {   # file first last -> stdout, checking the range opens the function
    local f=$1 a=$2 b=$3
    sed -n "${a}p" "$f" | grep -q "$4" || { echo "unexpected line $a in $f" >&2; exit 3; }
    sed -n "${a},${b}p" "$f"
}
# the reference's own constants, one namespace per indexer
{
    for ns in dsa_ref:dsa_indexer/indexer_vanilla.h lserve_ref:lserve/indexer_lserve.h \
              seer_budget_ref:seerattention/indexer_seer_token_budget.h \
              seer_threshold_ref:seerattention/indexer_seer_threshold.h; do
        echo "namespace ${ns%%:*} {"
        grep '^constexpr int' "$KER/${ns##*:}"
        echo "}"
    done
} > "$SCRATCH/dev/ref_consts.h"
HDR="#include \"$HERE/ref_ap_int.h\"
#include \"ref_consts.h\""
{
    echo "$HDR"; echo "namespace dsa_ref {"
    extract "$KER/dsa_indexer/indexer_tb.cpp" 17 57 '^void indexer_top_ref('
    echo "}"
} > "$SCRATCH/dsa_ref.cpp"
{
    echo "$HDR"; echo "namespace lserve_ref {"
    extract "$KER/lserve/indexer_lserve_tb.cpp" 20 92 '^void indexer_top_ref('
    echo "}"
} > "$SCRATCH/lserve_ref.cpp"
{
    echo "$HDR"; echo "namespace seer_budget_ref {"
    extract "$KER/seerattention/indexer_seer_token_budget_tb.cpp" 19 73 '^void indexer_top_ref('
    echo "}"
} > "$SCRATCH/seer_budget_ref.cpp"
{
    echo "$HDR"; echo "namespace seer_threshold_ref {"
    extract "$KER/seerattention/indexer_seer_threshold_tb.cpp" 18 77 '^void indexer_top_ref('
    echo "}"
} > "$SCRATCH/seer_threshold_ref.cpp"
{
    echo '#include "types/memory.h"'
    echo '#include "types/query.h"'
    echo '#include "types/retrieved_index.h"'
    echo '#include <algorithm>'
    echo '#include <cmath>'
    echo '#include <iostream>'
    echo '#include <numeric>'
    echo 'namespace heteromm { namespace step {'
    echo 'void bm25_ref_cpu_kernel(const data_type::BM25IndexMemory& memory,'
    echo '                         const data_type::BM25Query& query,'
    echo '                         data_type::TopKIndex& index) {'
    f="$DEV/steps/example_kernel/bm25_fpga_retrieval.cpp"
    sed -n '138p' "$f" | grep -q '^void FusedBM25Retrieval::run_cpu_kernel(' \
        || { echo "unexpected line 138 in $f" >&2; exit 3; }
    sed -n '143,205p' "$f" | sed 's/data_type::TopKIndex({})/data_type::TopKIndex(std::vector<int>{})/'
    echo '}}'
} > "$SCRATCH/bm25_ref.cpp"

# ---- shared library: reference step kernels + indexer refs + the C shim
KSRC="$SCRATCH/dev/steps/example_kernel"
$CXX -std=c++17 -O2 -fPIC -shared -pthread -I"$SCRATCH/dev" \
    -o "$OUT/libheteromm_ref.so" \
    "$KSRC/inner_product_compute.cpp" "$KSRC/topk_retrieval.cpp" \
    "$KSRC/threshold_retrieval.cpp" "$KSRC/paged_kv_index_builder.cpp" \
    "$KSRC/block_sparse_attention.cpp" \
    "$SCRATCH/dsa_ref.cpp" "$SCRATCH/lserve_ref.cpp" "$SCRATCH/seer_budget_ref.cpp" \
    "$SCRATCH/seer_threshold_ref.cpp" "$SCRATCH/bm25_ref.cpp" \
    "$HERE/ref_shim.cpp" 2> "$SCRATCH/warn_lib.txt" || {
    cat "$SCRATCH/warn_lib.txt" >&2; exit 4; }

echo "built: $(ls "$OUT")"
