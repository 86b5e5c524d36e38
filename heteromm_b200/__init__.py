"""heteromm_b200 — B200-native (sm_100a) kernels for the HeteroMM
score -> select -> apply path, behind the C ABI in include/heteromm_cuda.h.

Python is plumbing here (device memory, streams, torch.distributed); every
operation runs in libheteromm_cuda.so.
"""
from ._abi import HmmError, last_error, load, lib_path  # noqa: F401
from .flat import (ip_score_f32, ip_topk_bf16, ip_topk_f32, shard_merge_topk,  # noqa: F401
                   threshold_bitmap_f32, topk_f32)
from .bm25 import BM25Index  # noqa: F401
from .indexers import (dsa_indexer_fp8, dsa_indexer_fp8_host, lserve_topk_i16,  # noqa: F401
                       seer_budget_i16, seer_threshold_i16)
from .paged import (block_pages, block_sparse_attention_bf16, block_sparse_attention_f32,  # noqa: F401,E501
                    block_select_minmax, block_sparse_decode_bf16, paged_kv_minmax_bf16,
                    paged_kv_summary_bf16, paged_kv_summary_f32)

__version__ = "0.1.0"
