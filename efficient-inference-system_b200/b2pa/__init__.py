"""b2pa -- B200-native paged-attention backend.

Drop-in replacement for the GPU attention backend of
jacobzhang22/efficient-inference-system: the paged decode and chunked-prefill
attention kernels (src/kernels/triton_paged_attention.py) and the KV
append/scatter into the per-layer block pools (src/cache/paged_kv.py), backed
by hand-written sm_100a CUDA kernels in libb2pa.so behind a C ABI
(include/b2pa.h).
"""
from ._lib import clear_status, load as load_library, read_status, raise_on_device_status
from .attention import (
    SUPPORTED_BACKENDS,
    paged_attention,
    paged_attention_decode_b200,
    paged_attention_prefill_b200,
)
from .integration import install_into_reference
from .decoder import FusedDecodeExecutor, FusedDecoder
from .step import DecodeGraph, DecodeStep, SharedStepMetadata
from .serving import ContinuousBatchingRank, LeastOutstandingTokensRouter, ServeResult, gather_request_times, serve
from .paged_kv import (
    BatchedPagedKVCache,
    LayerBlockPool,
    PagedKVCacheState,
    device_metadata,
    flush_pending,
    set_fused_append,
)

__all__ = [
    "BatchedPagedKVCache",
    "ContinuousBatchingRank",
    "DecodeGraph",
    "DecodeStep",
    "FusedDecodeExecutor",
    "FusedDecoder",
    "SharedStepMetadata",
    "LeastOutstandingTokensRouter",
    "ServeResult",
    "gather_request_times",
    "serve",
    "LayerBlockPool",
    "PagedKVCacheState",
    "SUPPORTED_BACKENDS",
    "clear_status",
    "device_metadata",
    "flush_pending",
    "install_into_reference",
    "load_library",
    "paged_attention",
    "paged_attention_decode_b200",
    "paged_attention_prefill_b200",
    "raise_on_device_status",
    "read_status",
    "set_fused_append",
]
