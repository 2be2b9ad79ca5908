"""B200-native Q4 KV-cache attention for agent-memory.

Hot path (sm_100a CUDA kernels in ``libamq4.so``, C ABI in ``include/am_q4.h``):
quantize-on-append into 4-bit affine blocks, split-KV decode attention over contiguous
or paged Q4 caches, and tcgen05 chunked prefill.  The Python layer mirrors the reference's
quantized-attention op and Q4 cache classes; PyTorch only carries device memory.
"""

from ._lib import Q4KernelError, Q4KernelUnavailable
from .attention import (apply_fused_attention_patch, quantized_scaled_dot_product_attention,
                        scaled_dot_product_attention)
from .block_pool import (AgentBlocks, BlockPool, KVBlock, ModelCacheSpec, PoolExhaustedError,
                         BLOCK_SIZE_TOKENS)
from .cache import BatchQuantizedKVCache, QuantizedKVCache, validate_q4_pipeline
from .kernels import dequantize, quantize
from .masks import CausalMask, create_causal_mask
from .paged import PagedLayerCache, PagedQ4Pool, lpt_partition, shuffled_allocator
from .paged_cache import (DeviceBlockPool, PagedBatchQuantizedKVCache, PagedKV, PagedMask,
                          extract_agent_blocks, reconstruct_cache, slice_cache_to_length)

__all__ = [
    "AgentBlocks", "BLOCK_SIZE_TOKENS", "BatchQuantizedKVCache", "BlockPool", "CausalMask",
    "DeviceBlockPool", "KVBlock", "ModelCacheSpec", "PagedBatchQuantizedKVCache", "PagedKV",
    "PagedLayerCache", "PagedMask", "PagedQ4Pool", "PoolExhaustedError",
    "Q4KernelError", "Q4KernelUnavailable", "QuantizedKVCache", "apply_fused_attention_patch",
    "create_causal_mask", "dequantize", "extract_agent_blocks", "lpt_partition", "quantize",
    "reconstruct_cache", "slice_cache_to_length",
    "quantized_scaled_dot_product_attention", "scaled_dot_product_attention",
    "shuffled_allocator", "validate_q4_pipeline",
]
