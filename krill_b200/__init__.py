"""krill_b200 — B200-native int8 KV-cache hot path for Krill.

The product is libkrill_kv.so (C ABI: include/krill_kv.h, sm_100a kernels +
C++ host logic). This package is the Python mirror of the reference's cache
API on top of that ABI.
"""
from ._lib import (ATTN_CUDA_CORE, ATTN_TENSOR_CORE, ATTN_TENSOR_CORE_PAIR, ATTN_TENSOR_CORE_SYNC, KV_BF16, KV_INT8, DTYPE_BF16, DTYPE_F16, DTYPE_F32,
                   QUANT_F32, QUANT_INPUT_DTYPE, KrillError, lib)
from .cache import (KVPool, PrefixCache, QuantizedKVCache, QuantizedKVSnapshot,
                    QuantizedPrefixCacheHit, Sequence_, append_quantize,
                    build_batched_decode_mask, decode_attention, decode_step, decode_step_host,
                    make_quantized_kv_caches, prefix_key, scatter_back,
                    stack_caches_left_padded_quantized, verify_attention,
                    prefill_attention)

__all__ = [
    "KVPool", "Sequence_", "QuantizedKVCache", "QuantizedKVSnapshot", "PrefixCache",
    "QuantizedPrefixCacheHit", "make_quantized_kv_caches", "append_quantize", "decode_attention",
    "decode_step", "decode_step_host", "stack_caches_left_padded_quantized", "scatter_back", "build_batched_decode_mask",
    "prefix_key", "KrillError", "lib", "DTYPE_F16", "DTYPE_BF16", "DTYPE_F32", "QUANT_F32",
    "QUANT_INPUT_DTYPE", "ATTN_TENSOR_CORE", "ATTN_CUDA_CORE", "ATTN_TENSOR_CORE_SYNC", "ATTN_TENSOR_CORE_PAIR", "KV_INT8", "KV_BF16", "verify_attention", "prefill_attention",
]
