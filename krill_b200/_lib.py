"""ctypes binding of libkrill_kv.so (the C ABI in include/krill_kv.h).

The library is the product: every compute call goes to its sm_100a kernels.
There is no fallback — if the shared object is missing this module raises at
import time.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkrill_kv.so")

KRILL_OK = 0
KRILL_ERR_INVALID = 1
KRILL_ERR_OOM = 2
KRILL_ERR_CUDA = 3
KRILL_ERR_PEER = 4
KRILL_ERR_TIMEOUT = 5
KRILL_ERR_NOT_FOUND = 6
KRILL_ERR_NO_DEVICE = 7

DTYPE_F16, DTYPE_BF16, DTYPE_F32, DTYPE_U8 = 0, 1, 2, 3
QUANT_F32, QUANT_INPUT_DTYPE = 0, 1
ATTN_TENSOR_CORE, ATTN_CUDA_CORE, ATTN_TENSOR_CORE_SYNC, ATTN_TENSOR_CORE_PAIR = 0, 1, 2, 3
KV_INT8, KV_BF16 = 0, 1
DEVICE_ERR_TIMEOUT = 1

_STATUS_NAMES = {
    1: "KRILL_ERR_INVALID", 2: "KRILL_ERR_OOM", 3: "KRILL_ERR_CUDA", 4: "KRILL_ERR_PEER",
    5: "KRILL_ERR_TIMEOUT", 6: "KRILL_ERR_NOT_FOUND", 7: "KRILL_ERR_NO_DEVICE",
}


class KrillError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class PoolCfg(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32),
        ("num_kv_heads", C.c_int32),
        ("num_q_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("group_size", C.c_int32),
        ("window", C.c_int32),
        ("max_append", C.c_int32),
        ("quant_variant", C.c_int32),
        ("attn_impl", C.c_int32),
        ("split_tokens", C.c_int32),
        ("cascade_min_tokens", C.c_int32),
        ("kv_format", C.c_int32),
        ("num_blocks", C.c_int64),
        ("wait_timeout_us", C.c_int32),
    ]


if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is not built; run `make -C krill_b200/csrc` (or __graft_entry__.build())")

lib = C.CDLL(LIB_PATH)

vp = C.c_void_p
i32, i64, u64, f32 = C.c_int32, C.c_int64, C.c_uint64, C.c_float
P_i64 = C.POINTER(C.c_int64)
P_i32 = C.POINTER(C.c_int32)
P_u64 = C.POINTER(C.c_uint64)
cstr = C.c_char_p

_SIGS = {
    "krill_last_error_string": (cstr, []),
    "krill_version": (cstr, []),
    "krill_pool_create": (i32, [C.POINTER(PoolCfg), i32, C.POINTER(vp)]),
    "krill_pool_destroy": (i32, [vp]),
    "krill_pool_block_bytes": (i32, [vp, P_i64]),
    "krill_pool_free_blocks": (i32, [vp, P_i64]),
    "krill_pool_block_refcount": (i32, [vp, i32, P_i32]),
    "krill_pool_device_error": (i32, [vp, P_i32]),
    "krill_pool_test_stall": (i32, [vp, i32]),
    "krill_pool_set_profiling": (i32, [vp, i32]),
    "krill_pool_kernel_times": (i32, [vp, C.POINTER(C.c_double), P_i32, C.POINTER(C.c_double), P_i32]),
    "krill_pool_last_plan": (i32, [vp, P_i32, P_i32, P_i64, P_i32]),
    "krill_pool_last_cascade": (i32, [vp, P_i32, P_i64, P_i32, P_i32]),
    "krill_pool_last_kernels": (i32, [vp, C.c_char_p, i32]),
    "krill_pool_kernel_count": (i32, [vp, P_i64]),
    "krill_seq_create": (i32, [vp, P_u64]),
    "krill_seq_release": (i32, [vp, u64]),
    "krill_seq_reset": (i32, [vp, u64]),
    "krill_seq_length": (i32, [vp, u64, i32, P_i64]),
    "krill_seq_retained": (i32, [vp, u64, i32, P_i64]),
    "krill_seq_memory_bytes": (i32, [vp, u64, i32, P_i64]),
    "krill_seq_truncate": (i32, [vp, u64, i64]),
    "krill_seq_can_truncate": (i32, [vp, u64, i64, P_i32]),
    "krill_seq_blocks": (i32, [vp, u64, P_i32, i32, P_i32]),
    "krill_append_quantize": (i32, [vp, i32, P_u64, i32, i32, i32, vp, vp, i32, vp]),
    "krill_verify_attention": (i32, [vp, i32, P_u64, i32, i32, i32, vp, i32, vp, i32, C.c_float, vp]),
    "krill_prefill_attention": (i32, [vp, i32, P_u64, i32, i32, i32, vp, i32, vp, i32, C.c_float, vp]),
    "krill_append_quantize_rope": (i32, [vp, i32, P_u64, i32, i32, i32, vp, vp, i32, vp, vp, i64, vp]),
    "krill_decode_attention": (i32, [vp, i32, P_u64, i32, i32, vp, i32, vp, i32, f32, vp]),
    "krill_decode_attention_noalloc": (i32, [vp, i32, P_u64, i32, i32, vp, i32, vp, i32, f32, vp]),
    "krill_decode_step": (i32, [vp, i32, P_u64, i32, i32, vp, vp, i32, vp, i32, vp, i32, f32, vp]),
    "krill_decode_step_host": (i32, [vp, i32, P_u64, i32, i32, vp, vp, i32, vp, i32, vp, i32, f32, i32,
                                     vp]),
    "krill_seq_snapshot_quantized": (i32, [vp, u64, i32, vp, vp, vp, vp, vp, vp, vp]),
    "krill_seq_snapshot_dequantized": (i32, [vp, u64, i32, vp, vp, vp]),
    "krill_seq_restore_quantized": (i32, [vp, u64, i32, i64, i64, vp, vp, vp, vp, vp, vp, vp]),
    "krill_stack_left_padded": (i32, [vp, i32, P_u64, i32, i64, vp, vp, vp, vp, vp, vp, vp]),
    "krill_scatter_back": (i32, [vp, i32, P_u64, i32, P_i64, i64, i64, vp, vp, vp, vp, vp, vp, vp]),
    "krill_build_decode_mask": (i32, [P_i64, i32, i64, i64, C.POINTER(C.c_float)]),
    "krill_prefix_create": (i32, [vp, i32, i32, C.POINTER(vp)]),
    "krill_prefix_destroy": (i32, [vp]),
    "krill_prefix_store": (i32, [vp, u64, P_i64, i64, cstr, cstr]),
    "krill_prefix_lookup": (i32, [vp, P_i64, i64, cstr, cstr, C.POINTER(vp), P_i64]),
    "krill_prefix_lookup_longest": (i32, [vp, P_i64, i64, cstr, cstr, C.POINTER(vp), P_i64]),
    "krill_prefix_entry_length": (i32, [vp, P_i64]),
    "krill_prefix_entry_release": (i32, [vp, vp]),
    "krill_seq_fork_prefix": (i32, [vp, vp, i64, P_u64]),
    "krill_prefix_clear": (i32, [vp]),
    "krill_prefix_set_disk": (i32, [vp, cstr, i64]),
    "krill_prefix_wait_disk": (i32, [vp]),
    "krill_prefix_disk_count": (i32, [vp, P_i32]),
    "krill_prefix_memory_count": (i32, [vp, P_i32]),
    "krill_prefix_key": (u64, [P_i64, i64, cstr, cstr, i32]),
    "krill_prefix_peer_fetch": (i32, [vp, vp, vp, vp, C.POINTER(vp)]),
    "krill_pool_ipc_handle": (i32, [vp, vp]),
    "krill_prefix_entry_describe": (i32, [vp, vp, vp, i64, P_i64]),
    "krill_prefix_import": (i32, [vp, vp, vp, i64, vp, C.POINTER(vp)]),
}

for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED = tuple(_SIGS)


def last_error() -> str:
    return lib.krill_last_error_string().decode("utf-8", "replace")


def check(status: int, allow=(KRILL_OK,)) -> int:
    if status not in allow:
        raise KrillError(status, last_error())
    return status
