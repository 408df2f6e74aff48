"""ctypes binding of qwn_cuda.so (include/qwn_cuda_abi.h, include/qwn_kv_b200.h).

There is no CPU implementation behind this module: when the CUDA library is
missing the import of :func:`lib` raises, so no caller can silently run a
fallback.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "qwn_cuda.so")

ABI_VERSION = 1
STATUS = {0: "OK", -1: "INVALID_ARGUMENT", -2: "ABI_MISMATCH", -3: "UNAVAILABLE",
          -4: "OUT_OF_MEMORY", -5: "UNSUPPORTED", -6: "RUNTIME_ERROR"}

CODEC_Q8_B64_F32 = 1
CODEC_Q8_HEAD_F16 = 2
CODEC_TQ35_G64 = 3
CODEC_Q4_G32 = 4
CODEC_F16 = 5

CAP_HYPERVSQ2_GEMV = 1 << 0
CAP_Q8_KV = 1 << 5
CAP_PAGED_KV = 1 << 6
CAP_TQ_KV = 1 << 7
CAP_BATCHED_DEVICE = 1 << 8
CAP_SPLIT_KV_MERGE = 1 << 9
CAP_PAGE_EVICTION = 1 << 10

ST_POOL_EXHAUSTED = 1 << 0
ST_TABLE_OVERFLOW = 1 << 1
ST_BAD_PAGE = 1 << 2
ST_BAD_SEQUENCE = 1 << 3
ST_WAIT_TIMEOUT = 1 << 4
ST_BAD_LENGTH = 1 << 5
ST_PEER_TIMEOUT = 1 << 6

MAX_RANKS = 8
EXCHANGE_SEGMENTS = 64


class Header(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("abi_version", C.c_uint32), ("reserved", C.c_uint32 * 4)]


def init(struct):
    """qwn_cuda_abi_header_init on a ctypes structure whose first field is `header`."""
    struct.header.struct_size = C.sizeof(struct)
    struct.header.abi_version = ABI_VERSION
    return struct


class AbiInfo(C.Structure):
    _fields_ = [("header", Header), ("capability_bits", C.c_uint64), ("max_devices", C.c_uint32),
                ("max_resident_tensors", C.c_uint32), ("hypervsq2_block_bytes", C.c_uint32),
                ("hypervsq2_block_elements", C.c_uint32), ("abi_name", C.c_char * 32)]


class DeviceInfo(C.Structure):
    _fields_ = [("header", Header), ("device_id", C.c_int32), ("compute_major", C.c_int32),
                ("compute_minor", C.c_int32), ("total_vram_bytes", C.c_uint64),
                ("free_vram_bytes", C.c_uint64), ("name", C.c_char * 128), ("driver", C.c_char * 64)]


class ContextOptions(C.Structure):
    _fields_ = [("header", Header), ("device_id", C.c_int32), ("flags", C.c_uint32),
                ("memory_budget_bytes", C.c_uint64), ("context_size", C.c_uint64)]


class Handle(C.Structure):
    _fields_ = [("header", Header), ("opaque", C.c_void_p)]


class KvCacheOptions(C.Structure):
    _fields_ = [("header", Header), ("max_tokens", C.c_uint32), ("kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("reserved", C.c_uint32)]


class KvAppendRequest(C.Structure):
    _fields_ = [("header", Header), ("cache", Handle), ("host_key", C.POINTER(C.c_float)),
                ("host_value", C.POINTER(C.c_float)), ("n_channels", C.c_uint32), ("token", C.c_uint32)]


class KvAttentionRequest(C.Structure):
    _fields_ = [("header", Header), ("cache", Handle), ("host_query", C.POINTER(C.c_float)),
                ("host_output", C.POINTER(C.c_float)), ("query_heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("position", C.c_uint32),
                ("scale", C.c_float)]


class TensorUpload(C.Structure):
    _fields_ = [("header", Header), ("host_data", C.c_void_p), ("data_bytes", C.c_uint64),
                ("dtype", C.c_uint32), ("rows", C.c_uint32), ("cols", C.c_uint32),
                ("block_bytes", C.c_uint32)]


class GemmRequest(C.Structure):
    _fields_ = [("header", Header), ("tensor", Handle), ("input_q8", C.c_void_p),
                ("input_scale", C.c_float), ("input_scales", C.POINTER(C.c_float)),
                ("output", C.POINTER(C.c_float)), ("batch", C.c_uint32), ("rows", C.c_uint32),
                ("cols", C.c_uint32), ("input_stride", C.c_uint32), ("output_stride", C.c_uint32),
                ("input_mode", C.c_uint32)]


class Telemetry(C.Structure):
    _fields_ = [("header", Header), ("gpu_matmul_count", C.c_uint64), ("gpu_kernel_launch_count", C.c_uint64),
                ("gpu_projection_count", C.c_uint64), ("gpu_upload_count", C.c_uint64),
                ("gpu_upload_bytes", C.c_uint64), ("gpu_resident_bytes", C.c_uint64),
                ("cpu_matmul_fallback_count", C.c_uint64), ("unsupported_projection_count", C.c_uint64),
                ("gpu_kernel_ms", C.c_double), ("gpu_transfer_ms", C.c_double), ("gpu_sync_ms", C.c_double),
                ("device_id", C.c_int32), ("reserved_device", C.c_uint32), ("device_name", C.c_char * 128),
                ("kernel_type", C.c_char * 32), ("dll_hash", C.c_char * 65),
                ("kv_cache_kernel_count", C.c_uint64), ("kv_cache_upload_bytes", C.c_uint64),
                ("kv_cache_resident_bytes", C.c_uint64), ("kv_cache_kernel_ms", C.c_double),
                ("kv_cache_transfer_ms", C.c_double), ("kv_cache_kernel_type", C.c_char * 32)]


class PoolOptions(C.Structure):
    _fields_ = [("header", Header), ("device_id", C.c_int32), ("codec", C.c_uint32), ("layers", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("page_tokens", C.c_uint32),
                ("total_pages", C.c_uint32), ("max_seqs", C.c_uint32), ("max_pages_per_seq", C.c_uint32),
                ("max_query_heads", C.c_uint32), ("permutation_seed", C.c_uint64),
                ("memory_budget_bytes", C.c_uint64)]


class PoolInfo(C.Structure):
    _fields_ = [("header", Header), ("pages_dev", C.c_void_p), ("page_table_dev", C.c_void_p),
                ("seq_lens_dev", C.c_void_p), ("seq_pages_dev", C.c_void_p), ("free_stack_dev", C.c_void_p),
                ("free_top_dev", C.c_void_p), ("page_scores_dev", C.c_void_p), ("status_dev", C.c_void_p),
                ("tile_bytes", C.c_uint64), ("page_bytes", C.c_uint64), ("pool_bytes", C.c_uint64),
                ("scratch_bytes", C.c_uint64), ("attention_ctas", C.c_uint32), ("attention_warps", C.c_uint32),
                ("reserved", C.c_uint32)]


class DecodeRequest(C.Structure):
    _fields_ = [("header", Header), ("layer", C.c_uint32), ("num_seqs", C.c_uint32), ("seq_ids_dev", C.c_void_p),
                ("query_heads", C.c_uint32), ("scale", C.c_float), ("query_dev", C.c_void_p),
                ("key_dev", C.c_void_p), ("value_dev", C.c_void_p), ("output_dev", C.c_void_p),
                ("page_mass_dev", C.c_void_p), ("attend_limit", C.c_uint32), ("reserved", C.c_uint32),
                ("stream", C.c_void_p)]


class PartialRequest(C.Structure):
    _fields_ = [("header", Header), ("layer", C.c_uint32), ("num_seqs", C.c_uint32), ("seq_ids_dev", C.c_void_p),
                ("query_heads", C.c_uint32), ("scale", C.c_float), ("query_dev", C.c_void_p),
                ("m_dev", C.c_void_p), ("l_dev", C.c_void_p), ("o_dev", C.c_void_p), ("t_begin", C.c_uint32),
                ("t_end", C.c_uint32), ("stream", C.c_void_p)]


class EvictRequest(C.Structure):
    _fields_ = [("header", Header), ("num_seqs", C.c_uint32), ("seq_ids_dev", C.c_void_p),
                ("page_mass_dev", C.c_void_p), ("flags_dev", C.c_void_p), ("token_budget", C.c_uint32),
                ("reserved", C.c_uint32), ("stream", C.c_void_p)]


class HostStepRequest(C.Structure):
    _fields_ = [("header", Header), ("num_layers", C.c_uint32), ("num_seqs", C.c_uint32),
                ("query_heads", C.c_uint32), ("scale", C.c_float), ("host_query", C.c_void_p),
                ("host_key", C.c_void_p), ("host_value", C.c_void_p), ("host_output", C.c_void_p)]


class StaticAttentionRequest(C.Structure):
    _fields_ = [("header", Header), ("device_id", C.c_int32), ("codec", C.c_uint32), ("layers", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("page_tokens", C.c_uint32),
                ("total_pages", C.c_uint32), ("max_seqs", C.c_uint32), ("max_pages_per_seq", C.c_uint32),
                ("layer", C.c_uint32), ("num_seqs", C.c_uint32), ("query_heads", C.c_uint32),
                ("scale", C.c_float), ("pages_dev", C.c_void_p), ("page_table_dev", C.c_void_p),
                ("seq_lens_dev", C.c_void_p), ("seq_ids_dev", C.c_void_p), ("query_dev", C.c_void_p),
                ("output_dev", C.c_void_p), ("status_dev", C.c_void_p), ("stream", C.c_void_p)]



class PeerSet(C.Structure):
    _fields_ = [("header", Header), ("rank", C.c_uint32), ("world", C.c_uint32), ("max_rows", C.c_uint32),
                ("reserved", C.c_uint32), ("buffers", C.c_void_p * 8), ("timeout_ns", C.c_uint64)]


class SplitRequest(C.Structure):
    _fields_ = [("header", Header), ("layer", C.c_uint32), ("query_heads", C.c_uint32), ("seq_ids_dev", C.c_void_p),
                ("scale", C.c_float), ("epoch", C.c_uint32), ("query_dev", C.c_void_p), ("key_dev", C.c_void_p),
                ("value_dev", C.c_void_p), ("output_dev", C.c_void_p), ("t_begin", C.c_uint32),
                ("t_end", C.c_uint32), ("peers", C.c_void_p), ("stream", C.c_void_p)]

class LinearAttentionState(C.Structure):
    _fields_ = [("n_heads", C.c_int32), ("head_dim", C.c_int32), ("state", C.c_void_p), ("device_id", C.c_int32),
                ("reserved", C.c_uint32), ("staging", C.c_void_p), ("staging_bytes", C.c_uint64)]


_P = C.POINTER
_SIGS = {
    "qwn_cuda_abi_query": (C.c_int, [_P(AbiInfo)]),
    "qwn_cuda_abi_get_capabilities": (C.c_int, [_P(AbiInfo)]),
    "qwn_cuda_abi_enumerate_devices": (C.c_int, [_P(DeviceInfo), C.c_uint32, _P(C.c_uint32)]),
    "qwn_cuda_abi_context_create": (C.c_int, [_P(ContextOptions), _P(Handle)]),
    "qwn_cuda_abi_context_destroy": (C.c_int, [_P(Handle)]),
    "qwn_cuda_abi_upload_tensor": (C.c_int, [_P(Handle), _P(TensorUpload), _P(Handle)]),
    "qwn_cuda_abi_release_tensor": (C.c_int, [_P(Handle), _P(Handle)]),
    "qwn_cuda_abi_kv_cache_create": (C.c_int, [_P(Handle), _P(KvCacheOptions), _P(Handle)]),
    "qwn_cuda_abi_kv_cache_destroy": (C.c_int, [_P(Handle), _P(Handle)]),
    "qwn_cuda_abi_kv_cache_append": (C.c_int, [_P(Handle), _P(KvAppendRequest), _P(Telemetry)]),
    "qwn_cuda_abi_kv_cache_attention": (C.c_int, [_P(Handle), _P(KvAttentionRequest), _P(Telemetry)]),
    "qwn_cuda_abi_kv_cache_reset": (C.c_int, [_P(Handle), _P(Handle)]),
    "qwn_cuda_abi_hypervsq2_gemv": (C.c_int, [_P(Handle), _P(GemmRequest), _P(Telemetry)]),
    "qwn_cuda_abi_hypervsq2_gemm": (C.c_int, [_P(Handle), _P(GemmRequest), _P(Telemetry)]),
    "qwn_cuda_abi_synchronize": (C.c_int, [_P(Handle)]),
    "qwn_cuda_abi_get_telemetry": (C.c_int, [_P(Handle), _P(Telemetry)]),
    "qwn_cuda_abi_last_error": (C.c_int, [C.c_char_p, C.c_uint32]),
    "qwn_kv_pool_create": (C.c_int, [_P(PoolOptions), _P(Handle)]),
    "qwn_kv_pool_destroy": (C.c_int, [_P(Handle)]),
    "qwn_kv_pool_get_info": (C.c_int, [_P(Handle), _P(PoolInfo)]),
    "qwn_kv_pool_reset": (C.c_int, [_P(Handle)]),
    "qwn_kv_pool_check": (C.c_int, [_P(Handle), _P(C.c_uint32)]),
    "qwn_kv_seq_append": (C.c_int, [_P(Handle), C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "qwn_kv_decode": (C.c_int, [_P(Handle), _P(DecodeRequest)]),
    "qwn_kv_append": (C.c_int, [_P(Handle), C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_void_p]),
    "qwn_kv_partial": (C.c_int, [_P(Handle), _P(PartialRequest)]),
    "qwn_kv_merge_partials": (C.c_int, [C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p]),
    "qwn_kv_merge_partials_packed": (C.c_int, [C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "qwn_kv_exchange_bytes": (C.c_int, [C.c_uint32, _P(C.c_uint64)]),
    "qwn_kv_exchange_alloc": (C.c_int, [C.c_int32, C.c_uint64, _P(C.c_void_p), C.c_void_p]),
    "qwn_kv_exchange_free": (C.c_int, [C.c_int32, C.c_void_p]),
    "qwn_kv_exchange_open": (C.c_int, [C.c_int32, C.c_void_p, _P(C.c_void_p)]),
    "qwn_kv_exchange_close": (C.c_int, [C.c_int32, C.c_void_p]),
    "qwn_kv_decode_split": (C.c_int, [_P(Handle), _P(SplitRequest)]),
    "qwn_kv_store_tokens": (C.c_int, [_P(Handle), C.c_int32, C.c_uint32, C.c_uint32, C.c_uint32,
                                      C.c_void_p, C.c_void_p, C.c_void_p]),
    "qwn_kv_generate_rows": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64,
                                       C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "qwn_kv_prefill_synthetic": (C.c_int, [_P(Handle), C.c_uint32, C.c_void_p, C.c_void_p, C.c_uint64,
                                           C.c_void_p, C.c_void_p]),
    "qwn_kv_evict": (C.c_int, [_P(Handle), _P(EvictRequest)]),
    "qwn_kv_decode_step_host": (C.c_int, [_P(Handle), _P(HostStepRequest), _P(Telemetry)]),
    "qwn_kv_attention_static": (C.c_int, [_P(StaticAttentionRequest)]),
    "qwn_kv_memcpy_d2h": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "qwn_kv_memcpy_h2d": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "qwn_kv_launch_count": (C.c_uint64, []),
    "qwn_linear_attention_init": (C.c_int, [_P(LinearAttentionState), C.c_int32, C.c_int32, C.c_int32]),
    "qwn_linear_attention_reset": (C.c_int, [_P(LinearAttentionState), C.c_void_p]),
    "qwn_linear_attention_destroy": (C.c_int, [_P(LinearAttentionState)]),
    "qwn_linear_attention_decode": (C.c_int, [_P(LinearAttentionState), C.c_void_p, C.c_void_p, C.c_void_p,
                                              C.c_float, C.c_void_p, C.c_void_p]),
    "qwn_linear_attention_prefill": (C.c_int, [_P(LinearAttentionState), C.c_void_p, C.c_void_p, C.c_void_p,
                                               C.c_float, C.c_int32, C.c_void_p, C.c_void_p]),
    "qwn_linear_attention_prefill_host": (C.c_int, [_P(LinearAttentionState), C.c_void_p, C.c_void_p,
                                                    C.c_void_p, C.c_float, C.c_int32, C.c_void_p]),
}

_lib = None


def lib() -> C.CDLL:
    """Load qwn_cuda.so.  Raises if it was not built: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no CPU fallback exists)")
        # RTLD_LOCAL: the library exports the reference's C API names, which
        # must not interpose on another library of the process that defines
        # them too (the reference's own code loaded beside it in the tests)
        L = C.CDLL(LIB_PATH, mode=C.RTLD_LOCAL)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(512)
    lib().qwn_cuda_abi_last_error(buf, 512)
    return buf.value.decode(errors="replace")


class QwnCudaError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} -> {STATUS.get(code, code)}: {last_error()}")
        self.code = code


def check(fn: str, code: int) -> int:
    if code != 0:
        raise QwnCudaError(fn, code)
    return code
