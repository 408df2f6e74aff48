"""qwanto_b200 -- B200-native quantized paged KV-cache decode path for Qwanto.

The product is the shared library ``qwn_cuda.so`` (hand-written sm_100a CUDA
behind the C-ABI of include/qwn_cuda_abi.h and include/qwn_kv_b200.h).  This
package is the Python host side over that C-ABI, mirroring the reference's
interfaces:

* :class:`CudaContext` -- the qwnrun-facing ABI v1 (context, Q8 KV cache
  create/append/attention/reset/destroy, HyperVSQ-2 GEMV, telemetry), the
  calls c/qwanto_decode.c:267-462 and :1658-1724 make;
* :class:`KvPool` -- the paged, batched, device-resident extension
  (QwnKVBlockPool / block tables of c/qwn_paged_kv.h with the codecs of
  c/qwanto_turboquant.h, and page eviction after c/qwanto_pagedeviction.h).

Device buffers are passed as raw pointers; torch tensors (``.data_ptr()``)
or any CUDA allocation work.  Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import (CODEC_F16, CODEC_Q4_G32, CODEC_Q8_B64_F32, CODEC_Q8_HEAD_F16, CODEC_TQ35_G64, QwnCudaError, check,
                   init, lib)

__all__ = ["CudaContext", "KvPool", "lib", "QwnCudaError", "generate_rows", "merge_partials",
           "CODEC_Q8_B64_F32", "CODEC_Q8_HEAD_F16", "CODEC_TQ35_G64", "CODEC_Q4_G32", "CODEC_F16", "launch_count", "merge_partials_packed"]

TILE_BYTES = {CODEC_Q8_B64_F32: 4352, CODEC_Q8_HEAD_F16: 4160, CODEC_TQ35_G64: 2048, CODEC_Q4_G32: 2560,
              CODEC_F16: 8192}
# per token-head K+V bytes at head_dim 128 (the roofline's algorithmic bytes)
KV_BYTES_PER_TOKEN_HEAD = {CODEC_Q8_B64_F32: 272, CODEC_Q8_HEAD_F16: 260, CODEC_TQ35_G64: 128,
                           CODEC_Q4_G32: 160, CODEC_F16: 512}


def _ptr(x) -> int | None:
    """Device/host address of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)}")


def _stream(s) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream  # torch.cuda.Stream


def launch_count() -> int:
    """Kernel launches issued by qwn_cuda.so in this process."""
    return int(lib().qwn_kv_launch_count())


def d2h(dev_ptr: int, shape, dtype) -> np.ndarray:
    out = np.empty(shape, dtype=dtype)
    check("qwn_kv_memcpy_d2h", lib().qwn_kv_memcpy_d2h(out.ctypes.data, dev_ptr, out.nbytes))
    return out


def generate_rows(out, rows: int, width: int, kind: int, seed: int, layer: int, seq_ids, positions,
                  outlier_mask=None, stream=None) -> None:
    """Fill out[rows][width] with the synthetic ~N(0,1) rows (kind 1=Q, 2=K, 3=V)."""
    check("qwn_kv_generate_rows", lib().qwn_kv_generate_rows(
        _ptr(out), rows, width, kind, seed, layer, _ptr(seq_ids), _ptr(positions), _ptr(outlier_mask),
        _stream(stream)))


def merge_partials(parts: int, rows: int, m, l, o, out, stream=None) -> None:
    check("qwn_kv_merge_partials", lib().qwn_kv_merge_partials(parts, rows, _ptr(m), _ptr(l), _ptr(o),
                                                                _ptr(out), _stream(stream)))


def merge_partials_packed(parts: int, rows: int, packed, out, stream=None) -> None:
    """Merge `parts` blocks of rows*130 floats (o[rows][128], m[rows], l[rows])."""
    check("qwn_kv_merge_partials_packed", lib().qwn_kv_merge_partials_packed(parts, rows, _ptr(packed), _ptr(out),
                                                                              _stream(stream)))


class KvPool:
    """Device-resident paged quantized KV pool (one per GPU)."""

    def __init__(self, codec: int, layers: int, kv_heads: int, page_tokens: int, total_pages: int,
                 max_seqs: int, max_pages_per_seq: int, max_query_heads: int | None = None,
                 permutation_seed: int = 0, device: int = 0, memory_budget_bytes: int = 0):
        o = init(_lib.PoolOptions())
        o.device_id, o.codec, o.layers, o.kv_heads, o.head_dim = device, codec, layers, kv_heads, 128
        o.page_tokens, o.total_pages, o.max_seqs = page_tokens, total_pages, max_seqs
        o.max_pages_per_seq = max_pages_per_seq
        o.max_query_heads = max_query_heads or 0
        o.permutation_seed, o.memory_budget_bytes = permutation_seed, memory_budget_bytes
        self.h = init(_lib.Handle())
        check("qwn_kv_pool_create", lib().qwn_kv_pool_create(C.byref(o), C.byref(self.h)))
        self.codec, self.layers, self.kv_heads, self.page_tokens = codec, layers, kv_heads, page_tokens
        self.total_pages, self.max_seqs, self.max_pages_per_seq = total_pages, max_seqs, max_pages_per_seq
        self.device = device
        info = init(_lib.PoolInfo())
        check("qwn_kv_pool_get_info", lib().qwn_kv_pool_get_info(C.byref(self.h), C.byref(info)))
        self.info = info

    def close(self) -> None:
        if self.h is not None and self.h.opaque:
            lib().qwn_kv_pool_destroy(C.byref(self.h))
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- state ------------------------------------------------------------
    def check(self) -> int:
        bits = C.c_uint32(0)
        check("qwn_kv_pool_check", lib().qwn_kv_pool_check(C.byref(self.h), C.byref(bits)))
        return int(bits.value)

    def reset(self) -> None:
        check("qwn_kv_pool_reset", lib().qwn_kv_pool_reset(C.byref(self.h)))

    def lens(self) -> np.ndarray:
        return d2h(self.info.seq_lens_dev, (self.max_seqs,), np.int32)

    def npages(self) -> np.ndarray:
        return d2h(self.info.seq_pages_dev, (self.max_seqs,), np.int32)

    def page_table(self) -> np.ndarray:
        return d2h(self.info.page_table_dev, (self.max_seqs, self.max_pages_per_seq), np.int32)

    def scores(self) -> np.ndarray:
        return d2h(self.info.page_scores_dev, (self.max_seqs, self.max_pages_per_seq), np.float32)

    def free_stack(self) -> np.ndarray:
        top = int(d2h(self.info.free_top_dev, (1,), np.int32)[0])
        return d2h(self.info.free_stack_dev, (self.total_pages,), np.int32)[:top]

    def page(self, phys: int) -> np.ndarray:
        pb = int(self.info.page_bytes)
        return d2h(self.info.pages_dev + phys * pb, (pb,), np.uint8)

    # -- operations ---------------------------------------------------------
    def seq_append(self, num_seqs: int, seq_ids=None, counts=None, stream=None) -> None:
        check("qwn_kv_seq_append", lib().qwn_kv_seq_append(C.byref(self.h), num_seqs, _ptr(seq_ids),
                                                            _ptr(counts), _stream(stream)))

    def decode(self, layer: int, num_seqs: int, query_heads: int, query, output, key=None, value=None,
               seq_ids=None, scale: float = 0.0, page_mass=None, attend_limit: int = 0, stream=None) -> None:
        r = init(_lib.DecodeRequest())
        r.layer, r.num_seqs, r.seq_ids_dev, r.query_heads, r.scale = layer, num_seqs, _ptr(seq_ids), query_heads, scale
        r.query_dev, r.key_dev, r.value_dev, r.output_dev = _ptr(query), _ptr(key), _ptr(value), _ptr(output)
        r.page_mass_dev, r.attend_limit, r.stream = _ptr(page_mass), attend_limit, _stream(stream)
        check("qwn_kv_decode", lib().qwn_kv_decode(C.byref(self.h), C.byref(r)))

    def append(self, layer: int, num_seqs: int, key, value, seq_ids=None, stream=None) -> None:
        check("qwn_kv_append", lib().qwn_kv_append(C.byref(self.h), layer, num_seqs, _ptr(seq_ids), _ptr(key),
                                                    _ptr(value), _stream(stream)))

    def partial(self, layer: int, num_seqs: int, query_heads: int, query, m, l, o, t_begin: int = 0,
                t_end: int = 0, seq_ids=None, scale: float = 0.0, stream=None) -> None:
        r = init(_lib.PartialRequest())
        r.layer, r.num_seqs, r.seq_ids_dev, r.query_heads, r.scale = layer, num_seqs, _ptr(seq_ids), query_heads, scale
        r.query_dev, r.m_dev, r.l_dev, r.o_dev = _ptr(query), _ptr(m), _ptr(l), _ptr(o)
        r.t_begin, r.t_end, r.stream = t_begin, t_end, _stream(stream)
        check("qwn_kv_partial", lib().qwn_kv_partial(C.byref(self.h), C.byref(r)))

    def decode_split(self, layer: int, query_heads: int, query, output, exchange, t_begin: int = 0, t_end: int = 0,
                     key=None, value=None, seq_ids=None, scale: float = 0.0, stream=None) -> None:
        """Split-KV decode of one sequence over the ranks of `exchange`
        (a :class:`qwanto_b200.exchange.PeerExchange`): this rank attends
        [t_begin, t_end) (t_end 0 = to the end, where key/value store the
        newest token) and every rank receives the merged output rows."""
        r = init(_lib.SplitRequest())
        r.layer, r.query_heads, r.seq_ids_dev, r.scale = layer, query_heads, _ptr(seq_ids), scale
        r.epoch = exchange.next_epoch()
        r.query_dev, r.key_dev, r.value_dev, r.output_dev = _ptr(query), _ptr(key), _ptr(value), _ptr(output)
        r.t_begin, r.t_end = t_begin, t_end
        r.peers = C.addressof(exchange.peers)
        r.stream = _stream(stream)
        check("qwn_kv_decode_split", lib().qwn_kv_decode_split(C.byref(self.h), C.byref(r)))

    def store_tokens(self, seq: int, layer: int, first_pos: int, n_tokens: int, key, value, stream=None) -> None:
        check("qwn_kv_store_tokens", lib().qwn_kv_store_tokens(C.byref(self.h), seq, layer, first_pos, n_tokens,
                                                                _ptr(key), _ptr(value), _stream(stream)))

    def prefill_synthetic(self, seq_ids, lens, seed: int, outlier_mask: np.ndarray | None = None,
                          stream=None) -> None:
        ids = np.ascontiguousarray(seq_ids, dtype=np.int32)
        ln = np.ascontiguousarray(lens, dtype=np.int32)
        mask = None if outlier_mask is None else np.ascontiguousarray(outlier_mask, dtype=np.uint8)
        check("qwn_kv_prefill_synthetic", lib().qwn_kv_prefill_synthetic(
            C.byref(self.h), ids.size, ids.ctypes.data, ln.ctypes.data, seed,
            None if mask is None else mask.ctypes.data, _stream(stream)))

    def evict(self, num_seqs: int, page_mass, flags, token_budget: int, seq_ids=None, stream=None) -> None:
        r = init(_lib.EvictRequest())
        r.num_seqs, r.seq_ids_dev, r.page_mass_dev, r.flags_dev = num_seqs, _ptr(seq_ids), _ptr(page_mass), _ptr(flags)
        r.token_budget, r.stream = token_budget, _stream(stream)
        check("qwn_kv_evict", lib().qwn_kv_evict(C.byref(self.h), C.byref(r)))

    def decode_step_host(self, num_layers: int, num_seqs: int, query_heads: int, host_query, host_key,
                         host_value, host_output, scale: float = 0.0, telemetry=None) -> None:
        r = init(_lib.HostStepRequest())
        r.num_layers, r.num_seqs, r.query_heads, r.scale = num_layers, num_seqs, query_heads, scale
        r.host_query, r.host_key, r.host_value = _ptr(host_query), _ptr(host_key), _ptr(host_value)
        r.host_output = _ptr(host_output)
        tel = telemetry if telemetry is not None else init(_lib.Telemetry())
        check("qwn_kv_decode_step_host", lib().qwn_kv_decode_step_host(C.byref(self.h), C.byref(r), C.byref(tel)))


class CudaContext:
    """The qwnrun-facing ABI v1 (c/cuda/qwn_cuda_abi.h), one CUDA device."""

    def __init__(self, device: int = 0, memory_budget_bytes: int = 0, context_size: int = 0):
        o = init(_lib.ContextOptions())
        o.device_id, o.memory_budget_bytes, o.context_size = device, memory_budget_bytes, context_size
        self.h = init(_lib.Handle())
        check("qwn_cuda_abi_context_create", lib().qwn_cuda_abi_context_create(C.byref(o), C.byref(self.h)))

    @staticmethod
    def query() -> _lib.AbiInfo:
        info = init(_lib.AbiInfo())
        check("qwn_cuda_abi_query", lib().qwn_cuda_abi_query(C.byref(info)))
        return info

    @staticmethod
    def devices():
        arr = (_lib.DeviceInfo * 16)()
        for d in arr:
            init(d)
        n = C.c_uint32(0)
        rc = lib().qwn_cuda_abi_enumerate_devices(arr, 16, C.byref(n))
        return rc, [arr[i] for i in range(min(n.value, 16))]

    def close(self) -> None:
        if self.h is not None and self.h.opaque:
            lib().qwn_cuda_abi_context_destroy(C.byref(self.h))
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def kv_cache_create(self, max_tokens: int, kv_heads: int, head_dim: int) -> _lib.Handle:
        o = init(_lib.KvCacheOptions())
        o.max_tokens, o.kv_heads, o.head_dim = max_tokens, kv_heads, head_dim
        h = init(_lib.Handle())
        check("qwn_cuda_abi_kv_cache_create", lib().qwn_cuda_abi_kv_cache_create(C.byref(self.h), C.byref(o),
                                                                                  C.byref(h)))
        return h

    def kv_cache_append(self, cache, key: np.ndarray, value: np.ndarray, token: int) -> _lib.Telemetry:
        key = np.ascontiguousarray(key, dtype=np.float32)
        value = np.ascontiguousarray(value, dtype=np.float32)
        r = init(_lib.KvAppendRequest())
        r.cache = cache
        r.host_key = key.ctypes.data_as(C.POINTER(C.c_float))
        r.host_value = value.ctypes.data_as(C.POINTER(C.c_float))
        r.n_channels, r.token = key.size, token
        tel = init(_lib.Telemetry())
        check("qwn_cuda_abi_kv_cache_append", lib().qwn_cuda_abi_kv_cache_append(C.byref(self.h), C.byref(r),
                                                                                  C.byref(tel)))
        return tel

    def kv_cache_attention(self, cache, query: np.ndarray, query_heads: int, kv_heads: int, head_dim: int,
                           position: int, scale: float):
        query = np.ascontiguousarray(query, dtype=np.float32)
        out = np.zeros(query_heads * head_dim, dtype=np.float32)
        r = init(_lib.KvAttentionRequest())
        r.cache = cache
        r.host_query = query.ctypes.data_as(C.POINTER(C.c_float))
        r.host_output = out.ctypes.data_as(C.POINTER(C.c_float))
        r.query_heads, r.kv_heads, r.head_dim, r.position, r.scale = query_heads, kv_heads, head_dim, position, scale
        tel = init(_lib.Telemetry())
        check("qwn_cuda_abi_kv_cache_attention", lib().qwn_cuda_abi_kv_cache_attention(
            C.byref(self.h), C.byref(r), C.byref(tel)))
        return out, tel

    def kv_cache_reset(self, cache) -> None:
        check("qwn_cuda_abi_kv_cache_reset", lib().qwn_cuda_abi_kv_cache_reset(C.byref(self.h), C.byref(cache)))

    def kv_cache_destroy(self, cache) -> None:
        check("qwn_cuda_abi_kv_cache_destroy", lib().qwn_cuda_abi_kv_cache_destroy(C.byref(self.h),
                                                                                   C.byref(cache)))

    def telemetry(self) -> _lib.Telemetry:
        tel = init(_lib.Telemetry())
        check("qwn_cuda_abi_get_telemetry", lib().qwn_cuda_abi_get_telemetry(C.byref(self.h), C.byref(tel)))
        return tel
