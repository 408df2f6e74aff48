"""ctypes wrapper of the CPU oracle and of the reference's own CPU code.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg; the product package never imports it.

``lib()`` is this project's C restatement (qwn_oracle.c); ``ref()`` is the
reference's c/qwanto_turboquant.c, c/qwn_paged_kv.c and
c/qwanto_pagedeviction.c compiled from the reference sources by
oracle/Makefile (None when that build is absent).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libqwn_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libqwnref.so")

CODEC_Q8_B64_F32 = 1
CODEC_Q8_HEAD_F16 = 2
CODEC_TQ35_G64 = 3
CODEC_Q4_G32 = 4
CODEC_F16 = 5
CODEC_NAMES = {1: "q8_b64_f32", 2: "q8_head_f16", 3: "tq35_g64", 4: "q4_g32", 5: "f16"}
TILE_BYTES = {1: 4352, 2: 4160, 3: 2048, 4: 2560, 5: 8192}

_lib = None
_ref = None
_ref_tried = False

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int32)
u8p = C.POINTER(C.c_uint8)
i8p = C.POINTER(C.c_int8)
u16p = C.POINTER(C.c_uint16)
i16p = C.POINTER(C.c_int16)


def build(reference: bool = True) -> None:
    """Compile the oracle (and the reference objects when the sources exist)."""
    from oracle.refpath import reference_c
    targets = ["oracle"] + (["ref"] if reference else [])
    ref = reference_c() if reference else None
    subprocess.run(["make", "-s", "-C", HERE] + targets + ([f"REF={ref}"] if ref else []), check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class QorPool(C.Structure):
    _fields_ = [
        ("codec", C.c_int), ("layers", C.c_int), ("kv_heads", C.c_int),
        ("page_tokens", C.c_int), ("total_pages", C.c_int), ("max_seqs", C.c_int),
        ("max_pages_per_seq", C.c_int), ("tile_bytes", C.c_size_t),
        ("page_bytes", C.c_size_t), ("pages", u8p), ("free_stack", i32p),
        ("free_top", C.c_int32), ("page_table", i32p), ("lens", i32p),
        ("npages", i32p), ("page_score", f32p),
    ]


class VToken(C.Structure):
    _fields_ = [("token_id", C.c_uint32), ("importance_score", C.c_float),
                ("physical_slot", C.c_uint32), ("is_sink", C.c_uint8),
                ("is_active", C.c_uint8)]


class EvictionPool(C.Structure):
    """Layout of both QorEvictionPool and the reference QwnPagedEvictionPool
    (c/qwanto_pagedeviction.h:19-34)."""
    _fields_ = [("tokens", VToken * 32768), ("active_count", C.c_uint32),
                ("max_capacity", C.c_uint32), ("physical_pool_size", C.c_uint32),
                ("eviction_threshold", C.c_float), ("total_evictions", C.c_uint64)]


class KvContract(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("abi_version", C.c_uint32),
                ("cache_dtype", C.c_uint32), ("block_size", C.c_uint32),
                ("scale_bytes", C.c_uint32), ("zero_point_bytes", C.c_uint32),
                ("key_layout", C.c_uint32), ("value_layout", C.c_uint32),
                ("page_size", C.c_uint32), ("alignment", C.c_uint32),
                ("valid_token_count", C.c_uint32), ("reserved", C.c_uint32 * 5)]


class RefQ8Cache(C.Structure):
    """c/qwanto_turboquant.h:80-94"""
    _fields_ = [("packed_k", i8p), ("packed_v", i8p), ("scales_k", f32p),
                ("scales_v", f32p), ("n_channels", C.c_int), ("n_tokens", C.c_int),
                ("max_tokens", C.c_int), ("n_heads", C.c_int), ("head_dim", C.c_int),
                ("token_stride", C.c_size_t), ("scale_stride", C.c_size_t),
                ("total_bytes", C.c_size_t), ("contract", KvContract)]


class RefTQCache(C.Structure):
    """c/qwanto_turboquant.h:65-76"""
    _fields_ = [("packed_k", u8p), ("packed_v", u8p), ("n_channels", C.c_int),
                ("n_tokens", C.c_int), ("max_tokens", C.c_int), ("n_heads", C.c_int),
                ("head_dim", C.c_int), ("token_stride_k", C.c_size_t),
                ("token_stride_v", C.c_size_t), ("total_bytes", C.c_size_t)]


class RefLinearState(C.Structure):  # QwantoLinearAttentionState, c/qwanto_attention.h:11-15
    _fields_ = [("n_heads", C.c_int), ("head_dim", C.c_int), ("state", C.POINTER(C.c_float))]


class RefBlockPool(C.Structure):
    """c/qwn_paged_kv.h:15-25"""
    _fields_ = [("key_data", u16p), ("val_data", u16p), ("free_stack", i32p),
                ("free_top", C.c_int), ("total_blocks", C.c_int), ("layers", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("block_bytes", C.c_size_t)]


class RefBlockTable(C.Structure):
    """c/qwn_paged_kv.h:27-36"""
    _fields_ = [("req_id", C.c_int), ("num_tokens", C.c_int), ("max_tokens", C.c_int),
                ("block_ids", i32p), ("block_count", C.c_int), ("block_capacity", C.c_int),
                ("prefill_remaining", C.c_int), ("prefill_offset", C.c_int)]


def _decl(L, name, res, *args):
    fn = getattr(L, name)
    fn.restype = res
    fn.argtypes = list(args)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(reference=False)
        L = C.CDLL(ORACLE_SO)
        _decl(L, "qor_mix64", C.c_uint64, C.c_uint64)
        _decl(L, "qor_normal", C.c_float, C.c_uint64, C.c_uint64, C.c_uint64)
        _decl(L, "qor_fill_normal", None, C.c_uint64, C.c_uint64, C.c_uint64, f32p, C.c_size_t)
        _decl(L, "qor_stream", C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32)
        _decl(L, "qor_permuted_free_stack", None, C.c_uint64, C.c_int, i32p)
        _decl(L, "qor_outlier_channels", None, C.c_uint64, C.c_uint32, C.c_int, C.c_int, u8p)
        _decl(L, "qor_f32_to_f16_rne", C.c_uint16, C.c_float)
        _decl(L, "qor_f16_to_f32", C.c_float, C.c_uint16)
        _decl(L, "qor_tq_f32_to_f16", C.c_uint16, C.c_float)
        _decl(L, "qor_q8_b64_quantize", None, f32p, C.c_int, i8p, f32p)
        _decl(L, "qor_q8_head_quantize", None, f32p, C.c_int, i8p, u16p)
        _decl(L, "qor_tq35_quantize", None, f32p, C.c_int, u8p)
        _decl(L, "qor_tq35_unpack", None, u8p, u8p, u16p, u16p)
        _decl(L, "qor_q4g32_quantize", None, f32p, C.c_int, u8p, u16p, u16p)
        _decl(L, "qor_tile_bytes", C.c_size_t, C.c_int)
        _decl(L, "qor_tile_store", None, C.c_int, u8p, C.c_int, f32p, f32p)
        _decl(L, "qor_tile_dequant", C.c_float, C.c_int, u8p, C.c_int, C.c_int, C.c_int)
        _decl(L, "qor_linear_attention_decode", None, f32p, C.c_int, C.c_int, f32p, f32p, f32p, C.c_float, f32p)
        _decl(L, "qor_tile_load", None, C.c_int, u8p, C.c_int, C.c_int, i16p, f32p)
        _decl(L, "qor_pool_init", C.c_int, C.POINTER(QorPool), C.c_int, C.c_int, C.c_int,
              C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64)
        _decl(L, "qor_pool_init_ex", C.c_int, C.POINTER(QorPool), C.c_int, C.c_int, C.c_int,
              C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_int)
        _decl(L, "qor_pool_fill_synthetic", C.c_int, C.POINTER(QorPool), C.c_int, C.c_int, C.c_int,
              C.c_int, C.c_int, C.c_uint64, u8p)
        _decl(L, "qor_pool_free", None, C.POINTER(QorPool))
        _decl(L, "qor_pool_append", C.c_int, C.POINTER(QorPool), C.c_int, i32p, i32p)
        _decl(L, "qor_pool_write_token", C.c_int, C.POINTER(QorPool), C.c_int, C.c_int,
              C.c_int, f32p, f32p)
        _decl(L, "qor_pool_attention", None, C.POINTER(QorPool), C.c_int, C.c_int, C.c_int,
              f32p, C.c_int, C.c_float, f32p, f32p)
        _decl(L, "qor_partial_attention", None, C.POINTER(QorPool), C.c_int, C.c_int, C.c_int,
              C.c_int, f32p, C.c_int, C.c_float, f32p, f32p, f32p)
        _decl(L, "qor_merge_partials", None, C.c_int, C.c_int, f32p, f32p, f32p, f32p)
        _decl(L, "qor_vtoken_init", C.c_int, C.POINTER(EvictionPool), C.c_uint32, C.c_uint32,
              C.c_float)
        _decl(L, "qor_vtoken_insert", C.c_int, C.POINTER(EvictionPool), C.c_uint32, C.c_float,
              C.POINTER(C.c_uint32))
        _decl(L, "qor_vtoken_update_scores", None, C.POINTER(EvictionPool), f32p, C.c_uint32,
              C.c_int)
        _decl(L, "qor_vtoken_prune", C.c_uint32, C.POINTER(EvictionPool), C.c_uint32)
        _decl(L, "qor_vtoken_waste_pct", C.c_float, C.POINTER(EvictionPool))
        _decl(L, "qor_pool_evict", C.c_int, C.POINTER(QorPool), C.c_int, i32p, f32p, u8p, C.c_int)
        _decl(L, "qor_evict_trigger", C.c_int, C.c_uint64, C.c_uint32, C.c_uint32, C.c_double)
        _lib = L
    return _lib


def ref():
    """The reference's CPU library (oracle/_ref), or None when not built."""
    global _ref, _ref_tried
    if _ref is None and not _ref_tried:
        _ref_tried = True
        if os.path.exists(REF_SO):
            R = C.CDLL(REF_SO)
            _decl(R, "qwn_q8_cache_init", C.c_int, C.POINTER(RefQ8Cache), C.c_int, C.c_int, C.c_int)
            _decl(R, "qwn_q8_cache_free", None, C.POINTER(RefQ8Cache))
            _decl(R, "qwn_q8_cache_reset", None, C.POINTER(RefQ8Cache))
            _decl(R, "qwn_q8_cache_append", C.c_int, C.POINTER(RefQ8Cache), f32p, f32p, C.c_int)
            _decl(R, "qwn_q8_cache_attention_head", None, f32p, C.POINTER(RefQ8Cache), C.c_int,
                  C.c_int, C.c_float, f32p, f32p)
            _decl(R, "qwn_turboquant_init", C.c_int, C.POINTER(RefTQCache), C.c_int, C.c_int, C.c_int)
            _decl(R, "qwn_turboquant_free", None, C.POINTER(RefTQCache))
            _decl(R, "qwn_turboquant_quantize_token", None, f32p, u8p, C.c_int)
            _decl(R, "qwn_turboquant_attention_head", None, f32p, C.POINTER(RefTQCache), C.c_int,
                  C.c_int, C.c_int, C.c_int, C.c_float, f32p, f32p)
            _decl(R, "qwn_kv_cache_contract_init", None, C.POINTER(KvContract), C.c_int, C.c_uint32)
            _decl(R, "qwn_kv_cache_mode_parse", C.c_int, C.c_char_p, C.POINTER(C.c_int))
            _decl(R, "qwn_kv_pool_init", C.c_int, C.POINTER(RefBlockPool), C.c_int, C.c_int,
                  C.c_int, C.c_int)
            _decl(R, "qwn_kv_pool_free", None, C.POINTER(RefBlockPool))
            _decl(R, "qwn_kv_pool_free_block", None, C.POINTER(RefBlockPool), C.c_int)
            _decl(R, "qwn_block_table_init", C.c_int, C.POINTER(RefBlockTable), C.c_int, C.c_int)
            _decl(R, "qwn_block_table_append_token", C.c_int, C.POINTER(RefBlockPool),
                  C.POINTER(RefBlockTable))
            _decl(R, "qwn_block_table_free", None, C.POINTER(RefBlockPool), C.POINTER(RefBlockTable))
            _decl(R, "qwn_paged_eviction_init", C.c_int, C.POINTER(EvictionPool), C.c_uint32,
                  C.c_uint32, C.c_float)
            _decl(R, "qwn_paged_eviction_insert", C.c_int, C.POINTER(EvictionPool), C.c_uint32,
                  C.c_float, C.POINTER(C.c_uint32))
            _decl(R, "qwn_paged_eviction_update_scores", None, C.POINTER(EvictionPool), f32p,
                  C.c_uint32)
            _decl(R, "qwn_paged_eviction_prune", C.c_uint32, C.POINTER(EvictionPool), C.c_uint32)
            _decl(R, "qwn_paged_eviction_memory_waste_pct", C.c_float, C.POINTER(EvictionPool))
            _decl(R, "qref_batch_create", C.c_void_p, C.c_int, C.c_int, i32p, C.c_int, C.c_int,
                  C.c_int, C.c_int, C.c_int, C.c_uint64)
            _decl(R, "qref_batch_step", C.c_int, C.c_void_p, C.c_int)
            _decl(R, "qref_batch_ctx", f32p, C.c_void_p)
            _decl(R, "qref_batch_destroy", None, C.c_void_p)
            _decl(R, "qref_max_threads", C.c_int)
            _decl(R, "qref_set_threads", None, C.c_int)
            _decl(R, "qwanto_linear_attention_init", C.c_int, C.POINTER(RefLinearState), C.c_int, C.c_int)
            _decl(R, "qwanto_linear_attention_destroy", None, C.POINTER(RefLinearState))
            _decl(R, "qwanto_linear_attention_decode", None, C.POINTER(RefLinearState), f32p, f32p, f32p,
                  C.c_float, f32p)
            _decl(R, "qwanto_linear_attention_prefill", None, C.POINTER(RefLinearState), f32p, f32p, f32p,
                  C.c_float, C.c_int, f32p)
            _decl(R, "qref_f16_write", C.c_int, f32p, f32p, C.c_int, C.c_int, C.POINTER(C.c_uint16),
                  C.POINTER(C.c_uint16))
            _ref = R
    return _ref


# ---------------------------------------------------------------------------
# numpy conveniences
# ---------------------------------------------------------------------------

def stream(kind: int, seq: int, layer: int) -> int:
    return int(lib().qor_stream(kind, seq, layer))


def normal(seed: int, strm: int, first: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().qor_fill_normal(seed, strm, first, _ptr(out, f32p), n)
    return out


def gen_row(seed: int, kind: int, seq: int, layer: int, pos: int, width: int) -> np.ndarray:
    """Row `pos` of tensor kind (1=Q, 2=K, 3=V): the same values the device
    generator and the reference shim produce."""
    return normal(seed, stream(kind, seq, layer), pos * width, width)


def free_stack(seed: int, total: int) -> np.ndarray:
    s = np.empty(total, dtype=np.int32)
    lib().qor_permuted_free_stack(seed, total, _ptr(s, i32p))
    return s


def outlier_mask(seed: int, layer: int, channels: int, count: int) -> np.ndarray:
    m = np.zeros(channels, dtype=np.uint8)
    lib().qor_outlier_channels(seed, layer, channels, count, _ptr(m, u8p))
    return m


def q8_b64(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    codes = np.zeros(n, dtype=np.int8)
    scales = np.zeros((n + 63) // 64, dtype=np.float32)
    lib().qor_q8_b64_quantize(_ptr(x, f32p), n, _ptr(codes, i8p), _ptr(scales, f32p))
    return codes, scales


def q8_head(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(x.size, dtype=np.int8)
    s = np.zeros(1, dtype=np.uint16)
    lib().qor_q8_head_quantize(_ptr(x, f32p), x.size, _ptr(codes, i8p), _ptr(s, u16p))
    return codes, int(s[0])


def tq35(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(((x.size + 63) // 64) * 32, dtype=np.uint8)
    lib().qor_tq35_quantize(_ptr(x, f32p), x.size, _ptr(out, u8p))
    return out


def q4g32(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    g = (n + 31) // 32
    codes = np.zeros(n, dtype=np.uint8)
    r = np.zeros(g, dtype=np.uint16)
    m = np.zeros(g, dtype=np.uint16)
    lib().qor_q4g32_quantize(_ptr(x, f32p), n, _ptr(codes, u8p), _ptr(r, u16p), _ptr(m, u16p))
    return codes, r, m


def f16_rne(x: float) -> int:
    return int(lib().qor_f32_to_f16_rne(x))


def tile_load(codec: int, tile: np.ndarray, t: int, is_value: int):
    tile = np.ascontiguousarray(tile, dtype=np.uint8)
    codes = np.zeros(128, dtype=np.int16)
    params = np.zeros(8, dtype=np.float32)
    lib().qor_tile_load(codec, _ptr(tile, u8p), t, is_value, _ptr(codes, i16p), _ptr(params, f32p))
    return codes, params


class Pool:
    """Host simulation of the paged pool (page tables, free stack, tiles)."""

    def __init__(self, codec, layers, kv_heads, page_tokens, total_pages, max_seqs,
                 max_pages_per_seq, perm_seed=0, with_pages=True):
        self.p = QorPool()
        rc = lib().qor_pool_init_ex(C.byref(self.p), codec, layers, kv_heads, page_tokens,
                                    total_pages, max_seqs, max_pages_per_seq, perm_seed,
                                    1 if with_pages else 0)
        if rc != 0:
            raise MemoryError("oracle pool init failed")
        self.codec, self.layers, self.kv_heads = codec, layers, kv_heads
        self.page_tokens, self.max_seqs, self.mp = page_tokens, max_seqs, max_pages_per_seq

    def __del__(self):
        try:
            lib().qor_pool_free(C.byref(self.p))
        except Exception:
            pass

    def append(self, seq_ids, counts) -> int:
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        c = np.ascontiguousarray(counts, dtype=np.int32)
        return int(lib().qor_pool_append(C.byref(self.p), s.size, _ptr(s, i32p), _ptr(c, i32p)))

    def write(self, seq, layer, pos, k, v) -> int:
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        return int(lib().qor_pool_write_token(C.byref(self.p), seq, layer, pos,
                                              _ptr(k, f32p), _ptr(v, f32p)))

    def fill_synthetic(self, seq, layer, gen_layer, first, last, seed, k_outlier_mask=None) -> int:
        """Store the synthetic K/V rows of (seed, seq, gen_layer) for
        positions [first, last) into `layer`, in C."""
        m = None if k_outlier_mask is None else np.ascontiguousarray(k_outlier_mask, dtype=np.uint8)
        return int(lib().qor_pool_fill_synthetic(C.byref(self.p), seq, layer, gen_layer, first, last, seed,
                                                 None if m is None else _ptr(m, u8p)))

    def attention(self, seq, layer, length, q, heads, scale, want_probs=False):
        q = np.ascontiguousarray(q, dtype=np.float32)
        out = np.zeros((heads, 128), dtype=np.float32)
        probs = np.zeros((heads, max(length, 1)), dtype=np.float32) if want_probs else None
        lib().qor_pool_attention(C.byref(self.p), seq, layer, length, _ptr(q, f32p), heads,
                                 scale, _ptr(out, f32p),
                                 _ptr(probs, f32p) if want_probs else None)
        return (out, probs) if want_probs else out

    def evict(self, seq_ids, mass, flags, budget) -> int:
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        m = np.ascontiguousarray(mass, dtype=np.float32)
        f = np.ascontiguousarray(flags, dtype=np.uint8)
        return int(lib().qor_pool_evict(C.byref(self.p), s.size, _ptr(s, i32p), _ptr(m, f32p),
                                        _ptr(f, u8p), budget))

    # views
    def pages(self) -> np.ndarray:
        if not self.p.pages:
            raise ValueError("metadata-only oracle pool has no pages")
        n = self.p.total_pages * self.p.page_bytes
        return np.ctypeslib.as_array(self.p.pages, shape=(n,)).reshape(self.p.total_pages, -1)

    def page_table(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.p.page_table, shape=(self.max_seqs * self.mp,)).reshape(
            self.max_seqs, self.mp)

    def lens(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.p.lens, shape=(self.max_seqs,))

    def npages(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.p.npages, shape=(self.max_seqs,))

    def scores(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.p.page_score, shape=(self.max_seqs * self.mp,)).reshape(
            self.max_seqs, self.mp)

    def free_stack(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.p.free_stack, shape=(self.p.total_pages,))[: self.p.free_top]

    def tile(self, seq, layer, kv_head, pos) -> np.ndarray:
        P = self.page_tokens
        pg = int(self.page_table()[seq, pos // P])
        tb = self.p.tile_bytes
        off = (((layer * self.kv_heads) + kv_head) * (P // 16) + (pos % P) // 16) * tb
        return self.pages()[pg, off: off + tb]
