"""Parity of the reference-named C APIs (served by qwn_cuda.so on the GPU)
with the reference's own CPU library (oracle/_ref/libqwnref.so, compiled from
c/qwn_paged_kv.c, c/qwanto_turboquant.c and c/qwanto_attention.c), both
driven through ctypes on the same inputs and the same structs.

Bit-exact: Q8 codes and scales (qwn_q8_cache_append), TurboQuant blocks
(qwn_turboquant_quantize_token), fp16 pool bytes (qwn_paged_kv_write),
linear-attention states and outputs.  Attention heads, dot products and
value accumulations within |d| <= 1e-4 + 1e-3 |ref|.  Inputs include NaN,
+-Inf, +-0, subnormals, constant rows and partial 64-blocks.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from kvharness import assert_close

pytestmark = pytest.mark.gpu

f32p = C.POINTER(C.c_float)
u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)


def _decl(L, name, res, *args):
    f = getattr(L, name)
    f.restype, f.argtypes = res, list(args)


@pytest.fixture(scope="module")
def libs(cuda, oracle_mod, ref_lib):
    import qwanto_b200
    O = oracle_mod
    out = []
    for L in (qwanto_b200.lib(), ref_lib):
        Q8, TQ, BP, BT, LS = (C.POINTER(O.RefQ8Cache), C.POINTER(O.RefTQCache), C.POINTER(O.RefBlockPool),
                              C.POINTER(O.RefBlockTable), C.POINTER(O.RefLinearState))
        _decl(L, "qwn_q8_cache_init", C.c_int, Q8, C.c_int, C.c_int, C.c_int)
        _decl(L, "qwn_q8_cache_free", None, Q8)
        _decl(L, "qwn_q8_cache_append", C.c_int, Q8, f32p, f32p, C.c_int)
        _decl(L, "qwn_q8_cache_dot_key_scalar", C.c_float, Q8, C.c_int, C.c_int, f32p, C.c_int)
        _decl(L, "qwn_q8_cache_accum_value_scalar", None, Q8, C.c_int, C.c_int, C.c_float, f32p, C.c_int)
        _decl(L, "qwn_q8_cache_attention_head", None, f32p, Q8, C.c_int, C.c_int, C.c_float, f32p, f32p)
        _decl(L, "qwn_turboquant_init", C.c_int, TQ, C.c_int, C.c_int, C.c_int)
        _decl(L, "qwn_turboquant_free", None, TQ)
        _decl(L, "qwn_turboquant_quantize_token", None, f32p, u8p, C.c_int)
        _decl(L, "qwn_turboquant_dot_key_scalar", C.c_float, f32p, u8p, C.c_int)
        _decl(L, "qwn_turboquant_dot_key_avx2", C.c_float, f32p, u8p, C.c_int)
        _decl(L, "qwn_turboquant_accum_value_scalar", None, C.c_float, u8p, f32p, C.c_int)
        _decl(L, "qwn_turboquant_attention_head", None, f32p, TQ, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
              f32p, f32p)
        _decl(L, "qwn_turboquant_matmul_avx512", None, TQ, f32p, f32p, C.c_int, C.c_int)
        _decl(L, "qwn_kv_pool_init", C.c_int, BP, C.c_int, C.c_int, C.c_int, C.c_int)
        _decl(L, "qwn_kv_pool_free", None, BP)
        _decl(L, "qwn_block_table_init", C.c_int, BT, C.c_int, C.c_int)
        _decl(L, "qwn_block_table_append_token", C.c_int, BP, BT)
        _decl(L, "qwn_block_table_free", None, BP, BT)
        _decl(L, "qwn_paged_kv_write", C.c_int, BP, BT, C.c_int, C.c_int, f32p, f32p)
        _decl(L, "qwn_paged_attention_head", None, BP, BT, C.c_int, C.c_int, C.c_int, f32p, f32p, f32p)
        _decl(L, "qwn_paged_attention_gather_head", None, BP, BT, C.c_int, C.c_int, C.c_int, f32p, u16p, u16p,
              f32p, f32p)
        _decl(L, "qwanto_linear_attention_init", C.c_int, LS, C.c_int, C.c_int)
        _decl(L, "qwanto_linear_attention_reset", None, LS)
        _decl(L, "qwanto_linear_attention_destroy", None, LS)
        _decl(L, "qwanto_linear_attention_decode", None, LS, f32p, f32p, f32p, C.c_float, f32p)
        _decl(L, "qwanto_linear_attention_prefill", None, LS, f32p, f32p, f32p, C.c_float, C.c_int, f32p)
        out.append(L)
    return out


def P(a, t=f32p):
    return a.ctypes.data_as(t)


def _rows(rng, n, count):
    """count rows of n fp32 values: normal, scaled, and special-value rows."""
    out = []
    for i in range(count):
        x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 30.0])).astype(np.float32)
        kind = i % 6
        if kind == 1:
            x[rng.integers(0, n, 3)] = np.float32(np.nan)
            x[rng.integers(0, n)] = np.float32(np.inf)
            x[rng.integers(0, n)] = np.float32(-np.inf)
        elif kind == 2:
            x[:] = np.float32(0.75)                      # constant: zero range
        elif kind == 3:
            x[::3] = np.float32(0.0)
            x[1::7] = np.float32(-0.0)
            x[2::11] = np.float32(1e-41)                  # fp32 subnormal
        elif kind == 4:
            x[0] = np.float32(np.nan)                     # first element NaN
        elif kind == 5:
            x = (x * np.float32(1e-9)).astype(np.float32)  # range below 1e-8
        out.append(np.ascontiguousarray(x))
    return out


@pytest.mark.parametrize("heads,hd", [(2, 65), (2, 128), (8, 128), (1, 100)])
def test_q8_cache_bit_exact_and_attention(oracle_mod, libs, heads, hd):
    """qwn_q8_cache_append codes and scales bit-exact (partial 64-blocks
    included), then dot/accumulate helpers and attention heads against
    c/qwanto_turboquant.c:648-705."""
    O = oracle_mod
    rng = np.random.default_rng(heads * 1000 + hd)
    n, T = heads * hd, 37
    caches = [O.RefQ8Cache(), O.RefQ8Cache()]
    for L, c in zip(libs, caches):
        assert L.qwn_q8_cache_init(C.byref(c), 64, heads, hd) == 0
    try:
        ks, vs = _rows(rng, n, T), _rows(rng, n, T)
        for t in range(T):
            for L, c in zip(libs, caches):
                assert L.qwn_q8_cache_append(C.byref(c), P(ks[t]), P(vs[t]), n) == 0
        sb = caches[0].scale_stride
        for f, shape in (("packed_k", (T, n)), ("packed_v", (T, n))):
            a = np.ctypeslib.as_array(getattr(caches[0], f), shape=(64 * n,)).reshape(64, n)[:T]
            b = np.ctypeslib.as_array(getattr(caches[1], f), shape=(64 * n,)).reshape(64, n)[:T]
            assert np.array_equal(a, b), f
        for f in ("scales_k", "scales_v"):
            a = np.ctypeslib.as_array(getattr(caches[0], f), shape=(64 * sb,))[: T * sb]
            b = np.ctypeslib.as_array(getattr(caches[1], f), shape=(64 * sb,))[: T * sb]
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f
        q = np.ascontiguousarray(rng.standard_normal(hd).astype(np.float32))
        for kv in range(heads):
            for t in (0, 5, T - 1):
                d = [L.qwn_q8_cache_dot_key_scalar(C.byref(c), t, kv * hd, P(q), hd) for L, c in zip(libs, caches)]
                assert_close(d[0], d[1], "q8 dot") if np.isfinite(d[1]) else None
                ctx = [np.full(hd, 0.5, np.float32) for _ in range(2)]
                for L, c, x in zip(libs, caches, ctx):
                    L.qwn_q8_cache_accum_value_scalar(C.byref(c), t, kv * hd, 0.3, P(x), hd)
                assert_close(ctx[0], ctx[1], "q8 accumulate")
            for pos in (0, 11, T - 1):
                res = []
                for L, c in zip(libs, caches):
                    sc = np.zeros(64, np.float32)
                    out = np.zeros(hd, np.float32)
                    L.qwn_q8_cache_attention_head(P(q), C.byref(c), kv, pos, 0.09, P(sc), P(out))
                    res.append((sc[: pos + 1].copy(), out))
                if np.all(np.isfinite(res[1][1])):
                    assert_close(res[0][1], res[1][1], f"q8 head kv{kv} pos{pos}")
                    assert_close(res[0][0], res[1][0], f"q8 head exps kv{kv} pos{pos}")
    finally:
        for L, c in zip(libs, caches):
            L.qwn_q8_cache_free(C.byref(c))


@pytest.mark.parametrize("dim", [64, 100, 128, 130, 1024])
def test_turboquant_quantize_bit_exact(oracle_mod, libs, dim):
    """qwn_turboquant_quantize_token into host buffers: every byte of every
    32-byte block equals c/qwanto_turboquant.c:162-213's, special values and
    a partial last group included; the dot/accumulate helpers agree."""
    rng = np.random.default_rng(dim)
    nb = (dim + 63) // 64
    for x in _rows(rng, dim, 24):
        outs = [np.zeros(nb * 32, np.uint8) for _ in range(2)]
        for L, o in zip(libs, outs):
            L.qwn_turboquant_quantize_token(P(x), P(o, u8p), dim)
        assert np.array_equal(outs[0], outs[1]), np.nonzero(outs[0] != outs[1])[0][:10]
        if not np.all(np.isfinite(x)):
            continue
        q = np.ascontiguousarray(rng.standard_normal(dim).astype(np.float32))
        d = [L.qwn_turboquant_dot_key_scalar(P(q), P(outs[1], u8p), dim) for L in libs]
        assert abs(d[0] - d[1]) <= 1e-3 + 1e-4 * abs(d[1])   # c/tests/test_turboquant.c:91
        assert libs[0].qwn_turboquant_dot_key_avx2(P(q), P(outs[1], u8p), dim) == d[0]
        ctx = [np.zeros(dim, np.float32) for _ in range(2)]
        for L, c in zip(libs, ctx):
            L.qwn_turboquant_accum_value_scalar(0.723, P(outs[1], u8p), P(c), dim)
        assert np.abs(ctx[0] - ctx[1]).max() < 1e-3


@pytest.mark.parametrize("heads,hd", [(4, 128), (2, 192)])
def test_turboquant_cache_and_attention(oracle_mod, libs, heads, hd):
    """Tokens quantized into each library's own cache (managed memory here),
    caches byte-equal, attention heads and the matmul helper within
    tolerance of c/qwanto_turboquant.c:707-792."""
    O = oracle_mod
    rng = np.random.default_rng(hd)
    T = 300
    caches = [O.RefTQCache(), O.RefTQCache()]
    for L, c in zip(libs, caches):
        assert L.qwn_turboquant_init(C.byref(c), T, heads, hd) == 0
    try:
        bph = (hd + 63) // 64
        for t in range(T):
            for h in range(heads):
                k = rng.standard_normal(hd).astype(np.float32)
                v = rng.standard_normal(hd).astype(np.float32)
                for L, c in zip(libs, caches):
                    off = t * c.token_stride_k + h * bph * 32
                    L.qwn_turboquant_quantize_token(P(k), C.cast(C.addressof(c.packed_k.contents) + off, u8p), hd)
                    L.qwn_turboquant_quantize_token(P(v), C.cast(C.addressof(c.packed_v.contents) + off, u8p), hd)
        size = T * caches[0].token_stride_k
        for f in ("packed_k", "packed_v"):
            assert np.array_equal(np.ctypeslib.as_array(getattr(caches[0], f), shape=(size,)),
                                  np.ctypeslib.as_array(getattr(caches[1], f), shape=(size,))), f
        q = np.ascontiguousarray(rng.standard_normal(heads * hd).astype(np.float32))
        for kv in range(heads):
            for pos in (0, 63, T - 1):
                res = []
                for L, c in zip(libs, caches):
                    sc = np.zeros(T, np.float32)
                    out = np.zeros(hd, np.float32)
                    L.qwn_turboquant_attention_head(P(q[kv * hd:]), C.byref(c), 0, kv, kv, pos, 1 / np.sqrt(hd),
                                                    P(sc), P(out))
                    res.append((sc[: pos + 1].copy(), out))
                assert_close(res[0][1], res[1][1], f"tq head kv{kv} pos{pos}")
                assert_close(res[0][0], res[1][0], f"tq probabilities kv{kv} pos{pos}")
        outs = [np.full(heads * hd, 7.0, np.float32) for _ in range(2)]
        for L, c, o in zip(libs, caches, outs):
            L.qwn_turboquant_matmul_avx512(C.byref(c), P(q), P(o), heads, hd)
        assert_close(outs[0], outs[1], "tq matmul")
    finally:
        for L, c in zip(libs, caches):
            L.qwn_turboquant_free(C.byref(c))


@pytest.mark.parametrize("layers,heads,hd", [(2, 2, 128), (3, 4, 100), (1, 8, 64)])
def test_paged_fp16_pool_bit_exact_and_attention(oracle_mod, libs, layers, heads, hd):
    """qwn_kv_pool_init + block tables + qwn_paged_kv_write: the managed pool
    bytes equal c/qwn_paged_kv.c:151-198's (F16C round to nearest even, the
    truncating scalar tail for head_dim % 8, NaN/Inf/subnormals); both
    attention calls within tolerance, probabilities included."""
    O = oracle_mod
    rng = np.random.default_rng(layers * 100 + hd)
    blocks, T = 40, 150
    pools, tabs = [O.RefBlockPool(), O.RefBlockPool()], [O.RefBlockTable(), O.RefBlockTable()]
    for L, p, t in zip(libs, pools, tabs):
        assert L.qwn_kv_pool_init(C.byref(p), blocks, layers, heads, hd) == 0
        assert L.qwn_block_table_init(C.byref(t), 0, 2) == 0
    try:
        n = heads * hd
        for pos in range(T):
            for L, p, t in zip(libs, pools, tabs):
                assert L.qwn_block_table_append_token(C.byref(p), C.byref(t)) == 0
            for layer in range(layers):
                k = rng.standard_normal(n).astype(np.float32)
                v = rng.standard_normal(n).astype(np.float32)
                if pos % 17 == 3:
                    k[:4] = [np.nan, np.inf, -np.inf, 3e-7]
                    v[-3:] = [1e-6, 70000.0, -0.0]
                for L, p, t in zip(libs, pools, tabs):
                    assert L.qwn_paged_kv_write(C.byref(p), C.byref(t), layer, pos, P(k), P(v)) == 0
        size = blocks * pools[0].block_bytes // 2
        for f in ("key_data", "val_data"):
            a = np.ctypeslib.as_array(getattr(pools[0], f), shape=(size,))
            b = np.ctypeslib.as_array(getattr(pools[1], f), shape=(size,))
            assert np.array_equal(a, b), f"{f}: {int((a != b).sum())} fp16 values differ"
        # attention over clean tokens: rewrite the special-valued ones
        for pos in range(T):
            if pos % 17 == 3:
                for layer in range(layers):
                    k = rng.standard_normal(n).astype(np.float32)
                    v = rng.standard_normal(n).astype(np.float32)
                    for L, p, t in zip(libs, pools, tabs):
                        L.qwn_paged_kv_write(C.byref(p), C.byref(t), layer, pos, P(k), P(v))
        q = np.ascontiguousarray(rng.standard_normal(hd).astype(np.float32))
        for layer in range(layers):
            for kv in range(heads):
                res = []
                for i, (L, p, t) in enumerate(zip(libs, pools, tabs)):
                    sc, out = np.zeros(T, np.float32), np.zeros(hd, np.float32)
                    if (layer + kv) % 2:
                        L.qwn_paged_attention_head(C.byref(p), C.byref(t), layer, kv, kv, P(q), P(sc), P(out))
                    else:
                        gk, gv = np.zeros(T * hd + 16 * hd, np.uint16), np.zeros(T * hd + 16 * hd, np.uint16)
                        L.qwn_paged_attention_gather_head(C.byref(p), C.byref(t), layer, kv, kv, P(q), P(gk, u16p),
                                                          P(gv, u16p), P(sc), P(out))
                    res.append((sc, out))
                assert_close(res[0][1], res[1][1], f"paged head layer{layer} kv{kv}")
                assert_close(res[0][0], res[1][0], f"paged probabilities layer{layer} kv{kv}")
    finally:
        for L, p, t in zip(libs, pools, tabs):
            L.qwn_block_table_free(C.byref(p), C.byref(t))
            L.qwn_kv_pool_free(C.byref(p))


@pytest.mark.parametrize("heads,d", [(8, 64), (3, 128), (2, 40)])
def test_linear_attention_reference_api_bit_exact(oracle_mod, libs, heads, d):
    """qwanto_linear_attention_* on the GPU: states and outputs bit-identical
    to c/qwanto_attention.c (AVX2/AVX-512 order) over decode and prefill,
    the state read on the host through the struct's pointer."""
    O = oracle_mod
    rng = np.random.default_rng(d)
    sts = [O.RefLinearState(), O.RefLinearState()]
    for L, s in zip(libs, sts):
        assert L.qwanto_linear_attention_init(C.byref(s), heads, d) == 0
    try:
        n = heads * d
        for step in range(5):
            q, k, v = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
            outs = [np.zeros(n, np.float32) for _ in range(2)]
            for L, s, o in zip(libs, sts, outs):
                L.qwanto_linear_attention_decode(C.byref(s), P(q), P(k), P(v), 0.93, P(o))
            assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), f"decode step {step}"
        S = 17
        q, k, v = (rng.standard_normal(S * n).astype(np.float32) for _ in range(3))
        outs = [np.zeros(S * n, np.float32) for _ in range(2)]
        for L, s, o in zip(libs, sts, outs):
            L.qwanto_linear_attention_prefill(C.byref(s), P(q), P(k), P(v), 0.8, S, P(o))
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), "prefill"
        a = np.ctypeslib.as_array(sts[0].state, shape=(heads * d * d,))
        b = np.ctypeslib.as_array(sts[1].state, shape=(heads * d * d,))
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), "state"
        libs[0].qwanto_linear_attention_reset(C.byref(sts[0]))
        assert not np.ctypeslib.as_array(sts[0].state, shape=(heads * d * d,)).any()
    finally:
        for L, s in zip(libs, sts):
            L.qwanto_linear_attention_destroy(C.byref(s))
        assert not sts[0].state
