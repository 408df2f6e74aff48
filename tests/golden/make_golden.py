"""Generate golden vectors by running the reference's own CPU code.

Run in the build container (needs oracle/_ref, compiled from the reference
sources by oracle/Makefile):  python tests/golden/make_golden.py

Inputs follow the reference tests that pin this path:
  * c/tests/test_kv_cache.c:29-59 -- analytic Q8 inputs key[i]=(i-65)*0.03125,
    value[i]=sinf(0.07i), query[i]=cosf(0.03i), 2 heads x 65 channels, then
    a NaN/Inf row;
  * c/tests/test_turboquant.c:27-58, :206-232 -- dims {64..512} x five
    rand()-seeded distributions, seeds 5000+it*100+id*10+ids (glibc rand(),
    float arithmetic without contraction);
  * c/tests/test_nextgen_suite.c:138-177 -- vToken insert/update/prune;
  * the block table of c/qwn_paged_kv.c:115-138 under a sequence of appends.
Outputs are what the reference functions return for those inputs.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402

libc = C.CDLL("libc.so.6")
libm = C.CDLL("libm.so.6")
libm.sinf.restype = C.c_float
libm.sinf.argtypes = [C.c_float]
libm.cosf.restype = C.c_float
libm.cosf.argtypes = [C.c_float]
f32 = np.float32
RAND_MAX = f32(2147483647)


def kv_cache_inputs():
    key = np.array([f32(i - 65) * f32(0.03125) for i in range(130)], dtype=np.float32)
    value = np.array([libm.sinf(float(f32(i) * f32(0.07))) for i in range(130)], dtype=np.float32)
    query = np.array([libm.cosf(float(f32(i) * f32(0.03))) for i in range(65)], dtype=np.float32)
    return key, value, query


def synthetic(n, dist, seed):
    """generate_synthetic_data of c/tests/test_turboquant.c:27-58 (no contraction)."""
    libc.srand(seed)
    out = np.zeros(n, dtype=np.float32)
    for i in range(n):
        if dist == 0:
            out[i] = f32(f32(libc.rand()) / RAND_MAX) * f32(2.0) - f32(1.0)
        elif dist == 1:
            s = f32(0.0)
            for _ in range(12):
                s = f32(s + f32(f32(libc.rand()) / RAND_MAX))
            out[i] = f32(s - f32(6.0)) * f32(0.5)
        elif dist == 2:
            if libc.rand() % 10 == 0:
                out[i] = f32(f32(f32(libc.rand()) / RAND_MAX) * f32(2.0) - f32(1.0)) * f32(15.0)
            else:
                out[i] = f32(f32(libc.rand()) / RAND_MAX) * f32(0.2) - f32(0.1)
        elif dist == 3:
            out[i] = f32(0.01) + f32(f32(libc.rand()) / RAND_MAX) * f32(4.99)
        elif dist == 4:
            out[i] = f32(f32(f32(libc.rand()) / RAND_MAX) * f32(2.0) - f32(1.0)) * f32(0.01)
    return out


def ref_q8(R, x, n_heads, head_dim):
    c = O.RefQ8Cache()
    assert R.qwn_q8_cache_init(C.byref(c), 4, n_heads, head_dim) == 0
    n = x.size
    assert R.qwn_q8_cache_append(C.byref(c), O._ptr(x, O.f32p), O._ptr(x, O.f32p), n) == 0
    codes = np.ctypeslib.as_array(c.packed_k, shape=(n,)).copy()
    scales = np.ctypeslib.as_array(c.scales_k, shape=((n + 63) // 64,)).copy()
    R.qwn_q8_cache_free(C.byref(c))
    return codes, scales


def main():
    R = O.ref()
    if R is None:
        raise SystemExit("oracle/_ref not built (make -C oracle ref)")
    out = {}
    # --- c/tests/test_kv_cache.c ------------------------------------------
    key, value, query = kv_cache_inputs()
    c = O.RefQ8Cache()
    assert R.qwn_q8_cache_init(C.byref(c), 16, 2, 65) == 0
    assert R.qwn_q8_cache_append(C.byref(c), O._ptr(key, O.f32p), O._ptr(value, O.f32p), 130) == 0
    out["kv_key"], out["kv_value"], out["kv_query"] = key, value, query
    out["kv_codes_k"] = np.ctypeslib.as_array(c.packed_k, shape=(130,)).copy()
    out["kv_scales_k"] = np.ctypeslib.as_array(c.scales_k, shape=(3,)).copy()
    out["kv_codes_v"] = np.ctypeslib.as_array(c.packed_v, shape=(130,)).copy()
    out["kv_scales_v"] = np.ctypeslib.as_array(c.scales_v, shape=(3,)).copy()
    scores = np.zeros(16, np.float32)
    ctx = np.zeros(65, np.float32)
    R.qwn_q8_cache_attention_head(O._ptr(query, O.f32p), C.byref(c), 0, 0, C.c_float(1.0),
                                  O._ptr(scores, O.f32p), O._ptr(ctx, O.f32p))
    out["kv_attention_ctx"] = ctx.copy()
    R.qwn_q8_cache_reset(C.byref(c))
    key2, value2 = key.copy(), value.copy()
    key2[0], key2[1], value2[0], value2[1] = np.nan, np.inf, -np.inf, np.nan
    assert R.qwn_q8_cache_append(C.byref(c), O._ptr(key2, O.f32p), O._ptr(value2, O.f32p), 130) == 0
    out["kv_nan_key"], out["kv_nan_value"] = key2, value2
    out["kv_nan_codes_k"] = np.ctypeslib.as_array(c.packed_k, shape=(130,)).copy()
    out["kv_nan_scales_k"] = np.ctypeslib.as_array(c.scales_k, shape=(3,)).copy()
    out["kv_nan_codes_v"] = np.ctypeslib.as_array(c.packed_v, shape=(130,)).copy()
    out["kv_nan_scales_v"] = np.ctypeslib.as_array(c.scales_v, shape=(3,)).copy()
    R.qwn_q8_cache_free(C.byref(c))

    # --- c/tests/test_turboquant.c (first iteration: it = 0) ----------------
    dims = [64, 128, 192, 256, 320, 512]
    tq_inputs, tq_blocks, q8_codes, q8_scales = [], [], [], []
    for idd, dim in enumerate(dims):
        for dist in range(5):
            seed = 5000 + idd * 10 + dist
            k = synthetic(dim, dist, seed + 100)
            blk = np.zeros(((dim + 63) // 64) * 32, np.uint8)
            R.qwn_turboquant_quantize_token(O._ptr(k, O.f32p), O._ptr(blk, O.u8p), dim)
            tq_inputs.append(k)
            tq_blocks.append(blk)
            cds, scs = ref_q8(R, k, 1, dim)
            q8_codes.append(cds)
            q8_scales.append(scs)
    out["tq_inputs"] = np.concatenate(tq_inputs)
    out["tq_blocks"] = np.concatenate(tq_blocks)
    out["tq_q8_codes"] = np.concatenate(q8_codes)
    out["tq_q8_scales"] = np.concatenate(q8_scales)
    out["tq_dims"] = np.array([d for d in dims for _ in range(5)], np.int32)

    # --- block table under appends (c/qwn_paged_kv.c) ----------------------
    pool = O.RefBlockPool()
    assert R.qwn_kv_pool_init(C.byref(pool), 64, 1, 1, 8) == 0
    tables = [O.RefBlockTable() for _ in range(3)]
    for i, t in enumerate(tables):
        assert R.qwn_block_table_init(C.byref(t), i, 2) == 0
    order = [0, 1, 2] * 20 + [0] * 37 + [2] * 5
    for s in order:
        assert R.qwn_block_table_append_token(C.byref(pool), C.byref(tables[s])) == 0
    out["bt_order"] = np.array(order, np.int32)
    out["bt_tables"] = np.concatenate([np.ctypeslib.as_array(t.block_ids, shape=(t.block_count,)).copy()
                                       for t in tables] + [np.array([-1], np.int32)])
    out["bt_counts"] = np.array([t.block_count for t in tables], np.int32)
    out["bt_tokens"] = np.array([t.num_tokens for t in tables], np.int32)
    out["bt_free_top"] = np.array([pool.free_top], np.int32)
    for t in tables:
        R.qwn_block_table_free(C.byref(pool), C.byref(t))
    out["bt_free_after"] = np.ctypeslib.as_array(pool.free_stack, shape=(pool.free_top,)).copy()
    R.qwn_kv_pool_free(C.byref(pool))

    # --- vToken eviction (c/tests/test_nextgen_suite.c:138-177) ------------
    ep = O.EvictionPool()
    assert R.qwn_paged_eviction_init(C.byref(ep), 1024, 512, C.c_float(0.10)) == 0
    slot = C.c_uint32(0)
    for i in range(100):
        assert R.qwn_paged_eviction_insert(C.byref(ep), i, C.c_float(1.0), C.byref(slot)) == 0
    attn = np.array([0.9 if i % 2 == 0 else 0.01 for i in range(100)], np.float32)
    R.qwn_paged_eviction_update_scores(C.byref(ep), O._ptr(attn, O.f32p), 100)
    out["vt_scores"] = np.array([ep.tokens[i].importance_score for i in range(100)], np.float32)
    out["vt_evicted"] = np.array([R.qwn_paged_eviction_prune(C.byref(ep), 50)], np.uint32)
    out["vt_active"] = np.array([ep.tokens[i].is_active for i in range(100)], np.uint8)
    out["vt_waste"] = np.array([R.qwn_paged_eviction_memory_waste_pct(C.byref(ep))], np.float32)

    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_vectors.npz"), sorted(out))


if __name__ == "__main__":
    main()
