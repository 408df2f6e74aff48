"""The CPU oracle pinned against the reference: golden vectors from the
reference's own functions (tests/golden/make_golden.py) and, when
oracle/_ref is built, live differential checks on random inputs."""
import ctypes as C
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


# ---------------------------------------------------------------- golden ---

def test_q8_analytic_inputs_match_reference(oracle_mod, gold):
    """c/tests/test_kv_cache.c:29-46: 2 heads x 65 channels (partial block)."""
    ck, sk = oracle_mod.q8_b64(gold["kv_key"])
    cv, sv = oracle_mod.q8_b64(gold["kv_value"])
    assert np.array_equal(ck, gold["kv_codes_k"])
    assert np.array_equal(sk.view(np.uint32), gold["kv_scales_k"].view(np.uint32))
    assert np.array_equal(cv, gold["kv_codes_v"])
    assert np.array_equal(sv.view(np.uint32), gold["kv_scales_v"].view(np.uint32))
    # round trip within the reference's own 0.02 (test_kv_cache.c:44-46)
    deq = cv[:65].astype(np.float32) * sv[np.arange(65) // 64]
    assert abs(deq[0] - gold["kv_value"][0]) <= 0.02 and abs(deq[64] - gold["kv_value"][64]) <= 0.02


def test_q8_nonfinite_inputs_match_reference(oracle_mod, gold):
    """c/tests/test_kv_cache.c:52-59: NaN/Inf -> code 0, finite scale."""
    ck, sk = oracle_mod.q8_b64(gold["kv_nan_key"])
    cv, sv = oracle_mod.q8_b64(gold["kv_nan_value"])
    assert np.array_equal(ck, gold["kv_nan_codes_k"]) and np.array_equal(cv, gold["kv_nan_codes_v"])
    assert np.array_equal(sk.view(np.uint32), gold["kv_nan_scales_k"].view(np.uint32))
    assert np.array_equal(sv.view(np.uint32), gold["kv_nan_scales_v"].view(np.uint32))
    assert ck[0] == 0 and ck[1] == 0 and cv[0] == 0 and cv[1] == 0 and np.isfinite(sk).all()


def test_turboquant_test_inputs_match_reference(oracle_mod, gold):
    """c/tests/test_turboquant.c dims x distributions: 3.5-bit blocks and Q8
    codes bit-exact against the reference quantizers."""
    xs, blocks = gold["tq_inputs"], gold["tq_blocks"]
    qc, qs = gold["tq_q8_codes"], gold["tq_q8_scales"]
    xo = bo = so = 0
    for dim in gold["tq_dims"]:
        x = xs[xo: xo + dim]
        nb = (dim + 63) // 64
        assert np.array_equal(oracle_mod.tq35(x), blocks[bo: bo + nb * 32])
        c, s = oracle_mod.q8_b64(x)
        assert np.array_equal(c, qc[xo: xo + dim])
        assert np.array_equal(s.view(np.uint32), qs[so: so + nb].view(np.uint32))
        xo, bo, so = xo + dim, bo + nb * 32, so + nb


def test_block_table_matches_reference(oracle_mod, gold):
    """qwn_block_table_append_token order (c/qwn_paged_kv.c:115-138) and the
    LIFO free stack after qwn_block_table_free."""
    p = oracle_mod.Pool(oracle_mod.CODEC_Q8_HEAD_F16, 1, 1, 16, 64, 3, 64)
    for s in gold["bt_order"]:
        assert p.append([int(s)], [1]) == 0
    flat = []
    for s in range(3):
        flat += list(p.page_table()[s, : p.npages()[s]])
    assert np.array_equal(np.array(flat + [-1], np.int32), gold["bt_tables"])
    assert np.array_equal(p.npages()[:3], gold["bt_counts"])
    assert np.array_equal(p.lens()[:3], gold["bt_tokens"])
    assert p.p.free_top == int(gold["bt_free_top"][0])


def test_vtoken_suite_matches_reference(oracle_mod, gold):
    """c/tests/test_nextgen_suite.c:138-177 through the restated token pool."""
    L = oracle_mod.lib()
    ep = oracle_mod.EvictionPool()
    assert L.qor_vtoken_init(C.byref(ep), 1024, 512, 0.10) == 0
    slot = C.c_uint32(0)
    for i in range(100):
        assert L.qor_vtoken_insert(C.byref(ep), i, 1.0, C.byref(slot)) == 0 and slot.value == i
    attn = np.array([0.9 if i % 2 == 0 else 0.01 for i in range(100)], np.float32)
    L.qor_vtoken_update_scores(C.byref(ep), oracle_mod._ptr(attn, oracle_mod.f32p), 100, 1)
    scores = np.array([ep.tokens[i].importance_score for i in range(100)], np.float32)
    assert np.array_equal(scores.view(np.uint32), gold["vt_scores"].view(np.uint32))
    assert L.qor_vtoken_prune(C.byref(ep), 50) == int(gold["vt_evicted"][0])
    active = np.array([ep.tokens[i].is_active for i in range(100)], np.uint8)
    assert np.array_equal(active, gold["vt_active"])
    assert all(ep.tokens[i].is_active for i in range(4))  # sinks survive
    assert L.qor_vtoken_waste_pct(C.byref(ep)) == pytest.approx(float(gold["vt_waste"][0]))


# -------------------------------------------------------- live reference ---

def test_q8_random_bit_exact_live(oracle_mod, ref_lib):
    rng = np.random.default_rng(11)
    for trial in range(300):
        n = int(rng.choice([1, 4, 63, 64, 65, 128, 130, 1024]))
        x = (rng.standard_normal(n) * rng.choice([1e-30, 1e-6, 1.0, 300.0, 1e30])).astype(np.float32)
        if trial % 5 == 0:
            x[rng.integers(0, n)] = rng.choice([np.nan, np.inf, -np.inf])
        c = oracle_mod.RefQ8Cache()
        assert ref_lib.qwn_q8_cache_init(C.byref(c), 2, 1, n) == 0
        assert ref_lib.qwn_q8_cache_append(C.byref(c), oracle_mod._ptr(x, oracle_mod.f32p),
                                           oracle_mod._ptr(x, oracle_mod.f32p), n) == 0
        rc = np.ctypeslib.as_array(c.packed_k, shape=(n,)).copy()
        rs = np.ctypeslib.as_array(c.scales_k, shape=((n + 63) // 64,)).copy()
        ref_lib.qwn_q8_cache_free(C.byref(c))
        oc, os_ = oracle_mod.q8_b64(x)
        assert np.array_equal(rc, oc)
        assert np.array_equal(rs.view(np.uint32), os_.view(np.uint32))


def test_tq35_random_bit_exact_live(oracle_mod, ref_lib):
    rng = np.random.default_rng(12)
    for _ in range(300):
        n = int(rng.choice([64, 100, 128, 192, 512]))
        x = (rng.standard_normal(n) * rng.choice([1e-9, 1e-3, 1.0, 15.0, 1e4])).astype(np.float32)
        blk = np.zeros(((n + 63) // 64) * 32, np.uint8)
        ref_lib.qwn_turboquant_quantize_token(oracle_mod._ptr(x, oracle_mod.f32p),
                                              oracle_mod._ptr(blk, oracle_mod.u8p), n)
        assert np.array_equal(blk, oracle_mod.tq35(x))


def test_block_table_with_permuted_free_stack_live(oracle_mod, ref_lib):
    """The seeded page permutation is a permutation of the reference's
    initial free stack; allocation order then follows the reference."""
    total, seed = 97, 777
    pool = oracle_mod.RefBlockPool()
    assert ref_lib.qwn_kv_pool_init(C.byref(pool), total, 1, 1, 8) == 0
    perm = oracle_mod.free_stack(seed, total)
    np.ctypeslib.as_array(pool.free_stack, shape=(total,))[:] = perm
    tabs = [oracle_mod.RefBlockTable() for _ in range(4)]
    for i, t in enumerate(tabs):
        ref_lib.qwn_block_table_init(C.byref(t), i, 4)
    p = oracle_mod.Pool(oracle_mod.CODEC_Q8_HEAD_F16, 1, 1, 16, total, 4, 64, perm_seed=seed)
    rng = np.random.default_rng(3)
    for _ in range(600):
        s = int(rng.integers(0, 4))
        r_rc = ref_lib.qwn_block_table_append_token(C.byref(pool), C.byref(tabs[s]))
        o_rc = p.append([s], [1])
        assert (r_rc == 0) == (o_rc == 0)
    for s in range(4):
        ref_ids = np.ctypeslib.as_array(tabs[s].block_ids, shape=(tabs[s].block_count,))
        assert np.array_equal(ref_ids, p.page_table()[s, : p.npages()[s]])
    assert pool.free_top == p.p.free_top


def test_vtoken_contraction_form_live(oracle_mod, ref_lib):
    """Determine which EMA rounding the compiled reference performs and check
    the restatement reproduces it bit for bit on random scores."""
    L = oracle_mod.lib()
    rng = np.random.default_rng(5)
    for trial in range(50):
        cap = int(rng.integers(20, 300))
        phys = int(rng.integers(10, cap + 5))
        thr = float(rng.choice([0.0, 0.05, 0.3]))
        a, b = oracle_mod.EvictionPool(), oracle_mod.EvictionPool()
        ref_lib.qwn_paged_eviction_init(C.byref(a), cap, phys, thr)
        L.qor_vtoken_init(C.byref(b), cap, phys, thr)
        slot = C.c_uint32(0)
        for step in range(int(rng.integers(5, 400))):
            op = rng.integers(0, 3)
            if op == 0:
                tid, imp = int(rng.integers(0, 1000)), float(rng.standard_normal())
                ra = ref_lib.qwn_paged_eviction_insert(C.byref(a), tid, imp, C.byref(slot))
                rb = L.qor_vtoken_insert(C.byref(b), tid, imp, C.byref(slot))
                assert ra == rb
            elif op == 1:
                sc = rng.random(400).astype(np.float32)
                n = int(rng.integers(0, 400))
                ref_lib.qwn_paged_eviction_update_scores(C.byref(a), oracle_mod._ptr(sc, oracle_mod.f32p), n)
                L.qor_vtoken_update_scores(C.byref(b), oracle_mod._ptr(sc, oracle_mod.f32p), n, 1)
            else:
                t = int(rng.integers(0, cap))
                assert ref_lib.qwn_paged_eviction_prune(C.byref(a), t) == L.qor_vtoken_prune(C.byref(b), t)
        assert a.active_count == b.active_count and a.total_evictions == b.total_evictions
        for i in range(a.active_count):
            assert a.tokens[i].is_active == b.tokens[i].is_active
            assert np.float32(a.tokens[i].importance_score).view(np.uint32) == \
                np.float32(b.tokens[i].importance_score).view(np.uint32)


def test_q8_attention_oracle_vs_reference_live(oracle_mod, ref_lib):
    """qwn_q8_cache_attention_head (c/qwanto_turboquant.c:678-705) against the
    oracle's paged attention with the reference codec: identical codes, fp32
    results equal within reassociation noise."""
    rng = np.random.default_rng(9)
    HK, HD = 2, 128
    for H, ntok in [(4, 1), (12, 37), (12, 300)]:
        c = oracle_mod.RefQ8Cache()
        assert ref_lib.qwn_q8_cache_init(C.byref(c), ntok, HK, HD) == 0
        p = oracle_mod.Pool(oracle_mod.CODEC_Q8_B64_F32, 1, HK, 16, 64, 1, 64)
        assert p.append([0], [ntok]) == 0
        for t in range(ntok):
            k = rng.standard_normal(HK * HD).astype(np.float32)
            v = rng.standard_normal(HK * HD).astype(np.float32)
            assert ref_lib.qwn_q8_cache_append(C.byref(c), oracle_mod._ptr(k, oracle_mod.f32p),
                                               oracle_mod._ptr(v, oracle_mod.f32p), HK * HD) == 0
            assert p.write(0, 0, t, k, v) == 0
        q = rng.standard_normal(H * HD).astype(np.float32)
        scale = 1.0 / np.sqrt(HD)
        ours = p.attention(0, 0, ntok, q, H, scale)
        sc = np.zeros(ntok, np.float32)
        for h in range(H):
            ctx = np.zeros(HD, np.float32)
            ref_lib.qwn_q8_cache_attention_head(oracle_mod._ptr(q[h * HD:], oracle_mod.f32p), C.byref(c),
                                                (h * HK) // H, ntok - 1, C.c_float(scale),
                                                oracle_mod._ptr(sc, oracle_mod.f32p),
                                                oracle_mod._ptr(ctx, oracle_mod.f32p))
            np.testing.assert_allclose(ours[h], ctx, rtol=1e-5, atol=1e-6)
        ref_lib.qwn_q8_cache_free(C.byref(c))


def test_tq35_attention_oracle_vs_reference_live(oracle_mod, ref_lib):
    """qwn_turboquant_attention_head (SIMD dispatch) vs the oracle's scalar
    order over the 3.5-bit paged layout; tolerance of test_turboquant.c."""
    rng = np.random.default_rng(10)
    HK, HD, H, ntok = 2, 128, 4, 200
    tq = oracle_mod.RefTQCache()
    assert ref_lib.qwn_turboquant_init(C.byref(tq), ntok, HK, HD) == 0
    p = oracle_mod.Pool(oracle_mod.CODEC_TQ35_G64, 1, HK, 16, 64, 1, 64)
    assert p.append([0], [ntok]) == 0
    for t in range(ntok):
        k = rng.standard_normal(HK * HD).astype(np.float32)
        v = rng.standard_normal(HK * HD).astype(np.float32)
        for h in range(HK):
            ref_lib.qwn_turboquant_quantize_token(
                oracle_mod._ptr(k[h * HD:], oracle_mod.f32p),
                C.cast(C.addressof(tq.packed_k.contents) + t * tq.token_stride_k + h * 64, oracle_mod.u8p), HD)
            ref_lib.qwn_turboquant_quantize_token(
                oracle_mod._ptr(v[h * HD:], oracle_mod.f32p),
                C.cast(C.addressof(tq.packed_v.contents) + t * tq.token_stride_v + h * 64, oracle_mod.u8p), HD)
        assert p.write(0, 0, t, k, v) == 0
    tq.n_tokens = ntok
    q = rng.standard_normal(H * HD).astype(np.float32)
    scale = 1.0 / np.sqrt(HD)
    ours = p.attention(0, 0, ntok, q, H, scale)
    sc = np.zeros(ntok, np.float32)
    for h in range(H):
        ctx = np.zeros(HD, np.float32)
        ref_lib.qwn_turboquant_attention_head(oracle_mod._ptr(q[h * HD:], oracle_mod.f32p), C.byref(tq), 0, h,
                                              (h * HK) // H, ntok - 1, C.c_float(scale),
                                              oracle_mod._ptr(sc, oracle_mod.f32p), oracle_mod._ptr(ctx, oracle_mod.f32p))
        np.testing.assert_allclose(ours[h], ctx, rtol=1e-3, atol=1e-4)
    ref_lib.qwn_turboquant_free(C.byref(tq))


def _f16_specials():
    rng = np.random.default_rng(12)
    xs = [rng.standard_normal(1024).astype(np.float32) * s for s in (1e-9, 6e-8, 3e-5, 1.0, 1e3, 6.5e4)]
    edge = np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, -65520.0, 1e6, np.inf, -np.inf,
                     2.0 ** -24, 2.0 ** -25, 1.5 * 2.0 ** -25, 2.0 ** -14, 2.0 ** -14 * (1 - 2.0 ** -11)],
                    np.float32)
    nans = np.array([0x7FC00000, 0x7F800001, 0xFFC12345, 0x7FBFFFFF], np.uint32).view(np.float32)
    x = np.concatenate(xs + [edge, nans]).astype(np.float32)
    return np.concatenate([x, np.zeros((-len(x)) % (16 * 128), np.float32)])


def test_f16_store_matches_reference_pool_write_live(oracle_mod, ref_lib):
    """The fp16 codec's rounding against the reference's own pool write
    (qwn_paged_kv_write, c/qwn_paged_kv.c:151-198, F16C round to nearest
    even): bit-exact on random, subnormal, overflow, infinite and NaN inputs."""
    x = _f16_specials().reshape(-1, 16, 128)
    for blk in x:
        k16 = np.zeros((16, 128), np.uint16)
        v16 = np.zeros((16, 128), np.uint16)
        v = -blk[::-1].copy()
        assert ref_lib.qref_f16_write(oracle_mod._ptr(blk, oracle_mod.f32p), oracle_mod._ptr(v, oracle_mod.f32p),
                                      16, 128, oracle_mod._ptr(k16, oracle_mod.u16p),
                                      oracle_mod._ptr(v16, oracle_mod.u16p)) == 0
        mine_k = np.array([oracle_mod.f16_rne(float(e)) for e in blk.ravel()], np.uint16).reshape(16, 128)
        mine_v = np.array([oracle_mod.f16_rne(float(e)) for e in v.ravel()], np.uint16).reshape(16, 128)
        assert np.array_equal(mine_k, k16) and np.array_equal(mine_v, v16)


def test_f16_attention_oracle_vs_reference_live(oracle_mod, ref_lib):
    """The decoder's fp16 paged path (block table appends, qwn_paged_kv_write,
    qwn_paged_attention_gather_head; c/qwanto_decode.c:1600-1604, :1807-1835)
    run by the reference shim, against the oracle's fp16 codec on the same
    generated rows: equal within reassociation noise."""
    HK, HD, H, seed = 2, 128, 12, 33
    for ntok in (1, 17, 300):
        lens = np.array([ntok - 1], np.int32)
        b = ref_lib.qref_batch_create(5, 1, oracle_mod._ptr(lens, oracle_mod.i32p), 1, H, HK, HD, 1, seed)
        assert b
        assert ref_lib.qref_batch_step(b, 1) == 1
        ctx = np.ctypeslib.as_array(ref_lib.qref_batch_ctx(b), shape=(H * HD,)).copy().reshape(H, HD)
        ref_lib.qref_batch_destroy(b)
        p = oracle_mod.Pool(oracle_mod.CODEC_F16, 1, HK, 16, 64, 1, 64)
        assert p.append([0], [ntok]) == 0
        for t in range(ntok):
            assert p.write(0, 0, t, oracle_mod.gen_row(seed, 2, 0, 0, t, HK * HD),
                           oracle_mod.gen_row(seed, 3, 0, 0, t, HK * HD)) == 0
        ours = p.attention(0, 0, ntok, oracle_mod.gen_row(seed, 1, 0, 0, ntok - 1, H * HD), H, 1.0 / np.sqrt(HD))
        np.testing.assert_allclose(ours, ctx, rtol=1e-5, atol=1e-6)


def test_linear_attention_matches_reference_live(oracle_mod, ref_lib):
    """Linear-attention decode and prefill (c/qwanto_attention.c:34-156, the
    AVX2 path the reference is built with) against the oracle's restatement:
    states and outputs bit-exact over several steps."""
    rng = np.random.default_rng(21)
    H, D, T = 3, 128, 6
    st = oracle_mod.RefLinearState()
    assert ref_lib.qwanto_linear_attention_init(C.byref(st), H, D) == 0
    mine = np.zeros((H, D, D), np.float32)
    q = rng.standard_normal((T, H, D)).astype(np.float32)
    k = rng.standard_normal((T, H, D)).astype(np.float32)
    v = rng.standard_normal((T, H, D)).astype(np.float32)
    decay = np.float32(0.93)
    ref_o = np.zeros((T, H, D), np.float32)
    ref_lib.qwanto_linear_attention_prefill(C.byref(st), oracle_mod._ptr(q, oracle_mod.f32p),
                                            oracle_mod._ptr(k, oracle_mod.f32p), oracle_mod._ptr(v, oracle_mod.f32p),
                                            C.c_float(decay), T, oracle_mod._ptr(ref_o, oracle_mod.f32p))
    for s in range(T):
        o = np.zeros((H, D), np.float32)
        oracle_mod.lib().qor_linear_attention_decode(oracle_mod._ptr(mine, oracle_mod.f32p), H, D,
                                                     oracle_mod._ptr(q[s], oracle_mod.f32p),
                                                     oracle_mod._ptr(k[s], oracle_mod.f32p),
                                                     oracle_mod._ptr(v[s], oracle_mod.f32p), C.c_float(decay),
                                                     oracle_mod._ptr(o, oracle_mod.f32p))
        assert np.array_equal(o, ref_o[s])
    ref_state = np.ctypeslib.as_array(st.state, shape=(H, D, D))
    assert np.array_equal(mine, ref_state)
    ref_lib.qwanto_linear_attention_destroy(C.byref(st))


# ------------------------------------------------------- oracle internals ---

def test_f16_rne_matches_numpy(oracle_mod):
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(4000).astype(np.float32) * s
                         for s in [1e-8, 6e-8, 1e-6, 1e-4, 1.0, 3e4, 6.6e4]]).astype(np.float32)
    mine = np.array([oracle_mod.f16_rne(float(v)) for v in xs], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(mine, xs.astype(np.float16).view(np.uint16))


def test_f16_tile_round_trip(oracle_mod):
    """The fp16 codec's tile reads back fp16(x) at every (token, dim) slot."""
    rng = np.random.default_rng(5)
    tile = np.zeros(oracle_mod.TILE_BYTES[5], np.uint8)
    ks = rng.standard_normal((16, 128)).astype(np.float32) * 3
    vs = rng.standard_normal((16, 128)).astype(np.float32)
    L = oracle_mod.lib()
    for t in rng.permutation(16):
        L.qor_tile_store(5, oracle_mod._ptr(tile, oracle_mod.u8p), int(t),
                         oracle_mod._ptr(ks[t], oracle_mod.f32p), oracle_mod._ptr(vs[t], oracle_mod.f32p))
    for t in range(16):
        for isv, x in ((0, ks[t]), (1, vs[t])):
            got = np.array([L.qor_tile_dequant(5, oracle_mod._ptr(tile, oracle_mod.u8p), t, isv, d) for d in range(128)],
                           np.float32)
            assert np.array_equal(got, x.astype(np.float16).astype(np.float32))


@pytest.mark.parametrize("codec", [1, 2, 3, 4])
def test_tile_layout_round_trip(oracle_mod, codec):
    """Every slot of a tile reads back the logical codes and parameters the
    quantizer produced (the layout is a permutation)."""
    rng = np.random.default_rng(codec)
    tile = np.zeros(oracle_mod.TILE_BYTES[codec], np.uint8)
    ks = rng.standard_normal((16, 128)).astype(np.float32) * 3
    vs = rng.standard_normal((16, 128)).astype(np.float32)
    L = oracle_mod.lib()
    for t in rng.permutation(16):
        L.qor_tile_store(codec, oracle_mod._ptr(tile, oracle_mod.u8p), int(t),
                         oracle_mod._ptr(ks[t], oracle_mod.f32p), oracle_mod._ptr(vs[t], oracle_mod.f32p))
    for t in range(16):
        for isv, x in ((0, ks[t]), (1, vs[t])):
            codes, params = oracle_mod.tile_load(codec, tile, t, isv)
            if codec == 1:
                c, s = oracle_mod.q8_b64(x)
                assert np.array_equal(codes, c) and np.array_equal(params[:2], s)
            elif codec == 2:
                c, s16 = oracle_mod.q8_head(x)
                assert np.array_equal(codes, c)
                assert np.float16(params[0]).view(np.uint16) == s16
            elif codec == 4:
                c, r, m = oracle_mod.q4g32(x)
                assert np.array_equal(codes, c)
                assert np.array_equal(params[0::2][:4].astype(np.float16).view(np.uint16), r)
                assert np.array_equal(params[1::2][:4].astype(np.float16).view(np.uint16), m)
            else:
                blk = oracle_mod.tq35(x)
                for g in range(2):
                    cg = np.zeros(64, np.uint8)
                    r16 = np.zeros(1, np.uint16)
                    m16 = np.zeros(1, np.uint16)
                    oracle_mod.lib().qor_tq35_unpack(oracle_mod._ptr(blk[g * 32:], oracle_mod.u8p),
                                                     oracle_mod._ptr(cg, oracle_mod.u8p),
                                                     oracle_mod._ptr(r16, oracle_mod.u16p),
                                                     oracle_mod._ptr(m16, oracle_mod.u16p))
                    assert np.array_equal(codes[g * 64:(g + 1) * 64], cg)
                    assert np.float16(params[2 * g]).view(np.uint16) == r16[0]


def test_generator_is_normal_and_exact(oracle_mod):
    v = oracle_mod.normal(3, oracle_mod.stream(2, 0, 0), 0, 200_000)
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01
    assert np.all(v * 65536 == np.round(v * 65536))  # on the 2^-16 grid


def test_page_eviction_oracle_properties(oracle_mod):
    """Page 0 and the tail page survive, the budget is met, freed pages go
    back on the free stack in ascending logical order."""
    P, budget = 16, 64
    p = oracle_mod.Pool(oracle_mod.CODEC_Q8_HEAD_F16, 1, 1, P, 200, 3, 64, perm_seed=9)
    assert p.append([0, 1, 2], [300, 50, 170]) == 0
    rng = np.random.default_rng(2)
    mass = rng.random((3, 64)).astype(np.float32)
    before = p.page_table().copy()
    top_before = p.p.free_top
    n = p.evict([0, 1, 2], mass, [1, 1, 0], budget)
    lens = p.lens()[:3]
    assert lens[0] <= budget and lens[1] == 50 and lens[2] == 170
    np0 = (300 + P - 1) // P
    tbl = p.page_table()
    assert tbl[0, 0] == before[0, 0]
    assert tbl[0, p.npages()[0] - 1] == before[0, np0 - 1]
    freed = p.free_stack()[top_before:]
    assert len(freed) == n
    kept = set(tbl[0, : p.npages()[0]])
    expect = [pg for pg in before[0, :np0] if pg not in kept]
    assert list(freed) == expect


def test_fill_synthetic_equals_token_writes(oracle_mod):
    """The oracle's bulk synthetic fill (used by the full-size GPU tests)
    stores exactly the rows gen_row gives, K x 8 on outlier channels, into
    the chosen layer; a metadata-only pool keeps tables without pages."""
    O = oracle_mod
    a = O.Pool(4, 2, 8, 16, 40, 3, 20, perm_seed=3)
    b = O.Pool(4, 1, 8, 16, 40, 3, 20, perm_seed=3)
    mask = O.outlier_mask(3, 1, 1024, 10)
    for p in (a, b):
        assert p.append([0, 2], [50, 33]) == 0
    for s, n in ((0, 50), (2, 33)):
        for t in range(n):
            k = O.gen_row(9, 2, s, 1, t, 1024)
            k = np.where(mask != 0, k * np.float32(8), k).astype(np.float32)
            assert a.write(s, 1, t, k, O.gen_row(9, 3, s, 1, t, 1024)) == 0
        assert b.fill_synthetic(s, 0, 1, 0, n, 9, mask) == 0
        for t in range(0, n, 16):
            for h in range(8):
                assert np.array_equal(a.tile(s, 1, h, t), b.tile(s, 0, h, t))
    m = O.Pool(2, 1, 8, 16, 1 << 16, 4, 64, perm_seed=5, with_pages=False)
    full = O.Pool(2, 1, 8, 16, 1 << 16, 4, 64, perm_seed=5)
    for p in (m, full):
        assert p.append([1, 3], [100, 7]) == 0
    assert np.array_equal(m.page_table(), full.page_table())
    assert np.array_equal(m.free_stack(), full.free_stack())
    assert m.fill_synthetic(1, 0, 0, 0, 100, 9) == -1
