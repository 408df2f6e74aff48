"""Parity of the CUDA path (through the C-ABI) with the CPU oracle.

Bit-exact: quantized codes/scales in the pages, page tables, free stack,
eviction decisions.  Tolerance |d| <= 1e-4 + 1e-3|ref| for fp32 attention.
"""
import ctypes as C

import numpy as np
import pytest

from kvharness import Twin, assert_close

pytestmark = pytest.mark.gpu

CODECS = [1, 2, 3, 4, 5]


def test_generator_bit_exact(cuda, oracle_mod):
    import qwanto_b200 as qb
    torch = cuda
    ids = torch.tensor([0, 5, 9], dtype=torch.int32, device="cuda")
    pos = torch.tensor([0, 7, 4095], dtype=torch.int32, device="cuda")
    out = torch.empty((3, 1024), dtype=torch.float32, device="cuda")
    mask = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    mask[[3, 500]] = 1
    qb.generate_rows(out, 3, 1024, 2, 77, 3, ids, pos, mask)
    got = out.cpu().numpy()
    for r, (s, p) in enumerate([(0, 0), (5, 7), (9, 4095)]):
        ref = oracle_mod.gen_row(77, 2, s, 3, p, 1024)
        ref[[3, 500]] *= 8
        assert np.array_equal(got[r].view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("codec", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("page_tokens", [16, 64])
def test_prefill_pages_bit_exact(cuda, codec, page_tokens):
    """Quantize-on-append into pages: every byte of every used page, the page
    tables and the LIFO free stack equal the oracle's."""
    tw = Twin(cuda, codec, layers=2, kv_heads=2, page_tokens=page_tokens, total_pages=40, max_seqs=4,
              max_pages=16, query_heads=8, perm_seed=123, seed=5)
    try:
        tw.prefill([2, 0, 3], [17, 1, 70])
        assert tw.gpu.check() == 0
        tw.assert_state_equal()
        tw.assert_pages_equal()
    finally:
        tw.close()


@pytest.mark.parametrize("codec", CODECS)
@pytest.mark.parametrize("heads", [(12, 2), (32, 8), (4, 4), (16, 2)])
def test_decode_steps_parity(cuda, codec, heads):
    """Decode steps with append through qwn_kv_decode: outputs within the
    tolerance, pages and tables bit-exact after every step."""
    H, HK = heads
    tw = Twin(cuda, codec, layers=2, kv_heads=HK, page_tokens=16, total_pages=96, max_seqs=5,
              max_pages=24, query_heads=H, perm_seed=7, seed=11)
    try:
        tw.prefill([0, 1, 2, 3, 4], [1, 15, 16, 31, 200])
        for _ in range(3):
            g, o, _ = tw.step([0, 1, 2, 3, 4])
            assert_close(g, o, f"codec {codec} H={H} HK={HK}")
            assert tw.gpu.check() == 0
            tw.assert_state_equal()
        tw.assert_pages_equal()
    finally:
        tw.close()


@pytest.mark.parametrize("codec", CODECS)
def test_long_context_and_subset_batch(cuda, codec):
    """Long and ragged contexts, a batch that is a permuted subset of the
    sequence slots, page size 64."""
    tw = Twin(cuda, codec, layers=1, kv_heads=8, page_tokens=64, total_pages=160, max_seqs=6,
              max_pages=80, query_heads=48, perm_seed=99, seed=4)
    try:
        tw.prefill([5, 1, 3], [3000, 63, 1025])
        g, o, _ = tw.step([3, 5, 1])
        assert_close(g, o, f"codec {codec} long")
        tw.assert_state_equal()
        tw.assert_pages_equal()
    finally:
        tw.close()


@pytest.mark.parametrize("codec", [2, 3, 5])
def test_single_long_sequence_two_level_merge(cuda, codec):
    """One 24k-token sequence: every (sequence, kv head) segment is split over
    ~220 warps, so the partials merge in two levels (groups of 16, then the
    group results); page size 64, 6 query heads per kv head."""
    tw = Twin(cuda, codec, layers=1, kv_heads=8, page_tokens=64, total_pages=400, max_seqs=1,
              max_pages=400, query_heads=48, perm_seed=3, seed=31)
    try:
        tw.prefill([0], [24000])
        for _ in range(2):
            g, o, _ = tw.step([0])
            assert_close(g, o, f"codec {codec} two-level merge")
        tw.assert_state_equal()
    finally:
        tw.close()


@pytest.mark.parametrize("codec", [2, 4, 5])
@pytest.mark.parametrize("heads", [(32, 8), (12, 2)])
def test_identity_batch_cached_plans(cuda, codec, heads):
    """Calls without a sequence-id array cache the launch setup across the
    layers of a step; every step's append (and a pool reset) invalidates it."""
    H, HK = heads
    tw = Twin(cuda, codec, layers=3, kv_heads=HK, page_tokens=16, total_pages=120, max_seqs=4,
              max_pages=40, query_heads=H, perm_seed=7, seed=15)
    try:
        tw.prefill([0, 1, 2, 3], [37, 300, 1, 129])
        for _ in range(3):
            g, o, _ = tw.step([0, 1, 2, 3], identity=True)
            assert_close(g, o, f"codec {codec} identity batch")
        tw.assert_state_equal()
        tw.assert_pages_equal()
    finally:
        tw.close()


def test_identity_batch_plans_after_eviction(cuda):
    """Eviction and compaction change lengths and tables between steps; the
    cached launch setup must not survive it."""
    torch = cuda
    tw = Twin(cuda, 2, layers=2, kv_heads=8, page_tokens=16, total_pages=400, max_seqs=8, max_pages=64,
              query_heads=32, perm_seed=5, seed=8)
    seqs = list(range(8))
    try:
        tw.prefill(seqs, [40, 100, 600, 33, 700, 129, 16, 500])
        rng = np.random.default_rng(9)
        for step in range(4):
            g, o, masses = tw.step(seqs, page_mass=True, identity=True)
            assert_close(g, o, "churn outputs, identity batch")
            mass = masses[-1]
            flags = (rng.random(8) < 0.5).astype(np.uint8)
            tw.gpu.evict(8, torch.tensor(mass, device="cuda"), torch.tensor(flags, device="cuda"), 96)
            tw.ora.evict(seqs, mass, flags, 96)
            assert tw.gpu.check() == 0
            tw.assert_state_equal()
    finally:
        tw.close()


def test_outlier_channels_q4(cuda, oracle_mod):
    """Config-3 style K with 1% outlier channels x8, 4-bit groups of 32."""
    tw = Twin(cuda, 4, layers=2, kv_heads=8, page_tokens=16, total_pages=120, max_seqs=3, max_pages=40,
              query_heads=32, perm_seed=3, seed=3)
    tw.mask = np.stack([oracle_mod.outlier_mask(3, layer, 1024, 10) for layer in range(2)])
    try:
        tw.prefill([0, 1, 2], [300, 17, 129])
        g, o, _ = tw.step([0, 1, 2])
        assert_close(g, o, "q4 outliers")
        tw.assert_pages_equal()
    finally:
        tw.close()


def test_pool_exhaustion_latches_and_changes_nothing(cuda):
    """Host-visible failure: pool exhausted (c/qwanto_decode.c:1600-1604)."""
    import qwanto_b200 as qb
    from qwanto_b200 import _lib
    torch = cuda
    pool = qb.KvPool(2, 1, 2, 16, 4, 2, 8, max_query_heads=4)
    try:
        pool.prefill_synthetic([0, 1], [32, 32], 1)  # all 4 pages used
        assert pool.check() == 0
        before = (pool.lens().copy(), pool.page_table().copy())
        ids = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
        pool.seq_append(2, ids)
        assert pool.check() & _lib.ST_POOL_EXHAUSTED
        assert np.array_equal(pool.lens(), before[0]) and np.array_equal(pool.page_table(), before[1])
        assert pool.check() == 0  # cleared by the read
    finally:
        pool.close()


def test_partial_merge_equals_full(cuda):
    """Split-KV across ranges (the multi-GPU path on one device): partial
    (m, l, o) over token ranges merged equals the full attention."""
    import qwanto_b200 as qb
    torch = cuda
    tw = Twin(cuda, 2, layers=1, kv_heads=8, page_tokens=64, total_pages=64, max_seqs=1, max_pages=64,
              query_heads=48, seed=21)
    try:
        tw.prefill([0], [2500])
        q = torch.empty((1, 48 * 128), dtype=torch.float32, device="cuda")
        pos = torch.tensor([2499], dtype=torch.int32, device="cuda")
        qb.generate_rows(q, 1, 48 * 128, 1, 21, 0, None, pos)
        full = torch.zeros_like(q)
        tw.gpu.decode(0, 1, 48, q, full)
        bounds = [0, 640, 1280, 1920, 2500]
        parts = len(bounds) - 1
        m = torch.zeros((parts, 48), device="cuda")
        l = torch.zeros((parts, 48), device="cuda")
        o = torch.zeros((parts, 48, 128), device="cuda")
        for i in range(parts):
            tw.gpu.partial(0, 1, 48, q, m[i], l[i], o[i], t_begin=bounds[i], t_end=bounds[i + 1])
        merged = torch.zeros((48, 128), device="cuda")
        qb.merge_partials(parts, 48, m, l, o, merged)
        torch.cuda.synchronize()
        assert_close(merged.cpu().numpy(), full.cpu().numpy().reshape(48, 128), "merge")
        ref = tw.ora.attention(0, 0, 2500, tw.row(1, 0, 0, 2499, 48 * 128), 48, 1.0 / np.sqrt(128.0))
        assert_close(merged.cpu().numpy(), ref, "merge vs oracle")
        # the packed form: each part one block o | m | l, as the split-KV bench all-gathers it
        packed = torch.zeros((parts, 48 * 130), device="cuda")
        for i in range(parts):
            blk = packed[i]
            tw.gpu.partial(0, 1, 48, q, blk[48 * 128: 48 * 129], blk[48 * 129:], blk[: 48 * 128],
                           t_begin=bounds[i], t_end=bounds[i + 1])
        merged2 = torch.zeros((48, 128), device="cuda")
        qb.merge_partials_packed(parts, 48, packed, merged2)
        torch.cuda.synchronize()
        assert torch.equal(merged2, merged)
    finally:
        tw.close()


def test_page_mass_and_eviction_bit_exact(cuda):
    """Config-5 style churn: the GPU's per-page attention mass matches the
    oracle's probabilities; given that mass, EMA scores, eviction choices,
    compaction and free-stack order are bit-exact."""
    torch = cuda
    tw = Twin(cuda, 2, layers=1, kv_heads=8, page_tokens=16, total_pages=400, max_seqs=8, max_pages=64,
              query_heads=32, perm_seed=5, seed=8)
    seqs = list(range(8))
    try:
        tw.prefill(seqs, [40, 100, 600, 33, 700, 129, 16, 500])
        rng = np.random.default_rng(4)
        for step in range(6):
            g, o, masses = tw.step(seqs, page_mass=True)
            assert_close(g, o, "churn outputs")
            mass = masses[0]
            # mass vs oracle token probabilities of the same step
            for s in seqs:
                L = int(tw.ora.lens()[s])
                _, probs = tw.ora.attention(s, 0, L, tw.row(1, s, 0, L - 1, 32 * 128), 32,
                                            1.0 / np.sqrt(128.0), want_probs=True)
                tok = probs.sum(axis=0)
                ref_mass = np.array([tok[p * 16:(p + 1) * 16].sum() for p in range((L + 15) // 16)])
                assert_close(mass[s, : len(ref_mass)], ref_mass, "page mass")
            flags = (rng.random(8) < 0.5).astype(np.uint8)
            budget = 96
            fl = torch.tensor(flags, device="cuda")
            ids = torch.tensor(seqs, dtype=torch.int32, device="cuda")
            tw.gpu.evict(8, torch.tensor(mass, device="cuda"), fl, budget, seq_ids=ids)
            tw.ora.evict(seqs, mass, flags, budget)
            assert tw.gpu.check() == 0
            tw.assert_state_equal()
            assert np.array_equal(tw.gpu.scores().view(np.uint32), tw.ora.scores().view(np.uint32))
        tw.assert_pages_equal()
    finally:
        tw.close()


@pytest.mark.parametrize("L", [3, 12])
def test_host_step_matches_device_step(cuda, L):
    """The e2e entry point (host buffers, copies inside) gives the same
    outputs as the device-resident path.  It moves the layers in chunks (the
    first and last alone, the rest in spans): 12 layers make spans of two."""
    import qwanto_b200 as qb
    torch = cuda
    B, H, HK = 4, 32, 8
    pools = [qb.KvPool(2, L, HK, 16, 300, B, 64, max_query_heads=H, permutation_seed=2) for _ in range(2)]
    try:
        for p in pools:
            p.prefill_synthetic(list(range(B)), [100, 7, 300, 64], 6)
        gen = torch.Generator().manual_seed(0)
        hq = torch.randn((L, B, H * 128), generator=gen).pin_memory()
        hk = torch.randn((L, B, HK * 128), generator=gen).pin_memory()
        hv = torch.randn((L, B, HK * 128), generator=gen).pin_memory()
        ho = torch.zeros((L, B, H * 128)).pin_memory()
        pools[0].decode_step_host(L, B, H, hq, hk, hv, ho)
        dq, dk, dv = hq.cuda(), hk.cuda(), hv.cuda()
        outs = torch.zeros((L, B, H * 128), device="cuda")
        pools[1].seq_append(B)
        for layer in range(L):
            pools[1].decode(layer, B, H, dq[layer], outs[layer], key=dk[layer], value=dv[layer])
        torch.cuda.synchronize()
        assert np.array_equal(ho.numpy(), outs.cpu().numpy())
        assert np.array_equal(pools[0].page_table(), pools[1].page_table())
    finally:
        for p in pools:
            p.close()


# -------------------------------------------------------------- ABI v1 ---

def _cpu_attention_q8(keys, values, ks, vs, query, H, HK, hd, pos, scale):
    """The CPU restatement inside c/tests/test_cuda_q8_kv.cu:40-80."""
    ch = HK * hd
    blocks = (ch + 63) // 64
    out = np.zeros(H * hd, np.float32)
    for h in range(H):
        kvh = (h * HK) // H
        off = kvh * hd
        sc = np.zeros(pos + 1, np.float32)
        for t in range(pos + 1):
            d = np.float32(0)
            for c in range(hd):
                a = off + c
                d = np.float32(d + np.float32(query[h * hd + c] * np.float32(keys[t * ch + a]) * ks[t * blocks + a // 64]))
            sc[t] = d * np.float32(scale)
        mx = sc.max()
        e = np.exp(sc - mx).astype(np.float32)
        inv = np.float32(1) / e.sum(dtype=np.float32)
        for c in range(hd):
            a = off + c
            r = np.float32(0)
            for t in range(pos + 1):
                r = np.float32(r + e[t] * np.float32(values[t * ch + a]) * vs[t * blocks + a // 64])
            out[h * hd + c] = r * inv
    return out


@pytest.mark.parametrize("head_dim", [4, 128])
@pytest.mark.parametrize("H,HK", [(4, 2), (6, 4), (12, 8), (2, 4)])
def test_abi_v1_mirrors_reference_cuda_q8_test(cuda, oracle_mod, head_dim, H, HK):
    """c/tests/test_cuda_q8_kv.cu:82-167 through the ABI v1 entry points:
    2 tokens, 4 query heads, 2 kv heads, scale 0.5; max error <= 1e-4 and the
    resident bytes return to 0 after destroy.  head_dim 4 runs the generic
    kernels, head_dim 128 the paged B200 kernels.  The other head counts map
    query head h to kv head h * HK / H unevenly, as the reference allows (the
    paged path pads the groups)."""
    import qwanto_b200 as qb
    ctx = qb.CudaContext(0)
    try:
        tokens, hd = 2, head_dim
        ch = HK * hd
        cache = ctx.kv_cache_create(8, HK, hd)
        key = np.array([(i - 3) * 0.17 for i in range(tokens * ch)], np.float32)
        value = np.array([(i + 2) * -0.11 for i in range(tokens * ch)], np.float32)
        query = np.array([(i - 5) * 0.09 for i in range(H * hd)], np.float32)
        qk, qv = np.zeros(tokens * ch, np.int8), np.zeros(tokens * ch, np.int8)
        nb = (ch + 63) // 64
        ks, vs = np.zeros(tokens * nb, np.float32), np.zeros(tokens * nb, np.float32)
        launches = 0
        for t in range(tokens):
            c, s = oracle_mod.q8_b64(key[t * ch:(t + 1) * ch])
            qk[t * ch:(t + 1) * ch], ks[t * nb:(t + 1) * nb] = c, s
            c, s = oracle_mod.q8_b64(value[t * ch:(t + 1) * ch])
            qv[t * ch:(t + 1) * ch], vs[t * nb:(t + 1) * nb] = c, s
            tel = ctx.kv_cache_append(cache, key[t * ch:(t + 1) * ch], value[t * ch:(t + 1) * ch], t)
        expected = _cpu_attention_q8(qk, qv, ks, vs, query, H, HK, hd, tokens - 1, 0.5)
        got, tel = ctx.kv_cache_attention(cache, query, H, HK, hd, tokens - 1, 0.5)
        assert np.abs(got - expected).max() <= 1e-4
        # the reference test requires kernel_count >= 5 after 2 appends + 1 attention
        assert tel.kv_cache_kernel_count >= 5 and tel.kv_cache_resident_bytes > 0
        with pytest.raises(qb.QwnCudaError):  # token must equal the cache length
            ctx.kv_cache_append(cache, key[:ch], value[:ch], 0)
        ctx.kv_cache_destroy(cache)
        assert ctx.telemetry().kv_cache_resident_bytes == 0
    finally:
        ctx.close()


def test_abi_v1_decoder_sequence(cuda, oracle_mod):
    """The decoder's per-layer call pattern (c/qwanto_decode.c:1658-1724):
    append token pos then attend at pos, Qwen2-1.5B shapes (12/2/128);
    outputs vs the reference-codec oracle within tolerance."""
    import qwanto_b200 as qb
    H, HK, hd, n = 12, 2, 128, 70
    ctx = qb.CudaContext(0)
    ora = oracle_mod.Pool(1, 1, HK, 16, 8, 1, 8)
    try:
        cache = ctx.kv_cache_create(128, HK, hd)
        rng = np.random.default_rng(0)
        for pos in range(n):
            k = rng.standard_normal(HK * hd).astype(np.float32)
            v = rng.standard_normal(HK * hd).astype(np.float32)
            q = rng.standard_normal(H * hd).astype(np.float32)
            ctx.kv_cache_append(cache, k, v, pos)
            assert ora.append([0], [1]) == 0 and ora.write(0, 0, pos, k, v) == 0
            if pos % 7 == 0 or pos == n - 1:
                got, _ = ctx.kv_cache_attention(cache, q, H, HK, hd, pos, 1.0 / np.sqrt(hd))
                ref = ora.attention(0, 0, pos + 1, q, H, 1.0 / np.sqrt(hd))
                assert_close(got.reshape(H, hd), ref, f"pos {pos}")
        # attention over a prefix (position < tokens-1) is allowed by the ABI
        got, _ = ctx.kv_cache_attention(cache, q, H, HK, hd, 20, 1.0 / np.sqrt(hd))
        assert_close(got.reshape(H, hd), ora.attention(0, 0, 21, q, H, 1.0 / np.sqrt(hd)), "prefix")
        ctx.kv_cache_reset(cache)
        with pytest.raises(qb.QwnCudaError):
            ctx.kv_cache_attention(cache, q, H, HK, hd, 0, 1.0)
        ctx.kv_cache_destroy(cache)
    finally:
        ctx.close()


def _hvsq2_numpy(w, act, scales, cols):
    """The 74-byte HyperVSQ-2 block arithmetic (c/cuda/qwn_hypervsq2_cuda_abi.cu:225-289)
    in float64: per weight (q-1)*a*base*sub/8 + a*offset, times the token scale."""
    rows, nblk, _ = w.shape
    # the reference decodes the fp16 base and offset with subnormals flushed
    # to zero (half_to_float, c/cuda/qwn_hypervsq2_cuda_abi.cu:111-126)
    ftz = lambda x: np.where(np.abs(x) < 2.0 ** -14, 0.0, x)
    base = ftz(w[:, :, 0:2].copy().view(np.float16)[:, :, 0].astype(np.float64))
    offs = ftz(w[:, :, 2:4].copy().view(np.float16)[:, :, 0].astype(np.float64))
    sub = np.zeros((rows, nblk, 8), np.float64)
    for o in range(8):
        sb = w[:, :, 4 + o // 2]
        sub[:, :, o] = (sb >> 4) if o & 1 else (sb & 15)
    codes = np.zeros((rows, nblk, 256), np.float64)
    for e in range(256):
        codes[:, :, e] = (w[:, :, 10 + e // 4] >> (2 * (e % 4))) & 3
    eff = base[:, :, None] * np.repeat(sub, 32, axis=2) / 8.0          # [rows][nblk][256]
    wt = (codes - 1.0) * eff + offs[:, :, None]
    wt = wt.reshape(rows, nblk * 256)[:, :cols]
    return (act.astype(np.float64) @ wt.T) * scales[:, None].astype(np.float64)


@pytest.mark.parametrize("rows,cols,batch", [(300, 1000, 11), (64, 4096, 1), (129, 256, 9)])
def test_hypervsq2_gemm_shapes(cuda, rows, cols, batch):
    """The GEMV/GEMM over ragged column counts, batches larger than one pass of
    staged tokens and a single full block, against the format in numpy."""
    import qwanto_b200 as qb
    from qwanto_b200 import _lib
    rng = np.random.default_rng(rows + cols + batch)
    nblk = (cols + 255) // 256
    w = rng.integers(0, 256, size=(rows, nblk, 74), dtype=np.uint8)
    w[:, :, 0:2] = (rng.random((rows, nblk)) * 0.01 + 0.001).astype(np.float16).view(np.uint8).reshape(rows, nblk, 2)
    w[:, :, 2:4] = (rng.random((rows, nblk)) * 0.002 - 0.001).astype(np.float16).view(np.uint8).reshape(rows, nblk, 2)
    act = rng.integers(-127, 128, size=(batch, cols), dtype=np.int8)
    scales = (rng.random(batch) + 0.5).astype(np.float32)
    ref = _hvsq2_numpy(w, act, scales, cols)
    ctx = qb.CudaContext(0)
    try:
        up = _lib.init(_lib.TensorUpload())
        wb = np.ascontiguousarray(w.reshape(-1))
        up.host_data, up.data_bytes, up.dtype, up.rows, up.cols, up.block_bytes = wb.ctypes.data, wb.size, 1, rows, cols, 74
        th = _lib.init(_lib.Handle())
        _lib.check("upload", qb.lib().qwn_cuda_abi_upload_tensor(C.byref(ctx.h), C.byref(up), C.byref(th)))
        for _ in range(2):
            out = np.zeros((batch, rows), np.float32)
            rq = _lib.init(_lib.GemmRequest())
            rq.tensor, rq.input_q8 = th, act.ctypes.data
            rq.input_scales = scales.ctypes.data_as(C.POINTER(C.c_float))
            rq.output = out.ctypes.data_as(C.POINTER(C.c_float))
            rq.batch, rq.rows, rq.cols, rq.input_mode = batch, rows, cols, 1
            tel = _lib.init(_lib.Telemetry())
            _lib.check("gemm", qb.lib().qwn_cuda_abi_hypervsq2_gemm(C.byref(ctx.h), C.byref(rq), C.byref(tel)))
            np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-3)
        _lib.check("release", qb.lib().qwn_cuda_abi_release_tensor(C.byref(ctx.h), C.byref(th)))
    finally:
        ctx.close()


def test_hypervsq2_gemv_matches_reference_cpu(cuda, oracle_mod):
    """HyperVSQ-2 74-byte GEMV (required for qwnrun to load the library)
    against the format's arithmetic restated in numpy."""
    import qwanto_b200 as qb
    from qwanto_b200 import _lib
    rng = np.random.default_rng(1)
    rows, cols, batch = 37, 700, 3
    nblk = (cols + 255) // 256
    w = rng.integers(0, 256, size=(rows, nblk, 74), dtype=np.uint8)
    w[:, :, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    w[:, :, 2:4] = np.frombuffer(np.float16(-0.002).tobytes(), np.uint8)
    act = rng.integers(-127, 128, size=(batch, cols), dtype=np.int8)
    scales = rng.random(batch).astype(np.float32)
    ref = np.zeros((batch, rows), np.float64)
    for r in range(rows):
        for b in range(nblk):
            base, off = float(np.float16(0.01)), float(np.float16(-0.002))
            for o in range(8):
                sb = w[r, b, 4 + o // 2]
                sub = (sb >> 4) if o & 1 else (sb & 15)
                eff = base * sub / 8.0
                for lane in range(32):
                    e = b * 256 + o * 32 + lane
                    if e >= cols:
                        continue
                    q = (w[r, b, 10 + o * 8 + lane // 4] >> ((lane & 3) * 2)) & 3
                    ref[:, r] += (q - 1.0) * act[:, e] * eff + act[:, e] * off
    ref *= scales[:, None]
    ctx = qb.CudaContext(0)
    try:
        up = _lib.init(_lib.TensorUpload())
        wb = np.ascontiguousarray(w.reshape(-1))
        up.host_data, up.data_bytes, up.dtype, up.rows, up.cols, up.block_bytes = wb.ctypes.data, wb.size, 1, rows, cols, 74
        th = _lib.init(_lib.Handle())
        _lib.check("upload", qb.lib().qwn_cuda_abi_upload_tensor(C.byref(ctx.h), C.byref(up), C.byref(th)))
        out = np.zeros((batch, rows), np.float32)
        rq = _lib.init(_lib.GemmRequest())
        rq.tensor, rq.input_q8 = th, act.ctypes.data
        rq.input_scales = scales.ctypes.data_as(C.POINTER(C.c_float))
        rq.output = out.ctypes.data_as(C.POINTER(C.c_float))
        rq.batch, rq.rows, rq.cols, rq.input_mode = batch, rows, cols, 1
        tel = _lib.init(_lib.Telemetry())
        _lib.check("gemm", qb.lib().qwn_cuda_abi_hypervsq2_gemm(C.byref(ctx.h), C.byref(rq), C.byref(tel)))
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-3)
        _lib.check("release", qb.lib().qwn_cuda_abi_release_tensor(C.byref(ctx.h), C.byref(th)))
    finally:
        ctx.close()


@pytest.mark.parametrize("codec", [2, 4, 5])
def test_back_to_back_layer_launches_parity(cuda, codec):
    """The layers of a step launched back to back on one stream, as a decoder
    issues them: each launch starts its setup, tile stream and fused append
    while the previous layer's kernel finishes (early start), the first
    launch after the page allocation records the step's plan while the
    second may already read it.  Every layer's output equals the oracle,
    tables and pages stay bit-exact; then the same step with one output
    buffer shared by all layers (which disables the early start) leaves the
    last layer's rows in it."""
    import qwanto_b200 as qb
    torch = cuda
    L, H, HK = 6, 32, 8
    lens = [1500, 37, 900, 2100, 1, 640, 1203, 16]
    n = len(lens)
    tw = Twin(cuda, codec, layers=L, kv_heads=HK, page_tokens=16, total_pages=800, max_seqs=n, max_pages=160,
              query_heads=H, perm_seed=9, seed=17)
    try:
        tw.prefill(list(range(n)), lens)
        W, Wq = HK * 128, H * 128
        ids = torch.arange(n, dtype=torch.int32, device="cuda")
        for step in range(3):
            tw.gpu.seq_append(n)
            assert tw.ora.append(list(range(n)), [1] * n) == 0
            pos_host = tw.ora.lens().copy() - 1
            pos = torch.tensor(pos_host, dtype=torch.int32, device="cuda")
            q = torch.empty((L, n, Wq), device="cuda")
            k = torch.empty((L, n, W), device="cuda")
            v = torch.empty((L, n, W), device="cuda")
            for layer in range(L):
                qb.generate_rows(q[layer], n, Wq, 1, tw.seed, layer, ids, pos)
                qb.generate_rows(k[layer], n, W, 2, tw.seed, layer, ids, pos)
                qb.generate_rows(v[layer], n, W, 3, tw.seed, layer, ids, pos)
            torch.cuda.synchronize()
            shared = step == 2
            out = torch.zeros((1 if shared else L, n, Wq), device="cuda")
            for layer in range(L):
                tw.gpu.decode(layer, n, H, q[layer], out[0 if shared else layer], key=k[layer], value=v[layer])
            torch.cuda.synchronize()
            assert tw.gpu.check() == 0
            for layer in range(L):
                for s in range(n):
                    p = int(pos_host[s])
                    assert tw.ora.write(s, layer, p, tw.row(2, s, layer, p, W), tw.row(3, s, layer, p, W)) == 0
                if shared and layer != L - 1:
                    continue
                ref = np.stack([tw.ora.attention(s, layer, int(pos_host[s]) + 1, tw.row(1, s, layer, int(pos_host[s]), Wq),
                                                 H, 1.0 / np.sqrt(128.0)) for s in range(n)])
                got = out[0 if shared else layer].cpu().numpy().reshape(n, H, 128)
                assert_close(got, ref, f"codec {codec} step {step} layer {layer}")
            tw.assert_state_equal()
        tw.assert_pages_equal()
    finally:
        tw.close()
