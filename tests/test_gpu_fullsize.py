"""Parity at the benchmark configurations' real sizes.

Each test builds the GPU pool exactly as bench.py does for one BASELINE
configuration (every layer, full batch, full context lengths, the same
lengths, seeds and page permutation) and runs one layer of it against the
CPU oracle:

* cfg2 -- 36 layers, 32 sequences U[1024, 8192], 32/8 heads, page 16, Q8
  per token-head: every sequence's outputs, pages and tables;
* cfg3 -- 36 layers, 64 sequences U[4096, 16384], 4-bit groups of 32 with
  the 1% x8 K outlier channels: 16 sampled sequences in full, tables of all;
* cfg4 -- one 131,072-token sequence, 48/8, page 64 (the two-level merge),
  plus the split over 2, 4 and 8 contiguous page ranges on one GPU;
* cfg1 -- all 256 decode steps from 2048 tokens, 12/2 heads;
* cfg5 -- the 1,048,576-page pool with 256 sequences and seeded p=0.05
  eviction for 12 steps: page tables, free stack, EMA scores and eviction
  sets bit-exact every step, given the GPU-exported page mass.

The oracle holds only the checked layer (it stores the synthetic rows of
GPU layer L in its layer 0), or only metadata for cfg5, so host memory stays
small.  Tolerance for fp32 outputs: |d| <= 1e-4 + 1e-3 |ref|.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

from kvharness import assert_close

pytestmark = pytest.mark.gpu


def _bench():
    import bench
    return bench


class BigTwin:
    """A full-size GPU pool and a one-layer (or metadata-only) oracle pool
    with the same tables: GPU layer `layer` <-> oracle layer 0."""

    def __init__(self, torch, wl, layer, total_pages, max_pages, perm_seed, seed, oracle_pages=True):
        import qwanto_b200 as qb
        from oracle import oracle as O
        self.torch, self.qb, self.O = torch, qb, O
        self.codec, self.L, self.H, self.HK, self.P = wl["codec"], wl["layers"], wl["H"], wl["HK"], wl["P"]
        self.layer, self.seed = layer, seed
        self.gpu = qb.KvPool(self.codec, self.L, self.HK, self.P, total_pages, wl["batch"], max_pages,
                             max_query_heads=self.H, permutation_seed=perm_seed)
        self.ora = O.Pool(self.codec, 1, self.HK, self.P, total_pages, wl["batch"], max_pages, perm_seed=perm_seed,
                          with_pages=oracle_pages)
        self.mask = _bench().outlier_masks(wl)

    def close(self):
        self.gpu.close()

    def krow(self, s, pos):
        r = self.O.gen_row(self.seed, 2, s, self.layer, pos, self.HK * 128)
        if self.mask is not None:
            r = np.where(self.mask[self.layer] != 0, r * np.float32(8), r).astype(np.float32)
        return r

    def prefill(self, lens, fill):
        n = len(lens)
        self.gpu.prefill_synthetic(list(range(n)), lens, self.seed, self.mask)
        assert self.ora.append(list(range(n)), list(lens)) == 0
        m = None if self.mask is None else self.mask[self.layer]
        for s in fill:
            assert self.ora.fill_synthetic(s, 0, self.layer, 0, int(lens[s]), self.seed, m) == 0

    def step(self, check, page_mass=False):
        """Every sequence grows by one token; layer `layer` appends and
        attends on the GPU (identity batch, as the bench calls it); the
        oracle writes and attends the `check` sequences.  Returns the GPU
        outputs [n][H][128], the oracle's for `check`, and the page mass."""
        torch, qb = self.torch, self.qb
        n = self.gpu.max_seqs
        self.gpu.seq_append(n)
        assert self.ora.append(list(range(n)), [1] * n) == 0
        lens = self.ora.lens().copy()
        pos = torch.tensor(lens - 1, dtype=torch.int32, device="cuda")
        ids = torch.arange(n, dtype=torch.int32, device="cuda")
        W, Wq = self.HK * 128, self.H * 128
        q = torch.empty((n, Wq), dtype=torch.float32, device="cuda")
        k = torch.empty((n, W), dtype=torch.float32, device="cuda")
        v = torch.empty((n, W), dtype=torch.float32, device="cuda")
        mask_dev = None if self.mask is None else torch.tensor(self.mask[self.layer], device="cuda")
        qb.generate_rows(q, n, Wq, 1, self.seed, self.layer, ids, pos)
        qb.generate_rows(k, n, W, 2, self.seed, self.layer, ids, pos, mask_dev)
        qb.generate_rows(v, n, W, 3, self.seed, self.layer, ids, pos)
        out = torch.zeros((n, Wq), dtype=torch.float32, device="cuda")
        pm = None
        if page_mass:
            pm = torch.zeros((n, self.gpu.max_pages_per_seq), dtype=torch.float32, device="cuda")
        self.gpu.decode(self.layer, n, self.H, q, out, key=k, value=v, page_mass=pm)
        torch.cuda.synchronize()
        ref = {}
        for s in check:
            p = int(lens[s]) - 1
            assert self.ora.write(s, 0, p, self.krow(s, p), self.O.gen_row(self.seed, 3, s, self.layer, p, W)) == 0
            ref[s] = self.ora.attention(s, 0, p + 1, self.O.gen_row(self.seed, 1, s, self.layer, p, Wq), self.H,
                                        1.0 / np.sqrt(128.0))
        return out.cpu().numpy().reshape(n, self.H, 128), ref, (None if pm is None else pm.cpu().numpy())

    def assert_tables_equal(self):
        g, o = self.gpu, self.ora
        assert np.array_equal(g.lens(), o.lens())
        assert np.array_equal(g.npages(), o.npages())
        assert np.array_equal(g.page_table(), o.page_table())
        assert np.array_equal(g.free_stack(), o.free_stack())

    def assert_layer_tiles_equal(self, seqs):
        """Every byte of layer `layer` of every page the sequences hold."""
        info = self.gpu.info
        span = self.HK * (self.P // 16) * int(info.tile_bytes)
        pages_o = self.ora.pages()
        table = self.ora.page_table()
        for s in seqs:
            for lp in range(int(self.ora.npages()[s])):
                pg = int(table[s, lp])
                gpu = self.qb.d2h(info.pages_dev + pg * int(info.page_bytes) + self.layer * span, (span,), np.uint8)
                if not np.array_equal(gpu, pages_o[pg, :span]):
                    bad = np.nonzero(gpu != pages_o[pg, :span])[0]
                    raise AssertionError(f"seq {s} page {lp} (physical {pg}): {bad.size} bytes differ, "
                                         f"first at {bad[:8]}")


def _pages_for(lens, P, extra):
    return int(sum((int(n) + extra + P - 1) // P for n in lens))


def test_cfg2_full_batch_one_layer(cuda):
    """36-layer pool, 32 sequences U[1024, 8192] (the bench's lengths), one
    decode step of the last layer: all outputs, pages and tables."""
    B = _bench()
    wl = B.workload(2)
    lens = B.global_lengths(wl, 1)
    tw = BigTwin(cuda, wl, layer=wl["layers"] - 1, total_pages=_pages_for(lens, 16, 2) + 64,
                 max_pages=(int(lens.max()) + 2 + 15) // 16 + 1, perm_seed=1000, seed=1000 * wl["seed"])
    try:
        tw.prefill(lens, fill=range(len(lens)))
        tw.assert_layer_tiles_equal(range(len(lens)))
        for _ in range(2):
            g, ref, _ = tw.step(check=range(len(lens)))
            for s, r in ref.items():
                assert_close(g[s], r, f"cfg2 seq {s} (len {int(tw.ora.lens()[s])})")
            assert tw.gpu.check() == 0
            tw.assert_tables_equal()
        tw.assert_layer_tiles_equal(range(len(lens)))
    finally:
        tw.close()


def test_cfg3_full_batch_q4_outliers_sampled(cuda):
    """36-layer pool, 64 sequences U[4096, 16384], 4-bit groups of 32 with
    the K outlier channels; 16 sampled sequences checked in full (outputs
    and every byte of their pages), the tables of all 64."""
    B = _bench()
    wl = B.workload(3)
    lens = B.global_lengths(wl, 1)
    sample = list(range(0, len(lens), 4))
    tw = BigTwin(cuda, wl, layer=17, total_pages=_pages_for(lens, 16, 1) + 64,
                 max_pages=(int(lens.max()) + 1 + 15) // 16 + 1, perm_seed=1000, seed=1000 * wl["seed"])
    try:
        tw.prefill(lens, fill=sample)
        g, ref, _ = tw.step(check=sample)
        for s, r in ref.items():
            assert_close(g[s], r, f"cfg3 seq {s} (len {int(tw.ora.lens()[s])})")
        assert tw.gpu.check() == 0
        tw.assert_tables_equal()
        tw.assert_layer_tiles_equal(sample)
    finally:
        tw.close()


def test_cfg4_long_sequence_and_page_range_splits(cuda):
    """131,072 tokens, 48/8 heads, page 64: the single-sequence decode (two-
    level merge) against the oracle, then the same step split over 2, 4 and 8
    contiguous page ranges on one GPU: each range's partial (m, l, o) merged
    equals the oracle, and the fused split kernel on a range equals that
    range's partial merged alone."""
    import qwanto_b200 as qb
    from qwanto_b200.exchange import PeerExchange
    from qwanto_b200.sharding import kv_ranges
    torch = cuda
    B = _bench()
    wl = B.workload(4)
    T = wl["lo"]
    H, P = wl["H"], wl["P"]
    tw = BigTwin(cuda, wl, layer=0, total_pages=T // P + 8, max_pages=T // P + 8, perm_seed=1000,
                 seed=1000 * wl["seed"])
    ex = PeerExchange(H, device=0, timeout_ns=1_000_000_000)
    try:
        tw.prefill(np.array([T]), fill=[0])
        g, ref, _ = tw.step(check=[0])
        assert_close(g[0], ref[0], "cfg4 full decode")
        assert tw.gpu.check() == 0
        tw.assert_tables_equal()
        tw.assert_layer_tiles_equal([0])
        Tn = T + 1
        pos = torch.tensor([Tn - 1], dtype=torch.int32, device="cuda")
        q = torch.empty((1, H * 128), dtype=torch.float32, device="cuda")
        qb.generate_rows(q, 1, H * 128, 1, tw.seed, 0, None, pos)
        for world in (2, 4, 8):
            ranges = kv_ranges(Tn, world, P)
            m = torch.zeros((world, H), device="cuda")
            l = torch.zeros((world, H), device="cuda")
            o = torch.zeros((world, H, 128), device="cuda")
            for r, (a, b) in enumerate(ranges):
                tw.gpu.partial(0, 1, H, q, m[r], l[r], o[r], t_begin=a, t_end=b)
            merged = torch.zeros((H, 128), device="cuda")
            qb.merge_partials(world, H, m, l, o, merged)
            torch.cuda.synchronize()
            assert_close(merged.cpu().numpy(), ref[0], f"cfg4 split x{world} merged")
            a, b = ranges[world // 2]
            alone = torch.zeros((H, 128), device="cuda")
            qb.merge_partials(1, H, m[world // 2:world // 2 + 1], l[world // 2:world // 2 + 1],
                              o[world // 2:world // 2 + 1], alone)
            fused = torch.full_like(q, float("nan"))
            tw.gpu.decode_split(0, H, q, fused, ex, t_begin=a, t_end=b)
            torch.cuda.synchronize()
            assert_close(fused.cpu().numpy().reshape(H, 128), alone.cpu().numpy(), f"cfg4 fused range x{world}")
            assert tw.gpu.check() == 0
    finally:
        torch.cuda.synchronize()
        ex.close()
        tw.close()


def test_cfg1_all_256_steps(cuda):
    """One sequence from 2048 tokens, 12/2 heads, 256 decode steps: every
    step's output, the tables after each step, every page at the end."""
    B = _bench()
    wl = B.workload(1)
    T0, steps = wl["lo"], wl["steps"]
    tw = BigTwin(cuda, wl, layer=0, total_pages=(T0 + steps) // 16 + 16, max_pages=(T0 + steps) // 16 + 8,
                 perm_seed=1000, seed=1000 * wl["seed"])
    try:
        tw.prefill(np.array([T0]), fill=[0])
        worst = 0.0
        for i in range(steps):
            g, ref, _ = tw.step(check=[0])
            assert_close(g[0], ref[0], f"cfg1 step {i}")
            worst = max(worst, float(np.max(np.abs(g[0] - ref[0]) / (1e-4 + 1e-3 * np.abs(ref[0])))))
            if i % 32 == 31:
                tw.assert_tables_equal()
        assert tw.gpu.check() == 0
        tw.assert_tables_equal()
        tw.assert_layer_tiles_equal([0])
        print(f"cfg1: 256 steps, worst error / tolerance {worst:.4f}")
    finally:
        tw.close()


def test_cfg5_million_page_pool_churn_bit_exact(cuda):
    """The 1,048,576-page pool, 256 sequences U[2048, 4096], 12 churn steps
    with the bench's seeded p=0.05 eviction triggers and the 2048-token
    budget: after every step the page tables, lengths, the whole free stack
    and the EMA scores equal the oracle's bit for bit, given the page mass
    the GPU exported in that step; the eviction sets (pages that left each
    table) are compared explicitly."""
    torch = cuda
    B = _bench()
    wl = B.workload(5)
    lens = B.global_lengths(wl, 1)
    n, P, steps = len(lens), wl["P"], 12
    max_pages = (int(lens.max()) + steps + 2 + P - 1) // P + 1
    tw = BigTwin(cuda, wl, layer=0, total_pages=wl["pool_pages"], max_pages=max_pages, perm_seed=5000,
                 seed=1000 * wl["seed"], oracle_pages=False)
    rng = np.random.default_rng(wl["seed"] * 7919)
    flags_host = (rng.random((steps, n)) < wl["evict_p"]).astype(np.uint8)
    evicted_total = 0
    try:
        tw.prefill(lens, fill=[])
        tw.assert_tables_equal()
        for s in range(steps):
            _, _, mass = tw.step(check=[], page_mass=True)
            before = tw.ora.page_table().copy()
            fl = torch.tensor(flags_host[s], device="cuda")
            tw.gpu.evict(n, torch.tensor(mass, device="cuda"), fl, wl["budget"])
            evicted_total += tw.ora.evict(list(range(n)), mass, flags_host[s], wl["budget"])
            assert tw.gpu.check() == 0
            tw.assert_tables_equal()
            assert np.array_equal(tw.gpu.scores().view(np.uint32), tw.ora.scores().view(np.uint32))
            after_g = tw.gpu.page_table()
            for i in np.nonzero(flags_host[s])[0]:
                gone_g = set(before[i][before[i] >= 0].tolist()) - set(after_g[i][after_g[i] >= 0].tolist())
                gone_o = set(before[i][before[i] >= 0].tolist()) - set(tw.ora.page_table()[i][tw.ora.page_table()[i] >= 0].tolist())
                assert gone_g == gone_o, f"step {s} seq {i}: eviction sets differ"
        assert evicted_total > 0 and int(flags_host.sum()) > 0
        print(f"cfg5: {int(flags_host.sum())} eviction triggers, {evicted_total} pages evicted in {steps} steps")
    finally:
        tw.close()


def _abi_lib(path):
    from qwanto_b200 import _lib
    P = C.POINTER
    L = C.CDLL(path, mode=os.RTLD_LOCAL)
    for fn, argt in (("qwn_cuda_abi_context_create", [P(_lib.ContextOptions), P(_lib.Handle)]),
                     ("qwn_cuda_abi_context_destroy", [P(_lib.Handle)]),
                     ("qwn_cuda_abi_upload_tensor", [P(_lib.Handle), P(_lib.TensorUpload), P(_lib.Handle)]),
                     ("qwn_cuda_abi_release_tensor", [P(_lib.Handle), P(_lib.Handle)]),
                     ("qwn_cuda_abi_hypervsq2_gemm", [P(_lib.Handle), P(_lib.GemmRequest), P(_lib.Telemetry)]),
                     ("qwn_cuda_abi_hypervsq2_gemv", [P(_lib.Handle), P(_lib.GemmRequest), P(_lib.Telemetry)])):
        getattr(L, fn).restype = C.c_int
        getattr(L, fn).argtypes = argt
    return L


def _run_gemm(L, w, act, scales, rows, cols, single):
    from qwanto_b200 import _lib
    o = _lib.init(_lib.ContextOptions())
    ctx = _lib.init(_lib.Handle())
    assert L.qwn_cuda_abi_context_create(C.byref(o), C.byref(ctx)) == 0
    try:
        wb = np.ascontiguousarray(w.reshape(-1))
        up = _lib.init(_lib.TensorUpload())
        up.host_data, up.data_bytes, up.dtype, up.rows, up.cols, up.block_bytes = wb.ctypes.data, wb.size, 1, rows, cols, 74
        th = _lib.init(_lib.Handle())
        assert L.qwn_cuda_abi_upload_tensor(C.byref(ctx), C.byref(up), C.byref(th)) == 0
        batch = act.shape[0]
        out = np.zeros((batch, rows), np.float32)
        rq = _lib.init(_lib.GemmRequest())
        rq.tensor, rq.input_q8 = th, act.ctypes.data
        rq.output = out.ctypes.data_as(C.POINTER(C.c_float))
        rq.batch, rq.rows, rq.cols = batch, rows, cols
        if single:
            rq.input_scale, rq.input_mode = float(scales[0]), 1
        else:
            rq.input_scales = scales.ctypes.data_as(C.POINTER(C.c_float))
            rq.input_mode = 1
        tel = _lib.init(_lib.Telemetry())
        fn = L.qwn_cuda_abi_hypervsq2_gemv if single else L.qwn_cuda_abi_hypervsq2_gemm
        assert fn(C.byref(ctx), C.byref(rq), C.byref(tel)) == 0
        L.qwn_cuda_abi_release_tensor(C.byref(ctx), C.byref(th))
        return out
    finally:
        L.qwn_cuda_abi_context_destroy(C.byref(ctx))


@pytest.mark.parametrize("rows,cols,batch", [(300, 1000, 1), (512, 4096, 1), (257, 2304, 11), (1024, 4096, 8)])
def test_hypervsq2_matches_reference_gpu_library(cuda, rows, cols, batch):
    """HyperVSQ-2 GEMV/GEMM pinned against the reference's own GPU library
    (oracle/_ref/qwn_cuda_ref.so, compiled from c/cuda/qwn_hypervsq2_cuda_abi.cu,
    whose kernel is :231-289), both called through ABI v1 on the same
    weights and int8 activations; the two differ only in fp32 summation
    order."""
    ref_path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                            "qwn_cuda_ref.so")
    if not os.path.exists(ref_path):
        pytest.skip("reference GPU library oracle/_ref/qwn_cuda_ref.so not built")
    import qwanto_b200
    rng = np.random.default_rng(rows * 7 + cols + batch)
    nblk = (cols + 255) // 256
    w = rng.integers(0, 256, size=(rows, nblk, 74), dtype=np.uint8)
    w[:, :, 0:2] = (rng.random((rows, nblk)) * 0.01 + 0.001).astype(np.float16).view(np.uint8).reshape(rows, nblk, 2)
    w[:, :, 2:4] = (rng.random((rows, nblk)) * 0.002 - 0.001).astype(np.float16).view(np.uint8).reshape(rows, nblk, 2)
    act = rng.integers(-127, 128, size=(batch, cols), dtype=np.int8)
    scales = (rng.random(batch) + 0.5).astype(np.float32)
    single = batch == 1
    ours = _run_gemm(_abi_lib(qwanto_b200._lib.LIB_PATH), w, act, scales, rows, cols, single)
    ref = _run_gemm(_abi_lib(ref_path), w, act, scales, rows, cols, single)
    np.testing.assert_allclose(ours, ref, rtol=1e-4, atol=1e-4 * float(np.abs(ref).max()))
