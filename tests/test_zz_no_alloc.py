"""qwn_kv_attention_static: decode attention that allocates nothing.

Some callers cannot allocate device memory when they run attention (a server
whose arena already owns the free HBM, a latency-critical loop that cannot
let cudaMalloc synchronise the device, an FFI caller holding only raw pool
pointers).  This entry point keeps its scratch in a fixed array inside the
library.  The test calls it through the C-ABI twice in a row and checks each
result against qwn_kv_decode on the same pool and query, within the
tolerance used for attention everywhere in this suite.  It lives in a file
that pytest collects last and must pass alone as well as after the others."""
import ctypes as C

import numpy as np
import pytest

from kvharness import assert_close

pytestmark = pytest.mark.gpu


def _static_request(pool, layer, num_seqs, query_heads, query, output, seq_ids=None):
    from qwanto_b200 import _lib
    r = _lib.init(_lib.StaticAttentionRequest())
    r.device_id, r.codec, r.layers, r.kv_heads, r.head_dim = pool.device, pool.codec, pool.layers, pool.kv_heads, 128
    r.page_tokens, r.total_pages, r.max_seqs = pool.page_tokens, pool.total_pages, pool.max_seqs
    r.max_pages_per_seq, r.layer, r.num_seqs, r.query_heads = pool.max_pages_per_seq, layer, num_seqs, query_heads
    r.scale = 0.0
    r.pages_dev, r.page_table_dev, r.seq_lens_dev = pool.info.pages_dev, pool.info.page_table_dev, pool.info.seq_lens_dev
    r.seq_ids_dev = None if seq_ids is None else seq_ids.data_ptr()
    r.query_dev, r.output_dev, r.status_dev = query.data_ptr(), output.data_ptr(), pool.info.status_dev
    r.stream = None
    return r


@pytest.mark.parametrize("codec,H", [(2, 32), (1, 32), (4, 32), (3, 32), (5, 32), (2, 64), (4, 64), (3, 64)])
def test_static_scratch_attention_matches_decode_twice(cuda, codec, H):
    """H = 32 runs 4 query heads per kv head (one head group), H = 64 runs 8
    (two head groups, the kernel variant with its own grid size)."""
    import qwanto_b200 as qb
    torch = cuda
    B, L, HK = 6, 2, 8
    lens = [1, 17, 300, 1500, 4000, 64]
    pool = qb.KvPool(codec, L, HK, 16, 600, B, 300, max_query_heads=H, permutation_seed=12)
    try:
        pool.prefill_synthetic(list(range(B)), lens, 31)
        ids = torch.tensor([4, 0, 5, 2, 1, 3], dtype=torch.int32, device="cuda")
        for call, layer in enumerate((1, 0)):  # two calls in a row, different layer and query
            q = torch.randn((B, H * 128), device="cuda", generator=torch.Generator("cuda").manual_seed(call))
            want = torch.zeros_like(q)
            pool.decode(layer, B, H, q, want, seq_ids=ids)
            got = torch.full_like(q, float("nan"))
            req = _static_request(pool, layer, B, H, q, got, ids)
            rc = qb.lib().qwn_kv_attention_static(C.byref(req))
            assert rc == 0, qb._lib.last_error()
            torch.cuda.synchronize()
            assert_close(got.cpu().numpy(), want.cpu().numpy(), f"static scratch call {call}")
        assert pool.check() == 0
    finally:
        pool.close()


def test_static_scratch_rejects_oversized_batch(cuda):
    import qwanto_b200 as qb
    torch = cuda
    pool = qb.KvPool(2, 1, 8, 16, 64, 40, 4, max_query_heads=8)
    try:
        q = torch.zeros((33, 8 * 128), device="cuda")
        out = torch.zeros_like(q)
        req = _static_request(pool, 0, 33, 8, q, out)  # 33 x 8 = 264 segments > 256
        assert qb.lib().qwn_kv_attention_static(C.byref(req)) == -5
        assert "256 segments" in qb._lib.last_error()
    finally:
        pool.close()
