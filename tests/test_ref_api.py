"""The reference-named C APIs of qwn_cuda.so without a GPU: every function
the reference headers declare is exported, the struct layouts and constants
of include/qwn_paged_kv.h, qwanto_turboquant.h, qwanto_attention.h and
qwanto_pagedeviction.h equal the reference headers', and the host-side parts
(cache mode and contract, block tables on a caller's free stack, chunked-
prefill scheduler, token-level eviction) give the reference library's
results bit for bit.  Calls that need a device fail loudly here."""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

from oracle.refpath import reference_c

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
REF_C = reference_c()
HEADERS = ["qwn_paged_kv.h", "qwanto_turboquant.h", "qwanto_attention.h", "qwanto_pagedeviction.h"]

LAYOUTS = {
    "QwnKVBlockPool": ["key_data", "val_data", "free_stack", "free_top", "total_blocks", "layers", "kv_heads",
                       "head_dim", "block_bytes"],
    "QwnBlockTable": ["req_id", "num_tokens", "max_tokens", "block_ids", "block_count", "block_capacity",
                      "prefill_remaining", "prefill_offset"],
    "QwnChunkedScheduler": ["max_chunk_tokens", "active_requests"],
    "QwnKvCacheContract": ["struct_size", "abi_version", "cache_dtype", "block_size", "scale_bytes",
                           "zero_point_bytes", "key_layout", "value_layout", "page_size", "alignment",
                           "valid_token_count", "reserved"],
    "TurboQuantBlock": ["scale_fp16", "zero_point_fp16", "packed_data"],
    "TurboQuantCache": ["packed_k", "packed_v", "n_channels", "n_tokens", "max_tokens", "n_heads", "head_dim",
                        "token_stride_k", "token_stride_v", "total_bytes"],
    "QwnQ8Cache": ["packed_k", "packed_v", "scales_k", "scales_v", "n_channels", "n_tokens", "max_tokens",
                   "n_heads", "head_dim", "token_stride", "scale_stride", "total_bytes", "contract"],
    "QwnVToken": ["token_id", "importance_score", "physical_slot", "is_sink", "is_active"],
    "QwnPagedEvictionPool": ["virtual_tokens", "active_count", "max_capacity", "physical_pool_size",
                             "eviction_threshold", "total_evictions"],
    "QwantoLinearAttentionState": ["n_heads", "head_dim", "state"],
}
CONSTANTS = ["QWN_PAGE_BLOCK_SIZE", "QWN_KV_PAGE_BYTES", "TURBOQUANT_GROUP_SIZE", "TURBOQUANT_BLOCK_BYTES",
             "TURBOQUANT_PAYLOAD_BYTES", "QWN_KV_CACHE_ABI_VERSION", "QWN_KV_CACHE_PAGE_SIZE",
             "QWN_KV_CACHE_FP16", "QWN_KV_CACHE_Q8", "QWN_KV_CACHE_TURBOQUANT_Q4", "QWN_KV_CACHE_AUTO",
             "QWN_VTOKEN_MAX_CAPACITY", "QWN_VTOKEN_SINK_TOKENS"]


def _probe(include_dir):
    lines = ["#include <stdio.h>", "#include <stddef.h>"] + [f'#include "{h}"' for h in HEADERS]
    lines.append("int main(void){")
    for s, fields in LAYOUTS.items():
        lines.append(f'printf("{s} %zu\\n", sizeof({s}));')
        lines += [f'printf("{s}.{f} %zu\\n", offsetof({s}, {f}));' for f in fields]
    lines += [f'printf("{c} %lld\\n", (long long)({c}));' for c in CONSTANTS]
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "p.c"), os.path.join(d, "p")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-I", include_dir, src, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    return dict(line.rsplit(" ", 1) for line in out.strip().splitlines())


def declared(header_dir):
    names = []
    for h in HEADERS:
        text = open(os.path.join(header_dir, h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(qwn_\w+|qwanto_\w+)\s*\(", text)
    return sorted(set(names))


def test_every_reference_function_exported():
    import qwanto_b200
    L = qwanto_b200.lib()
    ours = declared(INCLUDE)
    assert len(ours) >= 45
    assert not [n for n in ours if not hasattr(L, n)]
    if REF_C:
        ref = declared(REF_C)
        assert set(ref) <= set(ours), sorted(set(ref) - set(ours))


@pytest.mark.skipif(REF_C is None, reason="reference headers not present")
def test_layouts_and_constants_equal_reference_headers():
    assert _probe(INCLUDE) == _probe(REF_C)


def _decl(L, name, res, *args):
    f = getattr(L, name)
    f.restype, f.argtypes = res, list(args)
    return f


@pytest.fixture(scope="module")
def both(oracle_mod, ref_lib):
    """(this library, the reference library) with the host-side calls declared."""
    import qwanto_b200
    O = oracle_mod
    out = []
    for L in (qwanto_b200.lib(), ref_lib):
        _decl(L, "qwn_paged_eviction_init", C.c_int, C.POINTER(O.EvictionPool), C.c_uint32, C.c_uint32, C.c_float)
        _decl(L, "qwn_paged_eviction_insert", C.c_int, C.POINTER(O.EvictionPool), C.c_uint32, C.c_float,
              C.POINTER(C.c_uint32))
        _decl(L, "qwn_paged_eviction_update_scores", None, C.POINTER(O.EvictionPool), O.f32p, C.c_uint32)
        _decl(L, "qwn_paged_eviction_prune", C.c_uint32, C.POINTER(O.EvictionPool), C.c_uint32)
        _decl(L, "qwn_paged_eviction_memory_waste_pct", C.c_float, C.POINTER(O.EvictionPool))
        _decl(L, "qwn_kv_cache_mode_parse", C.c_int, C.c_char_p, C.POINTER(C.c_int))
        _decl(L, "qwn_kv_cache_mode_name", C.c_char_p, C.c_int)
        _decl(L, "qwn_kv_cache_contract_init", None, C.POINTER(O.KvContract), C.c_int, C.c_uint32)
        _decl(L, "qwn_kv_pool_alloc_block", C.c_int, C.POINTER(O.RefBlockPool))
        _decl(L, "qwn_kv_pool_free_block", None, C.POINTER(O.RefBlockPool), C.c_int)
        _decl(L, "qwn_block_table_init", C.c_int, C.POINTER(O.RefBlockTable), C.c_int, C.c_int)
        _decl(L, "qwn_block_table_append_token", C.c_int, C.POINTER(O.RefBlockPool), C.POINTER(O.RefBlockTable))
        _decl(L, "qwn_block_table_free", None, C.POINTER(O.RefBlockPool), C.POINTER(O.RefBlockTable))
        out.append(L)
    return out


def test_token_eviction_bit_exact_vs_reference(oracle_mod, both):
    """c/qwanto_pagedeviction.c:7-103 on random insert / update / prune
    sequences: return codes, slots, active flags, EMA scores (bit for bit)
    and eviction counts equal the reference library's."""
    ours, ref = both
    rng = np.random.default_rng(11)
    for trial in range(60):
        cap = int(rng.integers(20, 400))
        phys = int(rng.integers(10, cap + 5))
        thr = float(rng.choice([0.0, 0.05, 0.3, -1.0]))
        a, b = oracle_mod.EvictionPool(), oracle_mod.EvictionPool()
        assert ours.qwn_paged_eviction_init(C.byref(a), cap, phys, thr) == ref.qwn_paged_eviction_init(
            C.byref(b), cap, phys, thr)
        sa, sb = C.c_uint32(0), C.c_uint32(0)
        for _ in range(int(rng.integers(5, 500))):
            op = int(rng.integers(0, 4))
            if op <= 1:
                tid, imp = int(rng.integers(0, 1000)), float(rng.standard_normal())
                assert ours.qwn_paged_eviction_insert(C.byref(a), tid, imp, C.byref(sa)) == \
                    ref.qwn_paged_eviction_insert(C.byref(b), tid, imp, C.byref(sb))
                assert sa.value == sb.value
            elif op == 2:
                sc = (rng.random(500) * rng.choice([1.0, 1e-3, 50.0])).astype(np.float32)
                n = int(rng.integers(0, 500))
                p = oracle_mod._ptr(sc, oracle_mod.f32p)
                ours.qwn_paged_eviction_update_scores(C.byref(a), p, n)
                ref.qwn_paged_eviction_update_scores(C.byref(b), p, n)
            else:
                t = int(rng.integers(0, cap))
                assert ours.qwn_paged_eviction_prune(C.byref(a), t) == ref.qwn_paged_eviction_prune(C.byref(b), t)
        assert bytes(a) == bytes(b), f"trial {trial}: pools differ"
        assert ours.qwn_paged_eviction_memory_waste_pct(C.byref(a)) == \
            ref.qwn_paged_eviction_memory_waste_pct(C.byref(b))
    assert ours.qwn_paged_eviction_init(None, 1, 1, 0.1) == -1
    assert ours.qwn_paged_eviction_insert(None, 0, 1.0, None) == -1


def test_mode_and_contract_vs_reference(oracle_mod, both):
    ours, ref = both
    for text in [b"fp16", b"q8", b"turboquant-q4", b"qwn-q4-kv", b"auto", b"Q8", b"", b"int4"]:
        ma, mb = C.c_int(-7), C.c_int(-7)
        assert ours.qwn_kv_cache_mode_parse(text, C.byref(ma)) == ref.qwn_kv_cache_mode_parse(text, C.byref(mb))
        assert ma.value == mb.value
    for mode in range(-1, 5):
        assert ours.qwn_kv_cache_mode_name(mode) == ref.qwn_kv_cache_mode_name(mode)
        a, b = oracle_mod.KvContract(), oracle_mod.KvContract()
        ours.qwn_kv_cache_contract_init(C.byref(a), mode, 77)
        ref.qwn_kv_cache_contract_init(C.byref(b), mode, 77)
        assert bytes(a) == bytes(b)


def test_block_tables_on_a_caller_free_stack_vs_reference(oracle_mod, both):
    """qwn_kv_pool_alloc_block / free_block and the block-table calls are
    integer bookkeeping on the caller's structs: on the same (permuted) free
    stack, random appends, frees and re-inits give the same tables, free
    stacks and return codes as c/qwn_paged_kv.c:95-149."""
    ours, ref = both
    O = oracle_mod
    rng = np.random.default_rng(2)
    total = 61
    stacks, pools, tabs = [], [], []
    for L in (ours, ref):
        st = O.free_stack(9, total).astype(np.int32)
        p = O.RefBlockPool()
        p.free_stack = st.ctypes.data_as(O.i32p)
        p.free_top, p.total_blocks, p.layers, p.kv_heads, p.head_dim = total, total, 1, 1, 8
        ts = [O.RefBlockTable() for _ in range(5)]
        for i, t in enumerate(ts):
            assert L.qwn_block_table_init(C.byref(t), i, int(rng.integers(0, 6))) == 0
        stacks.append(st)
        pools.append(p)
        tabs.append(ts)
    rng = np.random.default_rng(3)
    for _ in range(900):
        s, op = int(rng.integers(0, 5)), int(rng.integers(0, 20))
        if op == 0:
            for L, p, ts in zip((ours, ref), pools, tabs):
                L.qwn_block_table_free(C.byref(p), C.byref(ts[s]))
                assert L.qwn_block_table_init(C.byref(ts[s]), s, 4) == 0
        elif op == 1:
            blk = int(rng.integers(-2, total + 2))
            for L, p in zip((ours, ref), pools):
                L.qwn_kv_pool_free_block(C.byref(p), blk)
        else:
            rcs = [L.qwn_block_table_append_token(C.byref(p), C.byref(ts[s])) for L, p, ts in zip((ours, ref), pools, tabs)]
            assert rcs[0] == rcs[1]
        assert pools[0].free_top == pools[1].free_top
        assert np.array_equal(stacks[0][: pools[0].free_top], stacks[1][: pools[1].free_top])
    for s in range(5):
        a, b = tabs[0][s], tabs[1][s]
        assert (a.num_tokens, a.block_count, a.block_capacity) == (b.num_tokens, b.block_count, b.block_capacity)
        assert np.array_equal(np.ctypeslib.as_array(a.block_ids, shape=(a.block_count,)),
                              np.ctypeslib.as_array(b.block_ids, shape=(b.block_count,)))
    for L, p, ts in zip((ours, ref), pools, tabs):
        for t in ts:
            L.qwn_block_table_free(C.byref(p), C.byref(t))


def test_scheduler_next_chunk():
    """c/qwn_paged_kv.c:384-396: 1 token for a decode step, else the
    remaining prompt capped at max_chunk_tokens (512 when given <= 0)."""
    import qwanto_b200
    from oracle import oracle as O
    L = qwanto_b200.lib()

    class Sched(C.Structure):
        _fields_ = [("max_chunk_tokens", C.c_int), ("active_requests", C.c_int)]
    s = Sched()
    _decl(L, "qwn_scheduler_init", None, C.POINTER(Sched), C.c_int)
    _decl(L, "qwn_scheduler_next_chunk", C.c_int, C.POINTER(Sched), C.POINTER(O.RefBlockTable))
    L.qwn_scheduler_init(C.byref(s), 0)
    assert (s.max_chunk_tokens, s.active_requests) == (512, 0)
    L.qwn_scheduler_init(C.byref(s), 100)
    bt = O.RefBlockTable()
    for rem, want in [(0, 1), (-3, 1), (40, 40), (100, 100), (101, 100), (5000, 100)]:
        bt.prefill_remaining = rem
        assert L.qwn_scheduler_next_chunk(C.byref(s), C.byref(bt)) == want
    assert L.qwn_scheduler_next_chunk(None, C.byref(bt)) == 0


def test_device_calls_fail_loudly_without_gpu():
    """No CUDA device: the calls that allocate device memory return -1
    instead of running anything on the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    import qwanto_b200
    from oracle import oracle as O
    L = qwanto_b200.lib()
    _decl(L, "qwn_q8_cache_init", C.c_int, C.POINTER(O.RefQ8Cache), C.c_int, C.c_int, C.c_int)
    _decl(L, "qwn_kv_pool_init", C.c_int, C.POINTER(O.RefBlockPool), C.c_int, C.c_int, C.c_int, C.c_int)
    _decl(L, "qwanto_linear_attention_init", C.c_int, C.POINTER(O.RefLinearState), C.c_int, C.c_int)
    assert L.qwn_q8_cache_init(C.byref(O.RefQ8Cache()), 16, 2, 64) == -1
    assert L.qwn_kv_pool_init(C.byref(O.RefBlockPool()), 8, 1, 2, 128) == -1
    assert L.qwanto_linear_attention_init(C.byref(O.RefLinearState()), 2, 64) == -1
