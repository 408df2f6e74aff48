"""The C-ABI boundary, without a GPU: the library loads, exports every entry
point include/*.h declares, its structure layouts equal the reference's
(c/cuda/qwn_cuda_abi.h) and the loader checks qwnrun performs
(c/qwanto_decode.c:349-393) pass."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
from oracle.refpath import reference_c

_REF_C = reference_c()
REF_ABI = os.path.join(_REF_C, "cuda", "qwn_cuda_abi.h") if _REF_C else ""

STRUCTS = {
    "QwnCudaAbiHeader": ["struct_size", "abi_version", "reserved"],
    "QwnCudaAbiInfo": ["capability_bits", "max_devices", "hypervsq2_block_bytes", "abi_name"],
    "QwnCudaDeviceInfo": ["device_id", "total_vram_bytes", "free_vram_bytes", "name", "driver"],
    "QwnCudaContextOptions": ["device_id", "flags", "memory_budget_bytes", "context_size"],
    "QwnCudaContextHandle": ["opaque"],
    "QwnCudaKvCacheOptions": ["max_tokens", "kv_heads", "head_dim"],
    "QwnCudaKvAppendRequest": ["cache", "host_key", "host_value", "n_channels", "token"],
    "QwnCudaKvAttentionRequest": ["cache", "host_query", "host_output", "query_heads", "position", "scale"],
    "QwnCudaTensorUpload": ["host_data", "data_bytes", "dtype", "rows", "cols", "block_bytes"],
    "QwnCudaGemmRequest": ["tensor", "input_q8", "input_scale", "input_scales", "output", "batch",
                           "input_mode"],
    "QwnCudaTelemetry": ["gpu_kernel_ms", "device_id", "device_name", "kernel_type", "dll_hash",
                         "kv_cache_kernel_count", "kv_cache_resident_bytes", "kv_cache_kernel_type"],
}


def declared_symbols():
    names = []
    for h in ("qwn_cuda_abi.h", "qwn_kv_b200.h"):
        text = open(os.path.join(INCLUDE, h)).read()
        names += re.findall(r"QWN_CUDA_ABI_API\s+[\w\s\*]+?\b(qwn_\w+)\s*\(", text)
    return sorted(set(names))


def layout_probe(header_dir, header):
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{header}"', "int main(void){"]
    for s, fields in STRUCTS.items():
        lines.append(f'printf("{s} %zu\\n", sizeof({s}));')
        for f in fields:
            lines.append(f'printf("{s}.{f} %zu\\n", offsetof({s}, {f}));')
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "p.c"), os.path.join(d, "p")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-I", header_dir, src, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    return dict(line.rsplit(" ", 1) for line in out.strip().splitlines())


def test_library_exports_every_declared_symbol():
    import qwanto_b200
    L = qwanto_b200.lib()
    names = declared_symbols()
    assert len(names) >= 17 + 15
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_seventeen_qwnrun_symbols_declared():
    names = set(declared_symbols())
    qwnrun = ["query", "get_capabilities", "enumerate_devices", "context_create", "context_destroy",
              "upload_tensor", "release_tensor", "kv_cache_create", "kv_cache_destroy", "kv_cache_append",
              "kv_cache_attention", "kv_cache_reset", "hypervsq2_gemv", "hypervsq2_gemm", "synchronize",
              "get_telemetry", "last_error"]
    assert {"qwn_cuda_abi_" + n for n in qwnrun} <= names


def test_struct_layouts_match_ctypes_mirror():
    from qwanto_b200 import _lib
    ours = layout_probe(INCLUDE, "qwn_cuda_abi.h")
    mirror = {"QwnCudaAbiHeader": _lib.Header, "QwnCudaAbiInfo": _lib.AbiInfo,
              "QwnCudaDeviceInfo": _lib.DeviceInfo, "QwnCudaContextOptions": _lib.ContextOptions,
              "QwnCudaContextHandle": _lib.Handle, "QwnCudaKvCacheOptions": _lib.KvCacheOptions,
              "QwnCudaKvAppendRequest": _lib.KvAppendRequest, "QwnCudaKvAttentionRequest": _lib.KvAttentionRequest,
              "QwnCudaTensorUpload": _lib.TensorUpload, "QwnCudaGemmRequest": _lib.GemmRequest,
              "QwnCudaTelemetry": _lib.Telemetry}
    for name, cls in mirror.items():
        assert int(ours[name]) == C.sizeof(cls), name
        for f in STRUCTS[name]:
            assert int(ours[f"{name}.{f}"]) == getattr(cls, f).offset, f"{name}.{f}"


def test_linear_attention_state_layout():
    """QwnLinearAttentionState: the ctypes mirror matches the header, and the
    first three fields sit where QwantoLinearAttentionState keeps them
    (c/qwanto_attention.h:11-15: int, int, float *)."""
    from qwanto_b200 import _lib
    fields = ["n_heads", "head_dim", "state", "device_id", "reserved", "staging", "staging_bytes"]
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "qwn_kv_b200.h"', "int main(void){",
             'printf("size %zu\\n", sizeof(QwnLinearAttentionState));']
    lines += [f'printf("{f} %zu\\n", offsetof(QwnLinearAttentionState, {f}));' for f in fields]
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "p.c"), os.path.join(d, "p")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-I", INCLUDE, src, "-o", exe], check=True)
        out = dict(l.split() for l in subprocess.run([exe], check=True, capture_output=True,
                                                     text=True).stdout.strip().splitlines())
    assert int(out["size"]) == C.sizeof(_lib.LinearAttentionState)
    for f in fields:
        assert int(out[f]) == getattr(_lib.LinearAttentionState, f).offset, f
    assert (int(out["n_heads"]), int(out["head_dim"]), int(out["state"])) == (0, 4, 8)


def test_linear_attention_rejects_bad_arguments_without_gpu():
    from qwanto_b200 import _lib
    L = _lib.lib()
    st = _lib.LinearAttentionState()
    assert L.qwn_linear_attention_init(C.byref(st), 0, 0, 128) == -1
    assert L.qwn_linear_attention_init(C.byref(st), 0, 4, 0) == -1
    assert L.qwn_linear_attention_init(C.byref(st), 0, 4, 1024) == -5
    assert L.qwn_linear_attention_decode(C.byref(st), None, None, None, C.c_float(1.0), None, None) == -1


@pytest.mark.skipif(not os.path.exists(REF_ABI), reason="reference header not present")
def test_struct_layouts_identical_to_reference_header():
    ours = layout_probe(INCLUDE, "qwn_cuda_abi.h")
    ref = layout_probe(os.path.dirname(REF_ABI), "qwn_cuda_abi.h")
    assert ours == ref


def test_query_satisfies_qwnrun_loader_checks():
    """c/qwanto_decode.c:365-393: ABI 1, HyperVSQ-2 GEMV capability, 74/256,
    and the Q8 KV capability for --kv-cache q8."""
    import qwanto_b200
    from qwanto_b200 import _lib
    info = qwanto_b200.CudaContext.query()
    assert info.header.abi_version == 1 and info.header.struct_size >= C.sizeof(_lib.AbiInfo)
    assert info.capability_bits & _lib.CAP_HYPERVSQ2_GEMV and info.capability_bits & _lib.CAP_Q8_KV
    assert info.hypervsq2_block_bytes == 74 and info.hypervsq2_block_elements == 256
    assert info.capability_bits & _lib.CAP_PAGED_KV


def test_query_rejects_bad_header():
    import qwanto_b200
    from qwanto_b200 import _lib
    info = _lib.AbiInfo()
    info.header.struct_size = 8
    info.header.abi_version = 1
    assert qwanto_b200.lib().qwn_cuda_abi_query(C.byref(info)) == -1
    assert "invalid ABI query" in _lib.last_error()


def test_pool_create_rejects_bad_geometry_without_touching_gpu():
    """Argument validation happens on the host before any CUDA call."""
    import qwanto_b200
    from qwanto_b200 import _lib
    for kw in [dict(page_tokens=24), dict(codec=9), dict(total_pages=0)]:
        o = _lib.init(_lib.PoolOptions())
        o.codec, o.layers, o.kv_heads, o.head_dim = 2, 1, 2, 128
        o.page_tokens, o.total_pages, o.max_seqs, o.max_pages_per_seq = 16, 8, 1, 8
        for k, v in kw.items():
            setattr(o, k, v)
        h = _lib.init(_lib.Handle())
        assert qwanto_b200.lib().qwn_kv_pool_create(C.byref(o), C.byref(h)) == -1
    o = _lib.init(_lib.PoolOptions())
    o.codec, o.layers, o.kv_heads, o.head_dim = 2, 1, 2, 64
    o.page_tokens, o.total_pages, o.max_seqs, o.max_pages_per_seq = 16, 8, 1, 8
    h = _lib.init(_lib.Handle())
    assert qwanto_b200.lib().qwn_kv_pool_create(C.byref(o), C.byref(h)) == -1
    h.header.abi_version = 7
    assert qwanto_b200.lib().qwn_kv_pool_create(C.byref(o), C.byref(h)) == -2


def test_enumerate_without_device_reports_unavailable():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    import qwanto_b200
    rc, devs = qwanto_b200.CudaContext.devices()
    assert rc == -3 and devs == []


def test_static_attention_rejects_misaligned_pointers_without_gpu():
    """qwn_kv_attention_static takes raw device pointers from FFI callers: a
    pages pointer off the 16-byte grid (the tiles move by 1-D bulk copies) or
    a query/output pointer off it (16-byte loads and stores) is an argument
    error found on the host, before anything is launched.  The addresses
    below are never dereferenced."""
    import qwanto_b200
    from qwanto_b200 import _lib
    L = qwanto_b200.lib()
    base = 1 << 40

    def req(**kw):
        r = _lib.init(_lib.StaticAttentionRequest())
        r.device_id, r.codec, r.layers, r.kv_heads, r.head_dim = 0, 2, 1, 8, 128
        r.page_tokens, r.total_pages, r.max_seqs, r.max_pages_per_seq = 16, 64, 4, 16
        r.layer, r.num_seqs, r.query_heads = 0, 2, 32
        r.pages_dev, r.page_table_dev, r.seq_lens_dev = base, base + 4096, base + 8192
        r.query_dev, r.output_dev = base + 12288, base + 16384
        for k, v in kw.items():
            setattr(r, k, v)
        return r

    for kw in [dict(pages_dev=base + 4), dict(query_dev=base + 12288 + 8), dict(output_dev=base + 16384 + 4),
               dict(page_table_dev=base + 4096 + 2), dict(seq_lens_dev=base + 8192 + 1)]:
        r = req(**kw)
        assert L.qwn_kv_attention_static(C.byref(r)) == -1, kw
        assert "aligned" in _lib.last_error()
    r = req(codec=6)
    assert L.qwn_kv_attention_static(C.byref(r)) == -1
