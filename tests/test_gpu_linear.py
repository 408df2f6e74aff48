"""Linear-attention decode/prefill on the GPU (qwn_linear_attention_*) against
the oracle's restatement of c/qwanto_attention.c:34-156 and, where the
reference CPU library was built, the reference itself: states and outputs
bit-identical, over several steps, ragged prefill chunks, head dims that do
not fill a 32-column block, batched heads, reset and the host-buffer call."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _oracle_steps(oracle_mod, state, q, k, v, decay):
    """Run the oracle token by token; returns outputs [T][H][D] (state updated in place)."""
    T, H, D = q.shape
    out = np.zeros((T, H, D), np.float32)
    for t in range(T):
        o = np.zeros((H, D), np.float32)
        oracle_mod.lib().qor_linear_attention_decode(_f(state), H, D, _f(np.ascontiguousarray(q[t])),
                                                     _f(np.ascontiguousarray(k[t])),
                                                     _f(np.ascontiguousarray(v[t])), C.c_float(decay), _f(o))
        out[t] = o
    return out


def _inputs(rng, T, H, D, scale=1.0):
    return [(rng.standard_normal((T, H, D)) * scale).astype(np.float32) for _ in range(3)]


def _state_of(torch, st):
    """Copy the device state back to the host ([n_heads][head_dim][head_dim])."""
    import qwanto_b200
    torch.cuda.synchronize()
    host = np.empty((st.n_heads, st.head_dim, st.head_dim), np.float32)
    assert qwanto_b200.lib().qwn_kv_memcpy_d2h(host.ctypes.data, st.state_ptr, host.nbytes) == 0
    return host


@pytest.mark.parametrize("H,D", [(4, 128), (3, 64), (2, 256), (1, 512), (5, 24), (2, 8), (2, 96), (3, 4), (300, 32)])
def test_decode_steps_bit_exact(cuda, oracle_mod, H, D):
    from qwanto_b200.linear_attention import LinearAttentionState
    torch = cuda
    rng = np.random.default_rng(H * 1000 + D)
    T, decay = 5, 0.9375
    q, k, v = _inputs(rng, T, H, D)
    ref_state = np.zeros((H, D, D), np.float32)
    ref_out = _oracle_steps(oracle_mod, ref_state, q, k, v, decay)
    with LinearAttentionState(H, D) as st:
        qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
        od = torch.full((T, H, D), float("nan"), device="cuda")
        for t in range(T):
            st.decode(qd[t], kd[t], vd[t], decay, od[t])
        torch.cuda.synchronize()
        assert np.array_equal(od.cpu().numpy(), ref_out)
        assert np.array_equal(_state_of(torch, st), ref_state)


@pytest.mark.parametrize("H,D,T", [(4, 128, 19), (3, 64, 33), (2, 256, 7), (1, 512, 5), (5, 24, 9), (2, 40, 2), (2, 4, 11), (3, 32, 17), (2, 128, 100),
                                   (160, 128, 70), (300, 64, 40), (80, 256, 20)])
def test_prefill_bit_exact_and_equals_decodes(cuda, oracle_mod, H, D, T):
    """Prefill from a non-zero state (two decodes first), with a ragged last
    chunk; equals the oracle and the same tokens fed one decode at a time."""
    from qwanto_b200.linear_attention import LinearAttentionState
    torch = cuda
    rng = np.random.default_rng(7 * T + D)
    decay = 0.96875
    q, k, v = _inputs(rng, T + 2, H, D)
    ref_state = np.zeros((H, D, D), np.float32)
    ref_out = _oracle_steps(oracle_mod, ref_state, q, k, v, decay)
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    with LinearAttentionState(H, D) as a, LinearAttentionState(H, D) as b:
        oa = torch.full((T + 2, H, D), float("nan"), device="cuda")
        ob = torch.full_like(oa, float("nan"))
        for t in range(2):
            a.decode(qd[t], kd[t], vd[t], decay, oa[t])
        a.prefill(qd[2:], kd[2:], vd[2:], decay, T, oa[2:])
        for t in range(T + 2):
            b.decode(qd[t], kd[t], vd[t], decay, ob[t])
        torch.cuda.synchronize()
        assert np.array_equal(oa.cpu().numpy(), ref_out)
        assert np.array_equal(ob.cpu().numpy(), ref_out)
        assert np.array_equal(_state_of(torch, a), ref_state)
        assert np.array_equal(_state_of(torch, b), ref_state)


def test_prefill_matches_reference_library(cuda, oracle_mod, ref_lib):
    """The reference's own qwanto_linear_attention_prefill (built from its
    sources with its SIMD flags) on the same inputs: bit-identical."""
    from qwanto_b200.linear_attention import LinearAttentionState
    torch = cuda
    H, D, T = 6, 128, 12
    rng = np.random.default_rng(99)
    q, k, v = _inputs(rng, T, H, D, 0.5)
    decay = 0.99
    rs = oracle_mod.RefLinearState()
    assert ref_lib.qwanto_linear_attention_init(C.byref(rs), H, D) == 0
    ref_out = np.zeros((T, H, D), np.float32)
    ref_lib.qwanto_linear_attention_prefill(C.byref(rs), _f(q), _f(k), _f(v), C.c_float(decay), T, _f(ref_out))
    ref_state = np.ctypeslib.as_array(rs.state, shape=(H, D, D)).copy()
    ref_lib.qwanto_linear_attention_destroy(C.byref(rs))
    with LinearAttentionState(H, D) as st:
        od = torch.empty((T, H, D), device="cuda")
        st.prefill(*(torch.from_numpy(x).cuda() for x in (q, k, v)), decay, T, od)
        torch.cuda.synchronize()
        assert np.array_equal(od.cpu().numpy(), ref_out)
        assert np.array_equal(_state_of(torch, st), ref_state)


def test_batched_heads_reset_empty_and_host_call(cuda, oracle_mod):
    """256 heads (64 sequences x 4 heads) through the host-buffer call;
    seq_len 0 changes nothing; reset zeroes the state; decay 0 and 1."""
    from qwanto_b200.linear_attention import LinearAttentionState
    torch = cuda
    H, D, T = 256, 128, 3
    rng = np.random.default_rng(5)
    with LinearAttentionState(H, D) as st:
        for decay in (1.0, 0.0):
            st.reset()
            q, k, v = _inputs(rng, T, H, D)
            ref_state = np.zeros((H, D, D), np.float32)
            ref_out = _oracle_steps(oracle_mod, ref_state, q, k, v, decay)
            out = np.full((T, H, D), np.nan, np.float32)
            st.prefill_host(q, k, v, decay, T, out)
            assert np.array_equal(out, ref_out)
            st.prefill_host(q, k, v, decay, 0, out)  # no-op
            st.prefill(None, None, None, decay, 0, None)
            torch.cuda.synchronize()
            assert np.array_equal(_state_of(torch, st), ref_state)
        st.reset()
        torch.cuda.synchronize()
        assert not _state_of(torch, st).any()


def test_prefill_unaligned_inputs_take_the_checked_path(cuda, oracle_mod):
    """q/k/v that start 4 bytes past a 16-byte boundary: the kernel stages
    them with 4-byte copies and still matches the oracle bit for bit."""
    from qwanto_b200.linear_attention import LinearAttentionState
    torch = cuda
    H, D, T = 3, 128, 41
    rng = np.random.default_rng(17)
    q, k, v = _inputs(rng, T, H, D)
    ref_state = np.zeros((H, D, D), np.float32)
    ref_out = _oracle_steps(oracle_mod, ref_state, q, k, v, 0.95)
    dev = []
    for x in (q, k, v):
        buf = torch.empty(x.size + 1, device="cuda")
        buf[1:] = torch.from_numpy(x.reshape(-1)).cuda()
        dev.append(buf[1:])
    assert all(t.data_ptr() % 16 == 4 for t in dev)
    with LinearAttentionState(H, D) as st:
        od = torch.empty((T, H, D), device="cuda")
        st.prefill(*dev, 0.95, T, od)
        torch.cuda.synchronize()
        assert np.array_equal(od.cpu().numpy(), ref_out)
        assert np.array_equal(_state_of(torch, st), ref_state)


def test_host_call_pipelines_long_sequences(cuda, oracle_mod):
    """A host-buffer prefill longer than one staging chunk (4 MiB per input
    array: 2048 tokens of 4 heads x 128) runs as overlapped chunks, the last
    one a single token; the result equals the oracle bit for bit, and a
    second call continues from the state the first one left."""
    from qwanto_b200.linear_attention import LinearAttentionState
    torch = cuda
    H, D, T = 4, 128, 4097
    rng = np.random.default_rng(23)
    q, k, v = _inputs(rng, T + 3, H, D, 0.3)
    ref_state = np.zeros((H, D, D), np.float32)
    ref_out = _oracle_steps(oracle_mod, ref_state, q, k, v, 0.995)
    with LinearAttentionState(H, D) as st:
        out = np.full((T + 3, H, D), np.nan, np.float32)
        st.prefill_host(np.ascontiguousarray(q[:T]), np.ascontiguousarray(k[:T]), np.ascontiguousarray(v[:T]),
                        0.995, T, out[:T])
        st.prefill_host(np.ascontiguousarray(q[T:]), np.ascontiguousarray(k[T:]), np.ascontiguousarray(v[T:]),
                        0.995, 3, out[T:])
        assert np.array_equal(out, ref_out)
        assert np.array_equal(_state_of(torch, st), ref_state)
