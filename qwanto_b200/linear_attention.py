"""Linear attention on a device-resident fp32 state (``qwn_linear_attention_*``).

Mirrors the reference's QwantoLinearAttentionState API
(c/qwanto_attention.h:11-72): init / reset / destroy / decode / prefill with
the same argument meaning, on device buffers (torch tensors or raw
pointers).  Per token and head the state is updated as
``S = decay * S + k^T v`` and the output is ``o = q S``, with the
reference's rounding order, so results are bit-identical to it.  Several
sequences are simply more heads (``n_heads = sequences * heads``).
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from ._lib import check, lib


def _p(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    return x.ctypes.data


class LinearAttentionState:
    """``QwantoLinearAttentionState`` with its state matrix in device memory:
    [n_heads][head_dim][head_dim] fp32, zero after init and reset."""

    def __init__(self, n_heads: int, head_dim: int, device: int = 0):
        self._st = _lib.LinearAttentionState()
        check("qwn_linear_attention_init", lib().qwn_linear_attention_init(C.byref(self._st), device, n_heads,
                                                                           head_dim))
        self.n_heads, self.head_dim, self.device = n_heads, head_dim, device

    @property
    def state_ptr(self) -> int:
        return self._st.state

    @property
    def state_bytes(self) -> int:
        return self.n_heads * self.head_dim * self.head_dim * 4

    def reset(self, stream=None) -> None:
        check("qwn_linear_attention_reset", lib().qwn_linear_attention_reset(C.byref(self._st), stream))

    def decode(self, q, k, v, decay: float, o, stream=None) -> None:
        """One token: q/k/v/o are [n_heads][head_dim] fp32 device buffers."""
        check("qwn_linear_attention_decode", lib().qwn_linear_attention_decode(
            C.byref(self._st), _p(q), _p(k), _p(v), C.c_float(decay), _p(o), stream))

    def prefill(self, q, k, v, decay: float, seq_len: int, o, stream=None) -> None:
        """`seq_len` tokens in order: q/k/v/o are [seq_len][n_heads][head_dim]."""
        check("qwn_linear_attention_prefill", lib().qwn_linear_attention_prefill(
            C.byref(self._st), _p(q), _p(k), _p(v), C.c_float(decay), seq_len, _p(o), stream))

    def prefill_host(self, q, k, v, decay: float, seq_len: int, o) -> None:
        """The same on HOST buffers (numpy or pinned torch tensors); synchronous."""
        check("qwn_linear_attention_prefill_host", lib().qwn_linear_attention_prefill_host(
            C.byref(self._st), _p(q), _p(k), _p(v), C.c_float(decay), seq_len, _p(o)))

    def close(self) -> None:
        if self._st.state:
            lib().qwn_linear_attention_destroy(C.byref(self._st))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
