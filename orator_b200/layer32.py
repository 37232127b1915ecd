"""fp32 single decoder layer over the C ABI (``orx_layer32_*``).

One Qwen3-1.7B-shaped layer with fp32 weights, activations and KV cache and no
bf16 rounding: the correctness configuration of the decoder, whose reference
check is an fp32 CPU restatement of the same layer. Rows are processed
causally; each appends its K/V at its position.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import call, lib
from .decoder import AsrTextConfig, _f32, _stream


class Layer32:
    def __init__(self, config: AsrTextConfig | None = None):
        self.config = config or AsrTextConfig()
        h = C.c_void_p()
        cfg = self.config.to_c()
        call("orx_layer32_create", C.byref(cfg), C.byref(h))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().orx_layer32_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, name: str, array):
        """Layer-relative name (``self_attn.q_proj``, ``mlp.down_proj``, ...), fp32."""
        a = _f32(array)
        call("orx_layer32_set_tensor", self._h, name.encode(), a.ctypes.data_as(C.c_void_p),
             a.size, 0)

    def init_synthetic(self, seed: int, layer: int = 0):
        call("orx_layer32_init_synthetic", self._h, seed, layer)

    def forward(self, x, pos0: int, stream=None) -> np.ndarray:
        """Rows ``x`` [T, 2048] at positions pos0.. -> layer outputs [T, 2048]."""
        a = _f32(x).reshape(-1, self.config.hidden_size)
        out = np.empty_like(a)
        call("orx_layer32_forward", self._h, a.ctypes.data_as(C.c_void_p), a.shape[0], pos0,
             out.ctypes.data_as(C.c_void_p), _stream(stream))
        return out

    def forward_device(self, d_x: int, T: int, pos0: int, d_out: int, stream=None):
        call("orx_layer32_forward_device", self._h, C.c_void_p(d_x), T, pos0, C.c_void_p(d_out),
             _stream(stream))

    def cache_len(self) -> int:
        v = C.c_int()
        call("orx_layer32_cache_len", self._h, C.byref(v))
        return v.value

    def truncate(self, n: int):
        call("orx_layer32_truncate", self._h, n)
