"""Python host mirror of the reference ``AsrTextDecoder`` over the C ABI.

Method names, argument meaning and error behaviour follow
``include/model/asr_text_decoder.h:45-113`` of thomas-hiddenpeak/Orator: calls
raise ``OrxError`` where the reference throws. Host arrays are numpy; device
arguments (``d_token``, device embeds) are raw device addresses (ints), e.g.
``torch.Tensor.data_ptr()``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import Config, call, lib


@dataclass
class AsrTextConfig:
    """``AsrTextConfig`` (asr_text_decoder.h:30-43)."""
    hidden_size: int = 2048
    num_layers: int = 28
    num_q_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 6144
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_seq_len: int = 2048
    profile: bool = False
    cuda_graph_enabled: bool = True

    def to_c(self) -> Config:
        c = Config()
        for k in Config._fields_:
            setattr(c, k[0], int(getattr(self, k[0])) if k[1] is C.c_int
                    else float(getattr(self, k[0])))
        return c


def _stream(s) -> C.c_void_p:
    if s is None or s == 0:
        return C.c_void_p(0)
    if hasattr(s, "cuda_stream"):
        return C.c_void_p(s.cuda_stream)
    return C.c_void_p(int(s))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class AsrTextDecoder:
    def __init__(self, config: AsrTextConfig | None = None):
        self.config = config or AsrTextConfig()
        h = C.c_void_p()
        cfg = self.config.to_c()
        call("orx_decoder_create", C.byref(cfg), C.byref(h))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().orx_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # --- weights ---------------------------------------------------------
    def set_tensor(self, name: str, array=None, *, dtype: str = "bf16", device_ptr: int = 0,
                   numel: int = 0):
        """Place one ``thinker.model.*`` tensor (``LoadWeights``, cu:251-336).
        ``array``: numpy fp32 or uint16 (bf16 bits) host array."""
        if array is not None:
            a = np.ascontiguousarray(array)
            code = 1 if a.dtype == np.uint16 else 0
            if code == 0:
                a = a.astype(np.float32, copy=False)
            call("orx_decoder_set_tensor", self._h, name.encode(), a.ctypes.data_as(C.c_void_p),
                 code, a.size, 0)
        else:
            call("orx_decoder_set_tensor", self._h, name.encode(), C.c_void_p(device_ptr),
                 1 if dtype == "bf16" else 0, numel, 1)

    def load_weights(self, model_dir: str):
        call("orx_decoder_load_safetensors", self._h, model_dir.encode())

    LoadWeights = load_weights

    def init_synthetic(self, seed: int):
        call("orx_decoder_init_synthetic", self._h, seed)

    def weights_complete(self) -> bool:
        v = C.c_int()
        call("orx_decoder_weights_complete", self._h, C.byref(v))
        return bool(v.value)

    # --- cache -----------------------------------------------------------
    def ResetCache(self):
        call("orx_decoder_reset_cache", self._h)

    def TruncateCache(self, n: int):
        call("orx_decoder_truncate_cache", self._h, n)

    def cache_len(self) -> int:
        v = C.c_int()
        call("orx_decoder_cache_len", self._h, C.byref(v))
        return v.value

    def hidden_size(self) -> int:
        return self.config.hidden_size

    def vocab_size(self) -> int:
        return self.config.vocab_size

    def Embed(self, token_id: int, out: np.ndarray | None = None) -> np.ndarray:
        o = np.empty(self.config.hidden_size, np.float32) if out is None else out
        call("orx_decoder_embed", self._h, token_id, o.ctypes.data_as(C.c_void_p))
        return o

    # --- forward ---------------------------------------------------------
    def Prefill(self, embeds, T: int | None = None, stream=None):
        self.PrefillAt(embeds, T, 0, stream)

    def PrefillAt(self, embeds, T: int | None, pos0: int, stream=None):
        e = _f32(embeds).reshape(-1, self.config.hidden_size)
        T = e.shape[0] if T is None else T
        call("orx_decoder_prefill_at", self._h, e.ctypes.data_as(C.c_void_p), T, pos0,
             _stream(stream))

    def PrefillAtDevice(self, d_embeds: int, T: int, pos0: int, stream=None):
        call("orx_decoder_prefill_at_device", self._h, C.c_void_p(d_embeds), T, pos0,
             _stream(stream))

    def DecodeStep(self, embed, pos: int, stream=None):
        e = _f32(embed)
        call("orx_decoder_decode_step", self._h, e.ctypes.data_as(C.c_void_p), pos,
             _stream(stream))

    def DecodeStepDevice(self, d_token: int, pos: int, stream=None):
        call("orx_decoder_decode_step_device", self._h, C.c_void_p(d_token), pos,
             _stream(stream))

    def Argmax(self, ban0: int = -1, ban1: int = -1, stream=None) -> int:
        v = C.c_int()
        call("orx_decoder_argmax", self._h, ban0, ban1, _stream(stream), C.byref(v))
        return v.value

    def ArgmaxToDevice(self, d_out: int, ban0: int = -1, ban1: int = -1, stream=None):
        call("orx_decoder_argmax_to_device", self._h, C.c_void_p(d_out), ban0, ban1,
             _stream(stream))

    def ReadTokenId(self, d_token: int, stream=None) -> int:
        v = C.c_int()
        call("orx_decoder_read_token_id", self._h, C.c_void_p(d_token), _stream(stream),
             C.byref(v))
        return v.value

    def DecodeGreedy(self, start_pos: int, max_new: int, eos0: int, eos1: int,
                     ban_steps: int = 3, batch: int = 32, stream=None) -> list[int]:
        out = np.zeros(max(max_new, 1), np.int32)
        n = C.c_int()
        call("orx_decoder_decode_greedy", self._h, start_pos, max_new, eos0, eos1, ban_steps,
             batch, _stream(stream), out.ctypes.data_as(C.c_void_p), C.byref(n))
        return out[:n.value].tolist()

    def CopyLogits(self) -> np.ndarray:
        o = np.empty(self.config.vocab_size, np.float32)
        call("orx_decoder_copy_logits", self._h, o.ctypes.data_as(C.c_void_p))
        return o

    def logits_device_ptr(self) -> int:
        p = C.c_void_p()
        call("orx_decoder_logits_device", self._h, C.byref(p))
        return p.value

    def profile_kernels(self, iters: int = 20, stream=None) -> dict:
        ms = np.zeros(6, np.float32)
        call("orx_decoder_profile_kernels", self._h, iters, _stream(stream),
             ms.ctypes.data_as(C.c_void_p))
        return dict(zip(["qkv", "attention", "o", "gateup", "down", "lm_head"], ms.tolist()))

    def trace_decode(self, steps: int = 2, stream=None) -> np.ndarray:
        per = 5 * self.config.num_layers + 1
        out = np.zeros(steps * per * 3, np.uint64)
        n = C.c_int()
        call("orx_decoder_trace_decode", self._h, steps, _stream(stream),
             out.ctypes.data_as(C.c_void_p), C.byref(n))
        return out.reshape(steps, per, 3)

    def trace_ctas(self, steps: int = 2, stream=None) -> np.ndarray:
        """Per phase and CTA of the persistent decode kernel: [steps, per, grid, 2]
        global-timer ns of {inputs ready, phase done} (diagnostic)."""
        per = 5 * self.config.num_layers + 1
        grid = C.c_int()
        cap = steps * per * 1024 * 2
        out = np.zeros(cap, np.uint64)
        call("orx_decoder_trace_ctas", self._h, steps, _stream(stream),
             out.ctypes.data_as(C.c_void_p), C.c_size_t(cap), C.byref(grid))
        g = grid.value
        return out[: steps * per * g * 2].reshape(steps, per, g, 2)

    def device_error(self) -> int:
        v = C.c_int()
        call("orx_decoder_device_error", self._h, C.byref(v))
        return v.value


def synth_f32(d_out: int, n: int, seed: int, tensor_id: int, std: float, mean: float = 0.0,
              round_bf16: bool = False, stream=None):
    call("orx_synth_f32", C.c_void_p(d_out), n, seed, tensor_id, std, mean, int(round_bf16),
         _stream(stream))
