"""ctypes binding of liborator_b200.so (the C ABI in include/orx.h).

There is no fallback: if the library is missing or fails to load, importing
anything that needs it raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liborator_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "orx.h")


class OrxError(RuntimeError):
    """Raised on a non-zero status (the reference throws GpuMemoryException /
    std::runtime_error, src/gpu/memory.cc:14-20)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"orx error {code}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [("hidden_size", C.c_int), ("num_layers", C.c_int), ("num_q_heads", C.c_int),
                ("num_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("intermediate_size", C.c_int), ("vocab_size", C.c_int),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float),
                ("max_seq_len", C.c_int), ("profile", C.c_int),
                ("cuda_graph_enabled", C.c_int)]


_lib = None

_SIGS = {
    "orx_last_error": (C.c_char_p, []),
    "orx_version": (C.c_int, []),
    "orx_config_default": (None, [C.POINTER(Config)]),
    "orx_decoder_create": (C.c_int, [C.POINTER(Config), C.POINTER(C.c_void_p)]),
    "orx_decoder_destroy": (None, [C.c_void_p]),
    "orx_decoder_set_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int,
                                         C.c_size_t, C.c_int]),
    "orx_decoder_load_safetensors": (C.c_int, [C.c_void_p, C.c_char_p]),
    "orx_decoder_init_synthetic": (C.c_int, [C.c_void_p, C.c_int]),
    "orx_decoder_weights_complete": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_decoder_reset_cache": (C.c_int, [C.c_void_p]),
    "orx_decoder_truncate_cache": (C.c_int, [C.c_void_p, C.c_int]),
    "orx_decoder_cache_len": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_decoder_embed": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    "orx_decoder_prefill_at": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "orx_decoder_prefill_at_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                                C.c_void_p]),
    "orx_decoder_decode_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "orx_decoder_decode_step_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "orx_decoder_argmax": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                     C.POINTER(C.c_int)]),
    "orx_decoder_argmax_to_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                               C.c_void_p]),
    "orx_decoder_read_token_id": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p,
                                            C.POINTER(C.c_int)]),
    "orx_decoder_decode_greedy": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                            C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                            C.POINTER(C.c_int)]),
    "orx_decoder_copy_logits": (C.c_int, [C.c_void_p, C.c_void_p]),
    "orx_decoder_logits_device": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "orx_decoder_device_error": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_decoder_profile_kernels": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "orx_argmax_banned_noalloc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                            C.c_void_p]),
    "orx_decoder_trace_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                           C.POINTER(C.c_int)]),
    "orx_decoder_trace_ctas": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_size_t,
                                         C.POINTER(C.c_int)]),
    "orx_batch_create": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.POINTER(C.c_void_p)]),
    "orx_batch_destroy": (None, [C.c_void_p]),
    "orx_batch_session_create": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_batch_session_free": (C.c_int, [C.c_void_p, C.c_int]),
    "orx_batch_cache_len": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
    "orx_batch_truncate": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "orx_batch_free_pages": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_batch_prefill": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                    C.c_void_p]),
    "orx_batch_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "orx_batch_device_error": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_batch_set_ban": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "orx_batch_next_tokens": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "orx_layer32_create": (C.c_int, [C.POINTER(Config), C.POINTER(C.c_void_p)]),
    "orx_layer32_destroy": (None, [C.c_void_p]),
    "orx_layer32_set_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t, C.c_int]),
    "orx_layer32_init_synthetic": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "orx_layer32_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                      C.c_void_p]),
    "orx_layer32_forward_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                             C.c_void_p, C.c_void_p]),
    "orx_layer32_cache_len": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_layer32_truncate": (C.c_int, [C.c_void_p, C.c_int]),
    "orx_linear_pre": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                 C.c_int, C.c_int, C.c_void_p]),
    "orx_linear": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                             C.c_int, C.c_int, C.c_void_p]),
    "orx_f32_to_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p]),
    "orx_bf16_to_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p]),
    "orx_rms_norm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float,
                               C.c_void_p]),
    "orx_rope_half": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float,
                                C.c_void_p]),
    "orx_rope_interleaved": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                       C.c_float, C.c_void_p]),
    "orx_swiglu": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p]),
    "orx_gqa_attention": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                    C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p]),
    "orx_argmax_banned": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                    C.c_void_p]),
    "orx_vad_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "orx_vad_destroy": (None, [C.c_void_p]),
    "orx_vad_set_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]),
    "orx_vad_init_synthetic": (C.c_int, [C.c_void_p, C.c_int]),
    "orx_vad_reset": (C.c_int, [C.c_void_p]),
    "orx_vad_run": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
    "orx_tower_create": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "orx_tower_destroy": (None, [C.c_void_p]),
    "orx_tower_set_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int, C.c_size_t]),
    "orx_tower_load_safetensors": (C.c_int, [C.c_void_p, C.c_char_p]),
    "orx_tower_init_synthetic": (C.c_int, [C.c_void_p, C.c_int]),
    "orx_tower_weights_complete": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_tower_output_length": (C.c_int, [C.c_int]),
    "orx_tower_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                    C.POINTER(C.c_int), C.c_void_p]),
    "orx_tower_forward_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                          C.c_void_p, C.POINTER(C.c_int), C.c_void_p]),
    "orx_sf_create": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "orx_sf_destroy": (None, [C.c_void_p]),
    "orx_sf_set_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]),
    "orx_sf_load_safetensors": (C.c_int, [C.c_void_p, C.c_char_p]),
    "orx_sf_init_synthetic": (C.c_int, [C.c_void_p, C.c_int]),
    "orx_sf_weights_complete": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "orx_sf_pre_encode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                    C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int, C.c_void_p]),
    "orx_sf_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                 C.c_void_p]),
    "orx_sf_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int,
                              C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int,
                              C.c_void_p]),
    "orx_synth_f32": (C.c_int, [C.c_void_p, C.c_longlong, C.c_int, C.c_int, C.c_double,
                                C.c_float, C.c_int, C.c_void_p]),
}


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"\b(orx_[a-z0-9_]+)\s*\(", txt)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OrxError(-1, f"{LIB_PATH} not built (run python -m orator_b200.build)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def call(name: str, *args):
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise OrxError(rc, lib().orx_last_error().decode())
    return rc
