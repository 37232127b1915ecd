"""Streaming Sortformer diarizer network (Python side of orx_sf_*).

``Sortformer`` holds the reference's ConformerPreEncode, FastConformer stack
and SortformerDecoder (include/model/conformer_preencode.h,
conformer_layer.h, sortformer_decoder.h) on the GPU: ``pre_encode`` is
ConformerPreEncode::Forward, ``forward`` is
SortformerDiarizer::ForwardEncoderDecoder, ``step`` is the network part of one
streaming chunk ([speaker cache | FIFO | chunk] rows through the encoder and
decoder).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import call, lib
from .decoder import _stream

D_MODEL, N_SPK = 512, 4


def sub_len(n: int) -> int:
    """Frames after the three stride-2 stages (ConvOutLen(x, 3, 2, 1) thrice)."""
    for _ in range(3):
        n = (n + 2 - 3) // 2 + 1
    return n


class Sortformer:
    def __init__(self, conf_layers: int = 17, dec_layers: int = 18):
        h = C.c_void_p()
        call("orx_sf_create", conf_layers, dec_layers, C.byref(h))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().orx_sf_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, name: str, array):
        a = np.ascontiguousarray(array, np.float32)
        call("orx_sf_set_tensor", self._h, name.encode(), a.ctypes.data_as(C.c_void_p), a.size)

    def load(self, weights: dict):
        for k, v in weights.items():
            self.set_tensor(k, v)

    def load_safetensors(self, path: str):
        call("orx_sf_load_safetensors", self._h, path.encode())

    def init_synthetic(self, seed: int):
        call("orx_sf_init_synthetic", self._h, seed)

    def weights_complete(self) -> bool:
        c = C.c_int()
        call("orx_sf_weights_complete", self._h, C.byref(c))
        return bool(c.value)

    def pre_encode(self, mel: np.ndarray, valid: int | None = None):
        """mel [128, n_frames] (host) -> (emb [T2, 512], valid2)."""
        mel = np.ascontiguousarray(mel, np.float32)
        n = mel.shape[1]
        out = np.empty((sub_len(n), D_MODEL), np.float32)
        T2, v2 = C.c_int(), C.c_int()
        call("orx_sf_pre_encode", self._h, mel.ctypes.data_as(C.c_void_p), n,
             n if valid is None else valid, out.ctypes.data_as(C.c_void_p), C.byref(T2),
             C.byref(v2), 0, C.c_void_p(0))
        return out, v2.value

    def forward(self, emb: np.ndarray, valid: int | None = None) -> np.ndarray:
        """emb [T, 512] (host) -> preds [T, 4]."""
        emb = np.ascontiguousarray(emb, np.float32)
        T = emb.shape[0]
        out = np.empty((T, N_SPK), np.float32)
        call("orx_sf_forward", self._h, emb.ctypes.data_as(C.c_void_p), T,
             T if valid is None else valid, out.ctypes.data_as(C.c_void_p), 0, C.c_void_p(0))
        return out

    def step(self, mel: np.ndarray, cache: np.ndarray | None = None, valid: int | None = None):
        """One streaming chunk from host memory -> (preds [T, 4], valid rows)."""
        mel = np.ascontiguousarray(mel, np.float32)
        n = mel.shape[1]
        cache = np.zeros((0, D_MODEL), np.float32) if cache is None else np.ascontiguousarray(cache, np.float32)
        T = cache.shape[0] + sub_len(n)
        out = np.empty((T, N_SPK), np.float32)
        t, v = C.c_int(), C.c_int()
        call("orx_sf_step", self._h, mel.ctypes.data_as(C.c_void_p), n, n if valid is None else valid,
             cache.ctypes.data_as(C.c_void_p), cache.shape[0], out.ctypes.data_as(C.c_void_p),
             C.byref(t), C.byref(v), 0, C.c_void_p(0))
        return out, v.value

    def step_device(self, d_mel: int, n_frames: int, valid: int, d_cache: int, n_cache: int,
                    d_preds: int, stream=None) -> int:
        t, v = C.c_int(), C.c_int()
        call("orx_sf_step", self._h, C.c_void_p(d_mel), n_frames, valid, C.c_void_p(d_cache),
             n_cache, C.c_void_p(d_preds), C.byref(t), C.byref(v), 1, _stream(stream))
        return t.value
