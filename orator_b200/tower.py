"""Audio tower (Python side of orx_tower_*): the Qwen3-ASR encoder that turns
log-mel frames into the decoder's audio rows.

``AudioTower.forward`` is the reference's ``AsrAudioTower::Forward``
(include/model/asr_audio_tower.h:77-78): mel [128, n_frames] -> rows
[OutputLength(n_frames), 2048]. ``forward_batch`` runs many utterances in one
call on device tensors; attention stays inside each utterance.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import call, lib
from .decoder import _stream

MEL_BINS, OUT_DIM = 128, 2048


def output_length(n_frames: int) -> int:
    """AsrAudioTower::OutputLength (asr_audio_tower.cu:279-283)."""
    return lib().orx_tower_output_length(int(n_frames))


class AudioTower:
    def __init__(self, layers: int = 24, windowed: bool = False):
        h = C.c_void_p()
        call("orx_tower_create", layers, 1 if windowed else 0, C.byref(h))
        self._h, self.layers = h, layers

    def close(self):
        if getattr(self, "_h", None):
            lib().orx_tower_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, name: str, array):
        a = np.asarray(array)
        if a.dtype == np.uint16:
            dtype = 1
        else:
            a, dtype = a.astype(np.float32), 0
        a = np.ascontiguousarray(a)
        call("orx_tower_set_tensor", self._h, name.encode(), a.ctypes.data_as(C.c_void_p), dtype,
             a.size)

    def load(self, weights: dict):
        for k, v in weights.items():
            self.set_tensor(k, v)

    def load_safetensors(self, model_dir: str):
        call("orx_tower_load_safetensors", self._h, model_dir.encode())

    def init_synthetic(self, seed: int):
        call("orx_tower_init_synthetic", self._h, seed)

    def weights_complete(self) -> bool:
        c = C.c_int()
        call("orx_tower_weights_complete", self._h, C.byref(c))
        return bool(c.value)

    def forward(self, mel: np.ndarray) -> np.ndarray:
        """mel [128, n_frames] (host) -> [OutputLength(n_frames), 2048]."""
        mel = np.ascontiguousarray(mel, np.float32)
        if mel.ndim != 2 or mel.shape[0] != MEL_BINS:
            raise ValueError("mel must be [128, n_frames]")
        n = mel.shape[1]
        out = np.empty((output_length(n), OUT_DIM), np.float32)
        rows = C.c_int()
        call("orx_tower_forward", self._h, mel.ctypes.data_as(C.c_void_p), n,
             out.ctypes.data_as(C.c_void_p), C.byref(rows), C.c_void_p(0))
        return out[:rows.value]

    def forward_batch(self, d_mel: int, frames, d_out: int, stream=None) -> int:
        """Device pointers: d_mel holds the utterances' [128, frames[u]] blocks
        back to back; d_out gets sum(OutputLength(frames[u])) rows of 2048.
        Returns the row count (asynchronous on `stream`)."""
        fr = (C.c_int * len(frames))(*[int(f) for f in frames])
        rows = C.c_int()
        call("orx_tower_forward_batch", self._h, C.c_void_p(d_mel), fr, len(frames),
             C.c_void_p(d_out), C.byref(rows), _stream(stream))
        return rows.value
