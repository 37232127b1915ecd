"""Batched speech detector over many streams (Python side of orx_vad_*).

``BatchVad`` runs the Silero-shaped model of the reference's ``GpuVad``
(src/pipeline/gpu_vad.cu, include/pipeline/gpu_vad.h) for all streams at
once; ``VadPool`` adds the reference's per-stream streaming API on top:
``Push`` audio per stream, ``DrainSegments`` runs every stream's complete
windows in one batched call and applies the endpoint state machine
(GpuVad::DrainSegments / EmitPaddedSegment / state, gpu_vad.cu:369-470) per
stream: speech starts after ``min_speech_ms`` of windows with probability >=
threshold, ends after ``min_silence_ms`` below it, and segments are padded by
``speech_pad_ms`` without overlapping the previous one.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import call, lib
from .decoder import _stream

WINDOW, CONTEXT = 512, 64


class BatchVad:
    def __init__(self, streams: int):
        h = C.c_void_p()
        call("orx_vad_create", streams, C.byref(h))
        self._h, self.streams = h, streams

    def close(self):
        if getattr(self, "_h", None):
            lib().orx_vad_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, name: str, array):
        a = np.ascontiguousarray(array, np.float32)
        call("orx_vad_set_tensor", self._h, name.encode(), a.ctypes.data_as(C.c_void_p), a.size)

    def load(self, weights: dict):
        for k, v in weights.items():
            self.set_tensor(k, v)

    def init_synthetic(self, seed: int):
        call("orx_vad_init_synthetic", self._h, seed)

    def reset(self):
        call("orx_vad_reset", self._h)

    def run(self, pcm: np.ndarray) -> np.ndarray:
        """pcm [streams, steps * 512] (host) -> probabilities [streams, steps]."""
        pcm = np.ascontiguousarray(pcm, np.float32)
        steps = pcm.shape[1] // WINDOW
        out = np.empty((self.streams, steps), np.float32)
        call("orx_vad_run", self._h, pcm.ctypes.data_as(C.c_void_p), steps,
             out.ctypes.data_as(C.c_void_p), 0, C.c_void_p(0))
        return out

    def run_device(self, d_pcm: int, steps: int, d_probs: int, stream=None):
        call("orx_vad_run", self._h, C.c_void_p(d_pcm), steps, C.c_void_p(d_probs), 1,
             _stream(stream))


@dataclass
class VadParams:
    """GpuVad::Params (include/pipeline/gpu_vad.h:20-30)."""
    sample_rate: int = 16000
    silero_threshold: float = 0.5
    silero_min_speech_ms: int = 250
    silero_min_silence_ms: int = 120
    silero_speech_pad_ms: int = 60


class _StreamState:
    def __init__(self):
        self.buf = np.zeros(0, np.float32)
        self.next_abs = 0
        self.in_speech = False
        self.speech = self.silence = 0
        self.seg_start = 0
        self.last_end = 0


class VadPool:
    """Per-stream GpuVad semantics (Push / DrainSegments / state / Reset) for
    many streams whose windows run in one batched GPU call. Streams advance
    in lockstep: a drain processes the windows every stream has complete."""

    def __init__(self, vad: BatchVad, params: VadParams | None = None):
        self.vad, self.p = vad, params or VadParams()
        self.st = [_StreamState() for _ in range(vad.streams)]

    def Push(self, stream: int, samples):
        s = self.st[stream]
        s.buf = np.concatenate([s.buf, np.asarray(samples, np.float32)])

    def _emit(self, s, start, end, horizon, out):
        pad = self.p.silero_speech_pad_ms * self.p.sample_rate // 1000
        if end <= start:
            return
        ps = max(s.last_end, max(0, start - pad))
        pe = min(horizon, end + pad)
        if pe <= ps:
            return
        out.append((ps, pe))
        s.last_end = pe

    def DrainSegments(self, finalize: bool = False) -> list[list[tuple[int, int]]]:
        """Segments [start, end) (absolute samples) completed per stream."""
        n = min(len(s.buf) for s in self.st) // WINDOW
        sr = self.p.sample_rate
        min_speech = self.p.silero_min_speech_ms * sr // 1000
        min_silence = self.p.silero_min_silence_ms * sr // 1000
        out = [[] for _ in self.st]
        if n > 0:
            pcm = np.stack([s.buf[:n * WINDOW] for s in self.st])
            probs = self.vad.run(pcm)
            for i, s in enumerate(self.st):
                for k in range(n):
                    win_end = s.next_abs + (k + 1) * WINDOW
                    if probs[i, k] >= self.p.silero_threshold:
                        s.silence = 0
                        s.speech += WINDOW
                        if not s.in_speech and s.speech >= min_speech:
                            s.in_speech = True
                            s.seg_start = win_end - s.speech
                    elif s.in_speech:
                        s.silence += WINDOW
                        if s.silence >= min_silence:
                            s.in_speech = False
                            self._emit(s, s.seg_start, win_end - s.silence, win_end, out[i])
                            s.speech = 0
                    else:
                        s.speech = 0
                s.next_abs += n * WINDOW
                s.buf = s.buf[n * WINDOW:]
        if finalize:
            for i, s in enumerate(self.st):
                if s.in_speech:
                    self._emit(s, s.seg_start, s.next_abs, s.next_abs, out[i])
                    s.in_speech = False
                    s.speech = s.silence = 0
        return out

    def is_in_speech(self, stream: int) -> bool:
        return self.st[stream].in_speech

    def Reset(self):
        self.vad.reset()
        self.st = [_StreamState() for _ in self.st]
