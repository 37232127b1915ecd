"""CPU restatement of the reference's Silero-shaped speech detector, for many
independent streams at once (TEST INFRASTRUCTURE: the checker of the batched
GPU detector, never the product).

Per window (src/pipeline/gpu_vad.cu:44-171, test/utils/asr_vad_cpu.cc:80-175):
input = 64 context samples + 512 new ones; reflect-padded right by 64
(out[576 + i] = in[574 - i]); STFT as a conv with a 258 x 256 basis at hop 128
(4 frames), magnitude sqrt(re^2 + im^2) of 129 bins; four conv1d + ReLU
blocks 129->128 (k3 s1 p1), 128->64 (k3 s2 p1), 64->64 (k3 s2 p1),
64->128 (k3 s1 p1); one LSTM cell step (gates i, f, g, o; state carried
across windows); probability = sigmoid(b + sum_i relu(h_i) * w_i). The next
window's context is the last 64 samples of this window's input.

The endpoint state machine of GpuVad::DrainSegments / EmitPaddedSegment /
state (gpu_vad.cu:369-470) is restated in ``Endpoint``.

Synthetic weights (seed 4): every tensor N(0, s^2/fan_in)
from the repository's counter-hash generator (oracle/synth.py, tensor ids
70000 + i), the STFT basis included, with gain s = 1.5 for the conv blocks, 2
for the LSTM and 8 for the head, and a head bias of 0.3, so that the random
model's probabilities spread across the 0.5 threshold.
"""
from __future__ import annotations

import numpy as np

from . import synth

CONTEXT, WINDOW, INPUT, PADDED = 64, 512, 576, 640
NFFT, HOP, BINS, FRAMES, HIDDEN = 256, 128, 129, 4, 128

# (checkpoint name, shape, fan_in)
TENSORS = [
    ("stft.forward_basis_buffer", (258, 1, 256), 256),
    ("encoder.0.reparam_conv.weight", (128, 129, 3), 129 * 3),
    ("encoder.0.reparam_conv.bias", (128,), 129 * 3),
    ("encoder.1.reparam_conv.weight", (64, 128, 3), 128 * 3),
    ("encoder.1.reparam_conv.bias", (64,), 128 * 3),
    ("encoder.2.reparam_conv.weight", (64, 64, 3), 64 * 3),
    ("encoder.2.reparam_conv.bias", (64,), 64 * 3),
    ("encoder.3.reparam_conv.weight", (128, 64, 3), 64 * 3),
    ("encoder.3.reparam_conv.bias", (128,), 64 * 3),
    ("decoder.rnn.weight_ih", (512, 128), 128),
    ("decoder.rnn.weight_hh", (512, 128), 128),
    ("decoder.rnn.bias_ih", (512,), 128),
    ("decoder.rnn.bias_hh", (512,), 128),
    ("decoder.decoder.2.weight", (1, 128, 1), 128),
    ("decoder.decoder.2.bias", (1,), 128),
]
TID_VAD = 70000
TID_PCM = 71000


def gain(name: str) -> float:
    return 8.0 if name.startswith("decoder.decoder") else 2.0 if name.startswith("decoder.rnn") \
        else 1.5 if name.startswith("encoder") else 1.0


def synthetic_weights(seed: int = 4) -> dict:
    w = {}
    for i, (name, shape, fan_in) in enumerate(TENSORS):
        n = int(np.prod(shape))
        w[name] = synth.normal_f32(seed, TID_VAD + i, n,
                                   float(gain(name) / np.sqrt(fan_in))).reshape(shape)
    w["decoder.decoder.2.bias"] = np.full((1,), 0.3, np.float32)
    return w


def synthetic_pcm(seed: int, streams: int, samples: int) -> np.ndarray:
    """PCM uniform in [-1, 1): 24 bits of the counter hash per sample."""
    h = synth.hashes(seed, TID_PCM, 0, streams * samples)
    u = ((h >> np.uint64(40)).astype(np.float64) / float(1 << 24)).astype(np.float32)
    return (2.0 * u - 1.0).astype(np.float32).reshape(streams, samples)


def conv1d(x, w, b, stride, pad):
    """x [S, Cin, Lin], w [Cout, Cin, K] -> [S, Cout, Lout] (zero padding)."""
    S, cin, lin = x.shape
    cout, _, k = w.shape
    lout = (lin + 2 * pad - k) // stride + 1
    xp = np.zeros((S, cin, lin + 2 * pad), np.float32)
    xp[:, :, pad:pad + lin] = x
    cols = np.stack([xp[:, :, t * stride:t * stride + k] for t in range(lout)], 1)  # [S, Lout, Cin, K]
    y = np.einsum("stck,ock->sot", cols, w, dtype=np.float32)
    if b is not None:
        y = y + b[None, :, None]
    return y.astype(np.float32)


def sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


class BatchVadOracle:
    """All streams advance one window per step; state per stream."""

    def __init__(self, weights: dict, streams: int):
        self.w = {k: np.asarray(v, np.float32) for k, v in weights.items()}
        self.S = streams
        self.reset()

    def reset(self):
        self.h = np.zeros((self.S, HIDDEN), np.float32)
        self.c = np.zeros((self.S, HIDDEN), np.float32)
        self.ctx = np.zeros((self.S, CONTEXT), np.float32)

    def step(self, window: np.ndarray) -> np.ndarray:
        """window [S, 512] -> speech probability [S]."""
        w = self.w
        x = np.concatenate([self.ctx, np.asarray(window, np.float32)], 1)      # [S, 576]
        pad = x[:, INPUT - 2 - np.arange(64)]                                  # reflect right
        xp = np.concatenate([x, pad], 1)                                       # [S, 640]
        frames = np.stack([xp[:, t * HOP:t * HOP + NFFT] for t in range(FRAMES)], 1)  # [S, 4, 256]
        basis = w["stft.forward_basis_buffer"].reshape(258, 256)
        st = np.einsum("stk,fk->sft", frames, basis, dtype=np.float32)         # [S, 258, 4]
        mag = np.sqrt(st[:, :BINS] ** 2 + st[:, BINS:] ** 2).astype(np.float32)
        e = mag
        for i, (stride, pad_) in enumerate([(1, 1), (2, 1), (2, 1), (1, 1)]):
            e = np.maximum(conv1d(e, w[f"encoder.{i}.reparam_conv.weight"],
                                  w[f"encoder.{i}.reparam_conv.bias"], stride, pad_), 0)
        xin = e[:, :, 0]                                                        # [S, 128]
        g = (xin @ w["decoder.rnn.weight_ih"].T + self.h @ w["decoder.rnn.weight_hh"].T
             + w["decoder.rnn.bias_ih"] + w["decoder.rnn.bias_hh"]).astype(np.float32)
        gi, gf = sigmoid(g[:, :128]), sigmoid(g[:, 128:256])
        gg, go = np.tanh(g[:, 256:384]), sigmoid(g[:, 384:])
        self.c = (gf * self.c + gi * gg).astype(np.float32)
        self.h = (go * np.tanh(self.c)).astype(np.float32)
        dot = np.maximum(self.h, 0) @ w["decoder.decoder.2.weight"].reshape(128) + \
            w["decoder.decoder.2.bias"][0]
        self.ctx = x[:, INPUT - CONTEXT:].copy()
        return sigmoid(dot)

    def run(self, pcm: np.ndarray, steps: int) -> np.ndarray:
        """pcm [S, steps * 512] -> probabilities [S, steps]."""
        return np.stack([self.step(pcm[:, k * WINDOW:(k + 1) * WINDOW]) for k in range(steps)], 1)


class Endpoint:
    """Speech-segment state machine of one stream (GpuVad::DrainSegments,
    EmitPaddedSegment and state, src/pipeline/gpu_vad.cu:369-470), fed one
    window probability at a time."""

    def __init__(self, sample_rate=16000, threshold=0.5, min_speech_ms=250, min_silence_ms=120,
                 speech_pad_ms=60):
        self.sr, self.th = sample_rate, threshold
        self.min_speech = min_speech_ms * sample_rate // 1000
        self.min_silence = min_silence_ms * sample_rate // 1000
        self.pad = speech_pad_ms * sample_rate // 1000
        self.next_abs = 0
        self.in_speech = False
        self.speech = self.silence = 0
        self.seg_start = 0
        self.last_end = 0

    def _emit(self, start, end, horizon, out):
        if end <= start:
            return
        ps = max(self.last_end, max(0, start - self.pad))
        pe = min(horizon, end + self.pad)
        if pe <= ps:
            return
        out.append((ps, pe))
        self.last_end = pe

    def push(self, probs, finalize=False):
        out = []
        for i, p in enumerate(probs):
            win_end = self.next_abs + (i + 1) * WINDOW
            if p >= self.th:
                self.silence = 0
                self.speech += WINDOW
                if not self.in_speech and self.speech >= self.min_speech:
                    self.in_speech = True
                    self.seg_start = win_end - self.speech
            elif self.in_speech:
                self.silence += WINDOW
                if self.silence >= self.min_silence:
                    self.in_speech = False
                    self._emit(self.seg_start, win_end - self.silence, win_end, out)
                    self.speech = 0
            else:
                self.speech = 0
        self.next_abs += len(probs) * WINDOW
        if finalize and self.in_speech:
            self._emit(self.seg_start, self.next_abs, self.next_abs, out)
            self.in_speech = False
            self.speech = self.silence = 0
        return out


def write_safetensors(path: str, weights: dict) -> str:
    """One F32 safetensors file with the detector's tensors (the reference
    loads its weights by these names, src/pipeline/gpu_vad.cu:242-271)."""
    import json
    import struct
    header, off, blobs = {}, 0, []
    for name, shape, _ in TENSORS:
        a = np.ascontiguousarray(weights[name], np.float32).reshape(shape)
        header[name] = {"dtype": "F32", "shape": list(shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        blobs.append(a.tobytes())
    hj = json.dumps(header).encode()
    hj += b" " * ((-len(hj)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)
    return path
