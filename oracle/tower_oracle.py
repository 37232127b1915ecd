"""CPU restatement of the reference's Qwen3-ASR audio tower (encoder), the
producer of the decoder's audio rows (TEST INFRASTRUCTURE: a checker, never
the product).

Follows src/model/asr_audio_tower.cu (AsrAudioTower::Forward, :340-634):
* mel [128, n_frames] cut into chunks of 100 frames (the last one shorter),
  zero-padded to the longest chunk: [chunks, 1, 128, max_cl];
* three 3x3 stride-2 pad-1 convolutions 1 -> 480 -> 480 -> 480, each as
  im2col (columns rounded to bf16) x bf16 weights with fp32 accumulation,
  then + bias and exact GELU in fp32 (Im2ColKernel, ConvOutRearrangeKernel);
* [chunks, 480, 16, Wc] -> rows (chunk, t) of 480 * 16 features (channel
  major) -> conv_out Linear (no bias) to 1024, + sinusoidal position code of
  t inside the chunk (ReshapeC3Kernel, AddPeChunkedKernel);
* only each chunk's first OutputLength(chunk_len) rows are kept
  (DropPadGatherKernel);
* 24 pre-LayerNorm encoder layers (eps 1e-5): q / k / v / out projections
  with bias, full bidirectional attention over all N rows (16 heads of 64),
  fc1 (GELU) and fc2, residual adds in fp32;
* ln_post, proj1 (GELU), proj2 -> [N, 2048].
Every Linear rounds its fp32 input to bf16 (asr_gemm::Linear) and multiplies
by bf16 weights with fp32 accumulation, then adds the fp32 bias and applies
the activation.

Synthetic weights (seed 5): tensor ids 80000 + i in checkpoint order; matrices
and conv kernels N(0, 1/fan_in), biases N(0, 0.02^2), LayerNorm gains
1 + N(0, 0.02^2) and shifts N(0, 0.02^2); all rounded to bf16 (the file
format).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import synth

F, D, H, DH, FFN, DS, OUT = 128, 1024, 16, 64, 4096, 480, 2048
PREFIX = "thinker.audio_tower."
TID = 80000


def conv_out_len(x: int) -> int:
    return 0 if x <= 0 else (x - 1) // 2 + 1


def output_length(mel_frames: int) -> int:
    """AsrAudioTower::OutputLength (asr_audio_tower.cu:279-283)."""
    leave = mel_frames % 100
    return conv_out_len(conv_out_len(conv_out_len(leave))) + (mel_frames // 100) * 13


def tensor_list(layers: int):
    """(name, shape, kind) in checkpoint order; kind: w (fan-in scaled),
    b (bias), g (LayerNorm gain), s (LayerNorm shift)."""
    t = [(PREFIX + "conv2d1.weight", (DS, 1, 3, 3), "w"), (PREFIX + "conv2d1.bias", (DS,), "b"),
         (PREFIX + "conv2d2.weight", (DS, DS, 3, 3), "w"), (PREFIX + "conv2d2.bias", (DS,), "b"),
         (PREFIX + "conv2d3.weight", (DS, DS, 3, 3), "w"), (PREFIX + "conv2d3.bias", (DS,), "b"),
         (PREFIX + "conv_out.weight", (D, DS * 16), "w"),
         (PREFIX + "ln_post.weight", (D,), "g"), (PREFIX + "ln_post.bias", (D,), "s"),
         (PREFIX + "proj1.weight", (D, D), "w"), (PREFIX + "proj1.bias", (D,), "b"),
         (PREFIX + "proj2.weight", (OUT, D), "w"), (PREFIX + "proj2.bias", (OUT,), "b")]
    for i in range(layers):
        p = f"{PREFIX}layers.{i}."
        t += [(p + "self_attn_layer_norm.weight", (D,), "g"), (p + "self_attn_layer_norm.bias", (D,), "s")]
        for m in ("q_proj", "k_proj", "v_proj", "out_proj"):
            t += [(p + f"self_attn.{m}.weight", (D, D), "w"), (p + f"self_attn.{m}.bias", (D,), "b")]
        t += [(p + "final_layer_norm.weight", (D,), "g"), (p + "final_layer_norm.bias", (D,), "s"),
              (p + "fc1.weight", (FFN, D), "w"), (p + "fc1.bias", (FFN,), "b"),
              (p + "fc2.weight", (D, FFN), "w"), (p + "fc2.bias", (D,), "b")]
    return t


def std_mean(shape, kind):
    if kind == "w":
        return 1.0 / math.sqrt(int(np.prod(shape[1:]))), 0.0
    if kind == "g":
        return 0.02, 1.0
    return 0.02, 0.0


def synthetic_weights(layers: int, seed: int = 5, normal=None) -> dict:
    """``normal(seed, tid, n, std, mean)`` may replace synth.normal_f32 (e.g.
    by its bit-exact GPU twin for the 24-layer tower)."""
    normal = normal or synth.normal_f32
    w = {}
    for i, (name, shape, kind) in enumerate(tensor_list(layers)):
        sd, mu = std_mean(shape, kind)
        v = normal(seed, TID + i, int(np.prod(shape)), sd, mu)
        w[name] = synth.bf16_round(v).reshape(shape)
    return w


def bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def linear(x, w, b=None, act=0):
    """asr_gemm::Linear: bf16(x) @ W^T in fp32 (+ bias, act 1 = GELU)."""
    y = bf16(x) @ w.T
    if b is not None:
        y = y + b
    if act == 1:
        y = 0.5 * y * (1.0 + torch.erf(y * 0.70710678118654752440))
    return y


def layer_norm(x, g, s, eps=1e-5):
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) * torch.rsqrt(var + eps) * g + s


def positional(T: int) -> torch.Tensor:
    """Sinusoidal code (asr_audio_tower.cu:285-300): sin | cos halves."""
    inc = math.log(10000.0) / (D // 2 - 1)
    pos = np.arange(T, dtype=np.float64)[:, None]
    inv = np.exp(-inc * np.arange(D // 2, dtype=np.float64))[None, :]
    pe = np.concatenate([np.sin(pos * inv), np.cos(pos * inv)], 1).astype(np.float32)
    return torch.from_numpy(pe)


class TowerOracle:
    def __init__(self, weights: dict, layers: int):
        self.w = {k: torch.from_numpy(np.asarray(v, np.float32)) for k, v in weights.items()}
        self.L = layers

    def conv(self, x, name):
        """x [B, Cin, H, W] -> GELU(conv3x3 s2 p1 + b) with bf16 operands."""
        w = self.w[PREFIX + name + ".weight"]
        b = self.w[PREFIX + name + ".bias"]
        B, cin, hh, ww = x.shape
        cols = torch.nn.functional.unfold(x, 3, padding=1, stride=2)         # [B, Cin*9, L]
        ho, wo = conv_out_len(hh), conv_out_len(ww)
        y = bf16(cols).transpose(1, 2) @ w.reshape(w.shape[0], -1).T          # [B, L, Cout]
        y = y + b
        y = 0.5 * y * (1.0 + torch.erf(y * 0.70710678118654752440))
        return y.transpose(1, 2).reshape(B, -1, ho, wo)

    @torch.no_grad()
    def forward(self, mel: np.ndarray) -> np.ndarray:
        """mel [128, n_frames] -> [N, 2048]."""
        mel = torch.from_numpy(np.asarray(mel, np.float32))
        n = mel.shape[1]
        chunks = (n + 99) // 100
        lens = [100] * chunks
        if n % 100:
            lens[-1] = n % 100
        mcl = max(lens)
        x = torch.zeros(chunks, 1, F, mcl)
        for c in range(chunks):
            x[c, 0, :, :lens[c]] = mel[:, c * 100:c * 100 + lens[c]]
        c3 = self.conv(self.conv(self.conv(x, "conv2d1"), "conv2d2"), "conv2d3")  # [B, 480, 16, Wc]
        B, _, hc3, wc = c3.shape
        feat = c3.permute(0, 3, 1, 2).reshape(B * wc, DS * hc3)                  # (chunk, t) x (co, f)
        h = linear(feat, self.w[PREFIX + "conv_out.weight"])
        h = h.reshape(B, wc, D) + positional(wc)[None]
        rows = [h[c, :output_length(lens[c])] for c in range(chunks)]
        x = torch.cat(rows, 0)
        W = lambda k: self.w[k]
        for i in range(self.L):
            p = f"{PREFIX}layers.{i}."
            y = layer_norm(x, W(p + "self_attn_layer_norm.weight"), W(p + "self_attn_layer_norm.bias"))
            q, k, v = (linear(y, W(p + f"self_attn.{m}.weight"), W(p + f"self_attn.{m}.bias"))
                       for m in ("q_proj", "k_proj", "v_proj"))
            N = x.shape[0]
            q, k, v = (t.reshape(N, H, DH).transpose(0, 1) for t in (q, k, v))
            att = torch.softmax((q @ k.transpose(1, 2)) / math.sqrt(DH), -1) @ v
            att = att.transpose(0, 1).reshape(N, D)
            x = x + linear(att, W(p + "self_attn.out_proj.weight"), W(p + "self_attn.out_proj.bias"))
            y = layer_norm(x, W(p + "final_layer_norm.weight"), W(p + "final_layer_norm.bias"))
            y = linear(y, W(p + "fc1.weight"), W(p + "fc1.bias"), act=1)
            x = x + linear(y, W(p + "fc2.weight"), W(p + "fc2.bias"))
        y = layer_norm(x, W(PREFIX + "ln_post.weight"), W(PREFIX + "ln_post.bias"))
        y = linear(y, W(PREFIX + "proj1.weight"), W(PREFIX + "proj1.bias"), act=1)
        y = linear(y, W(PREFIX + "proj2.weight"), W(PREFIX + "proj2.bias"))
        return y.numpy()


def write_checkpoint(out_dir: str, weights: dict, layers: int) -> str:
    """The tower's tensors as one bf16 safetensors shard plus the index the
    reference's ShardedSafeTensors reads."""
    import json
    import os
    from . import st_writer
    os.makedirs(out_dir, exist_ok=True)
    names = [n for n, _, _ in tensor_list(layers)]
    tens = [(n, synth.f32_to_bf16_bits(weights[n]).reshape(weights[n].shape)) for n in names]
    st_writer.write_shard(os.path.join(out_dir, "model-00001-of-00001.safetensors"), tens)
    with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": {n: "model-00001-of-00001.safetensors" for n in names}}, f)
    return out_dir
