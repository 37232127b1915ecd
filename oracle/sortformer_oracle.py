"""CPU restatement of the reference's streaming Sortformer diarizer network
(TEST INFRASTRUCTURE: the checker of the B200 Sortformer step, never the
product). fp32 throughout, torch on the host cores.

Follows, operation for operation:
* ConformerPreEncode::Forward (src/model/conformer_preencode.cu:196-279):
  time-major mel [T, 128] with frames >= valid zeroed; conv 1->256 3x3 s2 p1
  + bias, mask, ReLU; depthwise 3x3 s2 + bias; pointwise 256->256 + bias,
  ReLU, mask; depthwise 3x3 s2 + bias; pointwise + bias, ReLU, mask; flatten
  (channel, freq) and Linear 4096 -> 512. Masks zero time rows at or past the
  valid length of that stage (ConvOutLen of the previous one).
* ConformerLayer::Forward (src/model/conformer_layer.cu:330-452): macaron
  FF (SiLU, half residual), relative-position MHSA with pos_bias_u / v and
  the rel_shift of RelShiftScoresKernel (score(i, j) uses projected position
  row T - 1 - i + j), keys >= valid masked, conv module (pointwise 512->1024,
  GLU, rows >= valid zeroed, depthwise k9, BatchNorm with running stats, SiLU,
  pointwise), second FF, final LayerNorm; LayerNorm eps 1e-5.
* ConformerLayer::BuildPosEmb (:296-312): rows idx = 0..2T-2 at position
  T - 1 - idx, interleaved sin / cos with div = exp(-ln(1e4) * i / d).
* SortformerDecoder::Forward (src/model/sortformer_decoder.cu:240-333):
  encoder_proj 512->192, 18 post-LN transformer layers (8 heads of 24, keys
  >= valid masked, ReLU FFN 768), head ReLU -> Linear + ReLU -> Linear +
  sigmoid, rows >= valid zeroed.
* SortformerDiarizer::ForwardEncoderDecoder (src/model/streaming_sortformer.cc
  :391-418): x * sqrt(512), the conformer stack, the decoder, preds of rows
  >= valid zeroed.

Synthetic weights (seed 3): tensor ids 90000 + i in ``tensor_list`` order;
matrices and conv kernels N(0, 1/fan_in), biases and pos_bias_u / v
N(0, 0.02^2), LayerNorm / BatchNorm gains 1 + N(0, 0.02^2), BatchNorm
running_var 1 + |N(0, 0.1^2)|; fp32 (not rounded).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import synth

D, H, DK, DFF, KCONV = 512, 8, 64, 2048, 9
CH, MELS = 256, 128
DD, DH, DDK, DDFF, NSPK = 192, 8, 24, 768, 4
TID = 90000
EPS = 1e-5


def conv_len(x: int) -> int:
    """ConvOutLen(x, 3, 2, 1)."""
    return (x + 2 - 3) // 2 + 1


def tensor_list(conf_layers: int = 17, dec_layers: int = 18):
    """(name, shape, kind): w = fan-in scaled, b = bias, g = gain (mean 1),
    v = BatchNorm running variance."""
    P = "encoder.pre_encode."
    t = [(P + "conv.0.weight", (CH, 1, 3, 3), "w"), (P + "conv.0.bias", (CH,), "b"),
         (P + "conv.2.weight", (CH, 1, 3, 3), "w"), (P + "conv.2.bias", (CH,), "b"),
         (P + "conv.3.weight", (CH, CH, 1, 1), "w"), (P + "conv.3.bias", (CH,), "b"),
         (P + "conv.5.weight", (CH, 1, 3, 3), "w"), (P + "conv.5.bias", (CH,), "b"),
         (P + "conv.6.weight", (CH, CH, 1, 1), "w"), (P + "conv.6.bias", (CH,), "b"),
         (P + "out.weight", (D, CH * 16), "w"), (P + "out.bias", (D,), "b")]
    for i in range(conf_layers):
        p = f"encoder.layers.{i}."
        for ff in ("feed_forward1",):
            t += [(p + "norm_feed_forward1.weight", (D,), "g"), (p + "norm_feed_forward1.bias", (D,), "b"),
                  (p + ff + ".linear1.weight", (DFF, D), "w"), (p + ff + ".linear1.bias", (DFF,), "b"),
                  (p + ff + ".linear2.weight", (D, DFF), "w"), (p + ff + ".linear2.bias", (D,), "b")]
        t += [(p + "norm_self_att.weight", (D,), "g"), (p + "norm_self_att.bias", (D,), "b")]
        for m in ("linear_q", "linear_k", "linear_v", "linear_out"):
            t += [(p + f"self_attn.{m}.weight", (D, D), "w"), (p + f"self_attn.{m}.bias", (D,), "b")]
        t += [(p + "self_attn.linear_pos.weight", (D, D), "w"),
              (p + "self_attn.pos_bias_u", (H, DK), "b"), (p + "self_attn.pos_bias_v", (H, DK), "b"),
              (p + "norm_conv.weight", (D,), "g"), (p + "norm_conv.bias", (D,), "b"),
              (p + "conv.pointwise_conv1.weight", (2 * D, D, 1), "w"),
              (p + "conv.pointwise_conv1.bias", (2 * D,), "b"),
              (p + "conv.depthwise_conv.weight", (D, 1, KCONV), "w"),
              (p + "conv.depthwise_conv.bias", (D,), "b"),
              (p + "conv.batch_norm.weight", (D,), "g"), (p + "conv.batch_norm.bias", (D,), "b"),
              (p + "conv.batch_norm.running_mean", (D,), "b"),
              (p + "conv.batch_norm.running_var", (D,), "v"),
              (p + "conv.pointwise_conv2.weight", (D, D, 1), "w"),
              (p + "conv.pointwise_conv2.bias", (D,), "b"),
              (p + "norm_feed_forward2.weight", (D,), "g"), (p + "norm_feed_forward2.bias", (D,), "b"),
              (p + "feed_forward2.linear1.weight", (DFF, D), "w"),
              (p + "feed_forward2.linear1.bias", (DFF,), "b"),
              (p + "feed_forward2.linear2.weight", (D, DFF), "w"),
              (p + "feed_forward2.linear2.bias", (D,), "b"),
              (p + "norm_out.weight", (D,), "g"), (p + "norm_out.bias", (D,), "b")]
    S = "sortformer_modules."
    t += [(S + "encoder_proj.weight", (DD, D), "w"), (S + "encoder_proj.bias", (DD,), "b"),
          (S + "first_hidden_to_hidden.weight", (DD, DD), "w"),
          (S + "first_hidden_to_hidden.bias", (DD,), "b"),
          (S + "single_hidden_to_spks.weight", (NSPK, DD), "w"),
          (S + "single_hidden_to_spks.bias", (NSPK,), "b")]
    for i in range(dec_layers):
        p = f"transformer_encoder.layers.{i}."
        for m, shp in (("first_sub_layer.query_net", (DD, DD)), ("first_sub_layer.key_net", (DD, DD)),
                       ("first_sub_layer.value_net", (DD, DD)),
                       ("first_sub_layer.out_projection", (DD, DD)),
                       ("second_sub_layer.dense_in", (DDFF, DD)),
                       ("second_sub_layer.dense_out", (DD, DDFF))):
            t += [(p + m + ".weight", shp, "w"), (p + m + ".bias", (shp[0],), "b")]
        t += [(p + "layer_norm_1.weight", (DD,), "g"), (p + "layer_norm_1.bias", (DD,), "b"),
              (p + "layer_norm_2.weight", (DD,), "g"), (p + "layer_norm_2.bias", (DD,), "b")]
    return t


def std_mean(shape, kind):
    if kind == "w":
        return 1.0 / math.sqrt(int(np.prod(shape[1:]))), 0.0
    if kind == "g":
        return 0.02, 1.0
    if kind == "v":
        return 0.1, 0.0
    return 0.02, 0.0


def synthetic_weights(conf_layers: int = 17, dec_layers: int = 18, seed: int = 3, normal=None):
    normal = normal or synth.normal_f32
    w = {}
    for i, (name, shape, kind) in enumerate(tensor_list(conf_layers, dec_layers)):
        sd, mu = std_mean(shape, kind)
        v = np.asarray(normal(seed, TID + i, int(np.prod(shape)), sd, mu), np.float32)
        if kind == "v":
            v = (1.0 + np.abs(v)).astype(np.float32)
        w[name] = v.reshape(shape)
    return w


def synthetic_mel(seed: int, n_frames: int) -> np.ndarray:
    """[128, n_frames] N(0, 1) log-mel (freq-major, the reference's layout)."""
    return synth.normal_f32(seed, 91000, MELS * n_frames, 1.0).reshape(MELS, n_frames)


def pos_emb(T: int) -> torch.Tensor:
    """ConformerLayer::BuildPosEmb, in the reference's fp32 arithmetic."""
    P = 2 * T - 1
    pos = torch.arange(T - 1, -T, -1, dtype=torch.float32)[:, None]       # T-1-idx
    div = torch.from_numpy(np.exp(-np.float32(math.log(10000.0)) * np.arange(0, D, 2, dtype=np.float32)
                                  / np.float32(D)).astype(np.float32))
    ang = pos * div[None, :]
    pe = torch.empty(P, D)
    pe[:, 0::2] = torch.sin(ang)
    pe[:, 1::2] = torch.cos(ang)
    return pe


def layer_norm(x, g, b):
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) * torch.rsqrt(var + EPS) * g + b


def silu(x):
    return x / (1.0 + torch.exp(-x))


class SortformerOracle:
    def __init__(self, weights: dict, conf_layers: int = 17, dec_layers: int = 18):
        self.w = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)) for k, v in weights.items()}
        self.L, self.DL = conf_layers, dec_layers

    def W(self, k):
        return self.w[k]

    # ---- pre-encode ----
    @torch.no_grad()
    def pre_encode(self, mel: np.ndarray, valid: int):
        """mel [128, n_frames] (freq-major) -> (emb [T2, 512], T2, valid2)."""
        P = "encoder.pre_encode."
        W = self.W
        x = torch.from_numpy(np.ascontiguousarray(mel, np.float32)).t().contiguous()  # [T, 128]
        n = x.shape[0]
        x[valid:] = 0
        x = x[None, None]                                                        # [1,1,T,F]
        y = torch.nn.functional.conv2d(x, W(P + "conv.0.weight"), W(P + "conv.0.bias"), 2, 1)
        l0 = conv_len(valid)
        y[:, :, l0:] = 0
        y = torch.relu(y)
        y = torch.nn.functional.conv2d(y, W(P + "conv.2.weight"), W(P + "conv.2.bias"), 2, 1, groups=CH)
        l1 = conv_len(l0)
        y = torch.nn.functional.conv2d(y, W(P + "conv.3.weight"), W(P + "conv.3.bias"))
        y = torch.relu(y)
        y[:, :, l1:] = 0
        y = torch.nn.functional.conv2d(y, W(P + "conv.5.weight"), W(P + "conv.5.bias"), 2, 1, groups=CH)
        l2 = conv_len(l1)
        y = torch.nn.functional.conv2d(y, W(P + "conv.6.weight"), W(P + "conv.6.bias"))
        y = torch.relu(y)
        y[:, :, l2:] = 0
        _, C, T2, F2 = y.shape
        flat = y[0].permute(1, 0, 2).reshape(T2, C * F2)                          # (c, f) c-major
        out = flat @ W(P + "out.weight").t() + W(P + "out.bias")
        return out.numpy(), T2, l2

    # ---- conformer layer ----
    def conformer_layer(self, x, i, valid, pp):
        W = lambda k: self.W(f"encoder.layers.{i}." + k)
        T = x.shape[0]
        y = layer_norm(x, W("norm_feed_forward1.weight"), W("norm_feed_forward1.bias"))
        y = silu(y @ W("feed_forward1.linear1.weight").t() + W("feed_forward1.linear1.bias"))
        x = x + 0.5 * (y @ W("feed_forward1.linear2.weight").t() + W("feed_forward1.linear2.bias"))
        y = layer_norm(x, W("norm_self_att.weight"), W("norm_self_att.bias"))
        q = (y @ W("self_attn.linear_q.weight").t() + W("self_attn.linear_q.bias")).view(T, H, DK)
        k = (y @ W("self_attn.linear_k.weight").t() + W("self_attn.linear_k.bias")).view(T, H, DK)
        v = (y @ W("self_attn.linear_v.weight").t() + W("self_attn.linear_v.bias")).view(T, H, DK)
        p = (pp @ W("self_attn.linear_pos.weight").t()).view(2 * T - 1, H, DK)
        qu = (q + W("self_attn.pos_bias_u")).transpose(0, 1)                     # [H, T, DK]
        qv = (q + W("self_attn.pos_bias_v")).transpose(0, 1)
        ac = qu @ k.transpose(0, 1).transpose(1, 2)                               # [H, T, T]
        bd_full = qv @ p.transpose(0, 1).transpose(1, 2)                          # [H, T, 2T-1]
        ii = torch.arange(T)[:, None]
        jj = torch.arange(T)[None, :]
        bd = bd_full[:, ii, T - 1 - ii + jj]                                      # rel_shift
        s = (ac + bd) / math.sqrt(DK)
        s[:, :, valid:] = -1e30
        a = torch.softmax(s, -1) @ v.transpose(0, 1)                              # [H, T, DK]
        a = a.transpose(0, 1).reshape(T, D)
        x = x + (a @ W("self_attn.linear_out.weight").t() + W("self_attn.linear_out.bias"))
        y = layer_norm(x, W("norm_conv.weight"), W("norm_conv.bias"))
        y = y @ W("conv.pointwise_conv1.weight")[:, :, 0].t() + W("conv.pointwise_conv1.bias")
        g = y[:, :D] * torch.sigmoid(y[:, D:])
        g[valid:] = 0
        dw = torch.nn.functional.conv1d(g.t()[None], W("conv.depthwise_conv.weight"),
                                        W("conv.depthwise_conv.bias"), padding=KCONV // 2,
                                        groups=D)[0].t()
        bn = (dw - W("conv.batch_norm.running_mean")) * torch.rsqrt(
            W("conv.batch_norm.running_var") + EPS) * W("conv.batch_norm.weight") + W("conv.batch_norm.bias")
        y = silu(bn) @ W("conv.pointwise_conv2.weight")[:, :, 0].t() + W("conv.pointwise_conv2.bias")
        x = x + y
        y = layer_norm(x, W("norm_feed_forward2.weight"), W("norm_feed_forward2.bias"))
        y = silu(y @ W("feed_forward2.linear1.weight").t() + W("feed_forward2.linear1.bias"))
        x = x + 0.5 * (y @ W("feed_forward2.linear2.weight").t() + W("feed_forward2.linear2.bias"))
        return layer_norm(x, W("norm_out.weight"), W("norm_out.bias"))

    def decoder(self, x, valid):
        S = "sortformer_modules."
        T = x.shape[0]
        x = x @ self.W(S + "encoder_proj.weight").t() + self.W(S + "encoder_proj.bias")
        for i in range(self.DL):
            W = lambda k: self.W(f"transformer_encoder.layers.{i}." + k)
            lin = lambda y, m: y @ W(m + ".weight").t() + W(m + ".bias")
            q = lin(x, "first_sub_layer.query_net").view(T, DH, DDK).transpose(0, 1)
            k = lin(x, "first_sub_layer.key_net").view(T, DH, DDK).transpose(0, 1)
            v = lin(x, "first_sub_layer.value_net").view(T, DH, DDK).transpose(0, 1)
            s = (q @ k.transpose(1, 2)) / math.sqrt(DDK)
            s[:, :, valid:] = -1e30
            a = (torch.softmax(s, -1) @ v).transpose(0, 1).reshape(T, DD)
            x = layer_norm(lin(a, "first_sub_layer.out_projection") + x,
                           W("layer_norm_1.weight"), W("layer_norm_1.bias"))
            f = torch.relu(lin(x, "second_sub_layer.dense_in"))
            x = layer_norm(lin(f, "second_sub_layer.dense_out") + x,
                           W("layer_norm_2.weight"), W("layer_norm_2.bias"))
        h = torch.relu(torch.relu(x) @ self.W(S + "first_hidden_to_hidden.weight").t()
                       + self.W(S + "first_hidden_to_hidden.bias"))
        p = torch.sigmoid(h @ self.W(S + "single_hidden_to_spks.weight").t()
                          + self.W(S + "single_hidden_to_spks.bias"))
        p[valid:] = 0
        return p

    @torch.no_grad()
    def encode_decode(self, emb: np.ndarray, valid: int) -> np.ndarray:
        """ForwardEncoderDecoder: emb [T, 512] -> preds [T, 4]."""
        x = torch.from_numpy(np.ascontiguousarray(emb, np.float32)) * np.float32(math.sqrt(D))
        T = x.shape[0]
        pp = pos_emb(T)
        for i in range(self.L):
            x = self.conformer_layer(x, i, valid, pp)
        return self.decoder(x, valid).numpy()


def write_safetensors(path: str, weights: dict, conf_layers: int, dec_layers: int) -> str:
    """One F32 safetensors file (the reference reads it with SafeTensorReader)."""
    import json
    import struct
    header, off, blobs = {}, 0, []
    for name, shape, _ in tensor_list(conf_layers, dec_layers):
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
