"""Python mirror of the reference's free operators over the C ABI.

``asr_ops`` (include/model/asr_ops.cuh:22-62): RmsNorm, RopeHalf,
RopeInterleaved, SwiGLU, GqaAttention, ArgmaxBanned; ``asr_gemm``
(include/model/asr_gemm.h:22-41): F32ToBf16, Bf16ToF32, Linear, LinearPre.
Arguments are device addresses (ints, e.g. ``torch.Tensor.data_ptr()``) and
sizes with the reference's meaning; calls are asynchronous on ``stream`` and
raise ``OrxError`` where the reference throws.
"""
from __future__ import annotations

import ctypes as C

from ._lib import call
from .decoder import _stream

P = C.c_void_p


def RmsNorm(x: int, weight: int, out: int, rows: int, dim: int, eps: float, stream=None):
    call("orx_rms_norm", P(x), P(weight), P(out), rows, dim, eps, _stream(stream))


def RopeHalf(x: int, positions: int, n_tokens: int, n_heads: int, head_dim: int,
             theta_base: float, stream=None):
    call("orx_rope_half", P(x), P(positions), n_tokens, n_heads, head_dim, theta_base,
         _stream(stream))


def RopeInterleaved(x: int, positions: int, n_tokens: int, n_heads: int, head_dim: int,
                    theta_base: float, stream=None):
    call("orx_rope_interleaved", P(x), P(positions), n_tokens, n_heads, head_dim, theta_base,
         _stream(stream))


def SwiGLU(gate: int, up: int, out: int, n: int, stream=None):
    call("orx_swiglu", P(gate), P(up), P(out), n, _stream(stream))


def GqaAttention(q: int, k: int, v: int, out: int, T: int, Hq: int, Hkv: int, Dh: int,
                 scale: float, causal: bool, stream=None):
    call("orx_gqa_attention", P(q), P(k), P(v), P(out), T, Hq, Hkv, Dh, scale, int(causal),
         _stream(stream))


def ArgmaxBanned(logits: int, n: int, ban0: int, ban1: int, out_idx: int, stream=None):
    call("orx_argmax_banned", P(logits), n, ban0, ban1, P(out_idx), _stream(stream))


def F32ToBf16(inp: int, out: int, n: int, stream=None):
    call("orx_f32_to_bf16", P(inp), P(out), n, _stream(stream))


def Bf16ToF32(inp: int, out: int, n: int, stream=None):
    call("orx_bf16_to_f32", P(inp), P(out), n, _stream(stream))


def Linear(in_f32: int, W_bf16: int, bias_f32: int | None, out_f32: int, M: int, K: int, N: int,
           act: int = 0, stream=None):
    call("orx_linear", P(in_f32), P(W_bf16), P(bias_f32 or 0), P(out_f32), M, K, N, act,
         _stream(stream))


def LinearPre(in_bf16: int, W_bf16: int, bias_f32: int | None, out_f32: int, M: int, K: int,
              N: int, act: int = 0, stream=None):
    call("orx_linear_pre", P(in_bf16), P(W_bf16), P(bias_f32 or 0), P(out_f32), M, K, N, act,
         _stream(stream))
