"""Seeded synthetic weights and inputs, bit-exact between this numpy code and
the CUDA generator in ``orator_b200/csrc/synth.cu``.

TEST INFRASTRUCTURE: part of the oracle. Only ``tests/``, ``bench.py``'s CPU
baseline leg and ``__graft_entry__.smoke()`` may import it.

There are no checkpoints on this pool, so both the reference decoder and this
build load random-init weights with the tensor names and shapes pinned by the
reference loader (``src/model/asr_text_decoder.cu:251-307``; the name list is
checked in ``test/unit/model/test_asr_weights.cc:46-56``).

Generator: element ``i`` of tensor ``tid`` under ``seed`` is
``splitmix64((seed << 52) | (tid << 36) | i)``; the four 16-bit fields of the
hash are summed (Irwin-Hall of 4, mean 131070, sd 37837.227), centred as an
exact integer, converted to fp32, multiplied by ``std / 37837.227`` and offset
by ``mean`` (two separately rounded fp32 operations, no FMA).  bf16 tensors are
then rounded to nearest even.  Integer-only hashing makes the CPU and GPU
streams identical bit for bit.
"""
from __future__ import annotations

import os

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
IH_SD = 37837.227  # sqrt(4 * (65536**2 - 1) / 12)

# Tensor ids (shared with csrc/synth.cu).
TID_EMBED = 0
TID_FINAL_NORM = 1
TID_AUDIO = 60000
TID_TOKENS = 60001
LAYER_BASE = 16
LAYER_STRIDE = 16
LAYER_TENSORS = ["input_layernorm", "post_attention_layernorm", "self_attn.q_norm",
                 "self_attn.k_norm", "self_attn.q_proj", "self_attn.k_proj",
                 "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
                 "mlp.up_proj", "mlp.down_proj"]
NORM_STD = 0.02
MATRIX_STD = 0.02


def layer_tid(layer: int, j: int) -> int:
    return LAYER_BASE + layer * LAYER_STRIDE + j


def splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        z = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def hashes(seed: int, tid: int, start: int, n: int) -> np.ndarray:
    base = (np.uint64(seed & 0xFFF) << np.uint64(52)) | (np.uint64(tid & 0xFFFF) << np.uint64(36))
    idx = np.arange(start, start + n, dtype=np.uint64)
    return splitmix64(base | idx)


def normal_f32(seed: int, tid: int, n: int, std: float, mean: float = 0.0,
               chunk: int = 1 << 22) -> np.ndarray:
    """Approximately N(mean, std) fp32 values; bit-exact with the CUDA twin."""
    out = np.empty(n, dtype=np.float32)
    scale = np.float32(std / IH_SD)
    m = np.float32(mean)
    f16 = np.uint64(0xFFFF)

    def fill(s):
        c = min(chunk, n - s)
        h = hashes(seed, tid, s, c)
        tot = ((h & f16) + ((h >> np.uint64(16)) & f16) + ((h >> np.uint64(32)) & f16)
               + (h >> np.uint64(48))).astype(np.int64) - 131070
        v = tot.astype(np.float32) * scale
        if mean != 0.0:
            v = v + m
        out[s:s + c] = v

    starts = range(0, n, chunk)
    if n > 4 * chunk:
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 4)) as ex:
            list(ex.map(fill, starts))
    else:
        for s in starts:
            fill(s)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit pattern (finite inputs), the
    same rounding as ``__float2bfloat16`` and the reference's host helper
    ``HostF32ToBf16`` (test/unit/model/test_asr_gemm.cc:21-27)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((b + r) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def token_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    h = hashes(seed, TID_TOKENS, 0, n)
    return ((h >> np.uint64(11)) % np.uint64(vocab)).astype(np.int32)


def audio_rows(seed: int, n: int, hidden: int) -> np.ndarray:
    return normal_f32(seed, TID_AUDIO, n * hidden, 1.0).reshape(n, hidden)


def model_tensors(seed: int, num_layers: int, vocab: int, hidden: int = 2048,
                  q_heads: int = 16, kv_heads: int = 8, head_dim: int = 128,
                  inter: int = 6144, dtype: str = "bf16"):
    """Yield (hf_name, tid, shape, is_norm) in reference load order."""
    pre = "thinker.model."
    yield pre + "embed_tokens.weight", TID_EMBED, (vocab, hidden), False
    yield pre + "norm.weight", TID_FINAL_NORM, (hidden,), True
    shapes = [(hidden,), (hidden,), (head_dim,), (head_dim,),
              (q_heads * head_dim, hidden), (kv_heads * head_dim, hidden),
              (kv_heads * head_dim, hidden), (hidden, q_heads * head_dim),
              (inter, hidden), (inter, hidden), (hidden, inter)]
    for l in range(num_layers):
        for j, (nm, shp) in enumerate(zip(LAYER_TENSORS, shapes)):
            yield f"{pre}layers.{l}.{nm}.weight", layer_tid(l, j), shp, j < 4


def make_tensor(seed: int, tid: int, shape, is_norm: bool, bf16: bool = True) -> np.ndarray:
    """fp32 array holding the (bf16-rounded when ``bf16``) synthetic values.
    Norm weights are 1 + N(0, 0.02): unit-gain norms keep logit margins
    meaningful for greedy-token parity."""
    n = int(np.prod(shape))
    if is_norm:
        v = normal_f32(seed, tid, n, NORM_STD, 1.0)
    else:
        v = normal_f32(seed, tid, n, MATRIX_STD)
    if bf16:
        v = bf16_round(v)
    return v.reshape(shape)
