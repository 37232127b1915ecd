"""CPU restatement of the reference Qwen3-ASR text decoder (``AsrTextDecoder``).

TEST INFRASTRUCTURE ONLY: this is the parity checker and the timed CPU
baseline.  Only ``tests/``, ``bench.py`` (CPU-baseline / reference arm) and
``__graft_entry__.smoke()`` may import it; the product never does.

Follows the reference step by step, at its quantization points:

* RMSNorm ``y = x * rsqrtf(sum(x^2)/dim + eps) * w`` in fp32
  (``src/model/asr_ops.cu:21-51``);
* every projection rounds its fp32 activation to bf16 (RNE) and multiplies by
  bf16 weights with fp32 accumulation (``src/model/asr_gemm.cu:162-215``);
* per-head q_norm / k_norm before rotate-half RoPE with
  ``inv_freq = powf(theta, -2j/Dh)`` and ``angle = (float)pos * inv_freq``
  (``src/model/asr_ops.cu:92-111``; order in ``src/model/asr_text_decoder.cu:404-411``);
* K (after norm+RoPE) and V stored as bf16 (``asr_text_decoder.cu:62-77``) and
  attention computed in fp32 against the bf16 cache, scale 1/sqrt(128)
  (``asr_text_decoder.cu:88-213``);
* SwiGLU ``g/(1+expf(-g))*u`` (``src/model/asr_ops.cu:80-87``), residual adds in fp32;
* final norm on the last row, tied lm_head (``asr_text_decoder.cu:255-257,560-567``);
* greedy argmax with up to two banned ids and the reference's tie rule
  (``src/model/asr_ops.cu:300-325``) and the ``DecodeGreedy`` control loop
  (``asr_text_decoder.cu:698-889``).

``quantize=False`` removes the bf16 activation/KV rounding so the same code can
be cross-checked against transformers' ``Qwen3ForCausalLM`` in fp32.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import synth


@dataclass
class Config:
    """Mirrors ``AsrTextConfig`` (include/model/asr_text_decoder.h:30-43)."""
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


def bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    ss = (x * x).sum(-1, keepdim=True)
    inv = torch.rsqrt(ss / x.shape[-1] + eps)
    return x * inv * w


def rope_tables(cfg: Config, max_pos: int):
    """cos/sin [max_pos, Dh/2] with the reference's fp32 angle math."""
    half = cfg.head_dim // 2
    j = np.arange(half, dtype=np.float32)
    expo = (np.float32(-2.0) * j) / np.float32(cfg.head_dim)
    inv_freq = np.power(np.float32(cfg.rope_theta), expo, dtype=np.float32)
    pos = np.arange(max_pos, dtype=np.float32)
    ang = (pos[:, None] * inv_freq[None, :]).astype(np.float32)
    # angle is fp32; cos/sin evaluated accurately then rounded to fp32
    c = np.cos(ang.astype(np.float64)).astype(np.float32)
    s = np.sin(ang.astype(np.float64)).astype(np.float32)
    return torch.from_numpy(c), torch.from_numpy(s)


def rope_half(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, Dh]; cos/sin [T, Dh/2]."""
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


def argmax_banned(logits: np.ndarray, ban0: int = -1, ban1: int = -1) -> int:
    """Reference tie rule (asr_ops.cu:300-325): thread t of 256 keeps the first
    strict max of i = t (mod 256) above -1e30; the shared-memory tree pairs
    slot t with t + s (s = 128 .. 1) and takes t + s only when strictly
    greater. Restated step by step, so no closed form is assumed here."""
    x = np.asarray(logits, dtype=np.float32).copy()
    x[np.isnan(x)] = -np.inf  # `v > best` is false for NaN: it never wins, like -inf
    n = x.shape[0]
    for b in (ban0, ban1):
        if 0 <= b < n:
            x[b] = -np.inf
    pad = (-n) % 256
    xp = np.concatenate([x, np.full(pad, -np.inf, np.float32)]).reshape(-1, 256)
    slot_best = xp.max(axis=0)
    slot_idx = xp.argmax(axis=0) * 256 + np.arange(256)
    # threads that never beat the -1e30 init keep index 0
    slot_best = np.where(slot_best > np.float32(-1e30), slot_best, np.float32(-1e30))
    slot_idx = np.where(slot_best > np.float32(-1e30), slot_idx, 0)
    # tree reduce: replace only on strictly greater
    vals, idxs = slot_best.copy(), slot_idx.copy()
    s = 128
    while s > 0:
        take = vals[s:2 * s] > vals[:s]
        vals[:s] = np.where(take, vals[s:2 * s], vals[:s])
        idxs[:s] = np.where(take, idxs[s:2 * s], idxs[:s])
        s //= 2
    return int(idxs[0])


class OracleDecoder:
    """fp32 CPU restatement of ``AsrTextDecoder`` (one session, contiguous KV)."""

    def __init__(self, cfg: Config, weights: dict, quantize: bool = True,
                 threads: int | None = None):
        self.cfg = cfg
        self.q = quantize
        if threads:
            torch.set_num_threads(threads)
        pre = "thinker.model."
        t = lambda n: torch.as_tensor(weights[pre + n], dtype=torch.float32)
        self.embed = t("embed_tokens.weight")
        self.final_norm = t("norm.weight")
        self.layers = []
        for l in range(cfg.num_layers):
            p = f"layers.{l}."
            L = {k: t(p + k + ".weight") for k in synth.LAYER_TENSORS}
            L["qkv"] = torch.cat([L["self_attn.q_proj"], L["self_attn.k_proj"],
                                  L["self_attn.v_proj"]], 0)
            L["gateup"] = torch.cat([L["mlp.gate_proj"], L["mlp.up_proj"]], 0)
            self.layers.append(L)
        kvd = cfg.num_kv_heads * cfg.head_dim
        self.kc = [torch.zeros(cfg.max_seq_len, kvd) for _ in range(cfg.num_layers)]
        self.vc = [torch.zeros(cfg.max_seq_len, kvd) for _ in range(cfg.num_layers)]
        self.cos, self.sin = rope_tables(cfg, cfg.max_seq_len)
        self.cache_len = 0
        self.logits = None

    @classmethod
    def synthetic(cls, cfg: Config, seed: int, **kw):
        return cls(cfg, synthetic_weights(cfg, seed), **kw)

    # --- helpers -----------------------------------------------------------
    def _cast(self, x):
        return bf16(x) if self.q else x

    def _linear(self, x, w):
        return self._cast(x) @ w.T

    def embed_row(self, tok: int) -> np.ndarray:
        return self.embed[tok].numpy().copy()

    def reset(self):
        self.cache_len = 0

    def truncate(self, n: int):
        self.cache_len = n

    # --- forward (Forward / DecodeForwardOnStream) -------------------------
    @torch.no_grad()
    def forward(self, x: np.ndarray, pos0: int) -> np.ndarray:
        c = self.cfg
        x = torch.as_tensor(np.asarray(x, np.float32)).reshape(-1, c.hidden_size).clone()
        T = x.shape[0]
        if pos0 + T > c.max_seq_len:
            raise ValueError("KV cache overflow")
        Hq, Hkv, Dh = c.num_q_heads, c.num_kv_heads, c.head_dim
        Qd, KVd, I = Hq * Dh, Hkv * Dh, c.intermediate_size
        cos, sin = self.cos[pos0:pos0 + T], self.sin[pos0:pos0 + T]
        scale = np.float32(1.0) / np.float32(np.sqrt(np.float32(Dh)))
        S = pos0 + T
        qpos = torch.arange(pos0, pos0 + T)[:, None]
        kpos = torch.arange(S)[None, :]
        mask = kpos <= qpos  # causal: row t attends [0, pos0+t]
        group = Hq // Hkv
        for li, L in enumerate(self.layers):
            n = rms_norm(x, L["input_layernorm"], c.rms_norm_eps)
            qkv = self._linear(n, L["qkv"])
            q = qkv[:, :Qd].reshape(T, Hq, Dh)
            k = qkv[:, Qd:Qd + KVd].reshape(T, Hkv, Dh)
            v = qkv[:, Qd + KVd:].reshape(T, Hkv, Dh)
            q = rms_norm(q, L["self_attn.q_norm"], c.rms_norm_eps)
            k = rms_norm(k, L["self_attn.k_norm"], c.rms_norm_eps)
            q = rope_half(q, cos, sin)
            k = rope_half(k, cos, sin)
            self.kc[li][pos0:S] = self._cast(k.reshape(T, KVd))
            self.vc[li][pos0:S] = self._cast(v.reshape(T, KVd))
            K = self.kc[li][:S].reshape(S, Hkv, Dh)
            V = self.vc[li][:S].reshape(S, Hkv, Dh)
            Kq = K.repeat_interleave(group, dim=1).permute(1, 2, 0)  # [Hq,Dh,S]
            Vq = V.repeat_interleave(group, dim=1).permute(1, 0, 2)  # [Hq,S,Dh]
            sc = torch.bmm(q.permute(1, 0, 2), Kq) * scale           # [Hq,T,S]
            sc = sc.masked_fill(~mask[None], float("-inf"))
            m = sc.amax(-1, keepdim=True)
            p = torch.exp(sc - m)
            inv = 1.0 / p.sum(-1, keepdim=True)
            att = (torch.bmm(p, Vq) * inv).permute(1, 0, 2).reshape(T, Qd)
            x = x + self._linear(att, L["self_attn.o_proj"])
            n = rms_norm(x, L["post_attention_layernorm"], c.rms_norm_eps)
            gu = self._linear(n, L["gateup"])
            g, u = gu[:, :I], gu[:, I:]
            s = (g / (1.0 + torch.exp(-g))) * u
            x = x + self._linear(s, L["mlp.down_proj"])
        self.cache_len = S
        last = rms_norm(x[-1:], self.final_norm, c.rms_norm_eps)
        self.logits = self._linear(last, self.embed)[0].numpy().copy()
        self.last_hidden = x.numpy()
        return self.logits

    def prefill_at(self, embeds, pos0: int):
        return self.forward(embeds, pos0)

    def decode_step(self, tok: int, pos: int):
        return self.forward(self.embed_row(tok)[None], pos)

    def argmax(self, ban0: int = -1, ban1: int = -1) -> int:
        return argmax_banned(self.logits, ban0, ban1)

    def decode_greedy(self, start_pos: int, max_new: int, eos0: int, eos1: int,
                      ban_steps: int = 3, batch: int = 32, record=None):
        """``DecodeGreedy`` (asr_text_decoder.cu:698-889): the argmax making
        token k is banned iff k < ban_steps; stop at EOS (excluded) or six equal
        tokens in a row, checked per batch; cache_len counts every run step."""
        tok = self.argmax(eos0 if ban_steps > 0 else -1, eos1 if ban_steps > 0 else -1)
        outp, out, pos, emitted = [], [], start_pos, 0

        def harvest(upto):
            for i in range(len(out), upto):
                t = outp[i]
                if t in (eos0, eos1):
                    return True
                out.append(t)
                if len(out) >= 6 and all(v == out[-1] for v in out[-6:]):
                    return True
            return False

        while emitted < max_new:
            nb = (emitted + 1) < ban_steps
            this_batch = 1 if nb else min(batch, max_new - emitted)
            for _ in range(this_batch):
                outp.append(tok)
                lg = self.decode_step(tok, pos)
                if record is not None:
                    record.append(lg.copy())
                k = len(outp)
                tok = self.argmax(*((eos0, eos1) if k < ban_steps else (-1, -1)))
                pos += 1
            emitted += this_batch
            if harvest(emitted):
                break
        self.cache_len = start_pos + emitted
        return out


def synthetic_weights(cfg: Config, seed: int, bf16: bool = True) -> dict:
    """The seeded synthetic checkpoint; ``bf16=False`` keeps the unrounded fp32
    values (the fp32 single-layer configuration)."""
    w = {}
    for name, tid, shape, is_norm in synth.model_tensors(
            seed, cfg.num_layers, cfg.vocab_size, cfg.hidden_size, cfg.num_q_heads,
            cfg.num_kv_heads, cfg.head_dim, cfg.intermediate_size):
        w[name] = synth.make_tensor(seed, tid, shape, is_norm, bf16=bf16)
    return w
