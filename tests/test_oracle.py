"""Oracle pinning on CPU: the restatement against transformers' Qwen3 (fp32),
its quantization points, the argmax tie rule and the greedy control loop."""
import numpy as np
import pytest
import torch

from oracle import decoder_oracle as D
from oracle import synth


def test_synth_properties():
    v = synth.normal_f32(3, 5, 1 << 16, 0.02)
    assert abs(float(v.std()) - 0.02) < 5e-4 and abs(float(v.mean())) < 5e-4
    # deterministic and position-addressable
    a = synth.normal_f32(3, 5, 1000, 0.02)
    b = synth.normal_f32(3, 5, 2000, 0.02, chunk=333)
    assert np.array_equal(a, b[:1000])
    assert not np.array_equal(a, synth.normal_f32(4, 5, 1000, 0.02))


def test_bf16_rounding_matches_torch():
    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 3
    x[:4] = [1.00390625, 1.01171875, -2.5, 0.0]  # exact ties round to even
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(synth.f32_to_bf16_bits(x), ref)


def test_oracle_matches_transformers_fp32():
    pytest.importorskip("transformers")
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = D.Config(num_layers=2, vocab_size=4096, max_seq_len=64)
    w = D.synthetic_weights(cfg, 0)
    hc = Qwen3Config(hidden_size=2048, intermediate_size=6144, num_hidden_layers=2,
                     num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                     rms_norm_eps=1e-6, rope_theta=1e6, vocab_size=4096,
                     tie_word_embeddings=True, max_position_embeddings=4096)
    m = Qwen3ForCausalLM(hc).float().eval()
    sd = {k[len("thinker."):]: torch.from_numpy(v) for k, v in w.items()}
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    m.load_state_dict(sd, strict=False)
    x = synth.audio_rows(1, 20, 2048)
    o = D.OracleDecoder(cfg, w, quantize=False)
    o.forward(x[:12], 0)
    lg = o.forward(x[12:], 12)  # split prefill through the cache
    with torch.no_grad():
        ref = m(inputs_embeds=torch.from_numpy(x)[None]).logits[0, -1].numpy()
    assert np.abs(lg - ref).max() < 1e-4 * max(1.0, np.abs(ref).max())
    # with bf16 quantization points the logits move only at the bf16 noise floor
    oq = D.OracleDecoder(cfg, w, quantize=True)
    assert np.abs(oq.forward(x, 0) - ref).max() < 0.1


def test_oracle_decode_equals_prefill_rows():
    """A decode step is the T=1 case of the same forward (cu:360-455 vs 457-583)."""
    cfg = D.Config(num_layers=1, vocab_size=512, max_seq_len=32)
    w = D.synthetic_weights(cfg, 2)
    x = synth.audio_rows(2, 9, 2048)
    a = D.OracleDecoder(cfg, w)
    la = a.forward(x, 0)
    b = D.OracleDecoder(cfg, w)
    b.forward(x[:8], 0)
    lb = b.forward(x[8:], 8)
    assert np.abs(la - lb).max() < 2e-2  # fp32 summation order only


def test_argmax_tie_rule():
    x = np.zeros(1000, np.float32)
    x[300] = 5.0
    x[44] = 5.0  # both in thread slot 44: the first strict max in the slot wins
    assert D.argmax_banned(x) == 44
    y = np.zeros(1000, np.float32)
    y[260] = 2.0  # slot 4
    y[10] = 2.0   # slot 10
    assert D.argmax_banned(y) == 260  # lowest thread slot wins, not lowest id
    assert D.argmax_banned(y, 260) == 10
    assert D.argmax_banned(y, 260, 10) == 0
    z = np.full(300, -1e31, np.float32)  # nothing beats the -1e30 init
    assert D.argmax_banned(z) == 0


def _key_rule(x, ban0=-1, ban1=-1):
    """Closed form of the reference tie rule that the CUDA kernels pack into
    one 64-bit key (orator_b200/csrc/common.cuh argmax_key): among values
    > -1e30, the largest value, then the slot i % 256 with the smallest
    8-bit bit reversal, then the smallest i; nothing eligible -> 0."""
    best = None
    for i, v in enumerate(np.asarray(x, np.float32)):
        if i in (ban0, ban1) or not (v > np.float32(-1e30)):
            continue
        s = i & 255
        rev = int(f"{s:08b}"[::-1], 2)
        key = (float(v), -rev, -(i >> 8))
        if best is None or key > best[0]:
            best = (key, i)
    return 0 if best is None else best[1]


def test_argmax_key_closed_form_equals_tree():
    rng = np.random.default_rng(11)
    for trial in range(300):
        n = int(rng.integers(1, 3000))
        x = rng.integers(-3, 4, n).astype(np.float32)  # many exact ties
        if trial % 5 == 0:
            x[rng.integers(0, n, max(1, n // 7))] = np.nan
        if trial % 7 == 0:
            x[:] = -1e31
            x[rng.integers(0, n)] = np.float32(-1e30)
        if trial % 11 == 0:
            x = np.where(x == 0, np.float32(-0.0), x).astype(np.float32)
        b0 = int(rng.integers(-1, n)) if trial % 3 else -1
        b1 = int(rng.integers(-1, n)) if trial % 4 else -1
        assert _key_rule(x, b0, b1) == D.argmax_banned(x, b0, b1), trial


class _FakeDecoder(D.OracleDecoder):
    """Scripted logits: exercises DecodeGreedy's control loop only."""

    def __init__(self, script, vocab=16):
        self.script = list(script)
        self.vocab = vocab
        self.logits = self._onehot(self.script.pop(0))
        self.cache_len = 0
        self.calls = []

    def _onehot(self, t):
        v = np.zeros(self.vocab, np.float32)
        v[t] = 1.0
        v[(t + 1) % self.vocab] = 0.5  # runner-up used when t is banned
        return v

    def decode_step(self, tok, pos):
        self.calls.append((tok, pos))
        self.logits = self._onehot(self.script.pop(0) if self.script else 3)
        return self.logits


def test_greedy_stops_on_eos_and_bans_early():
    eos = 9
    f = _FakeDecoder([eos, eos, 4, eos, 7])
    out = f.decode_greedy(10, 8, eos, 15, ban_steps=3, batch=4)
    # tokens 0 and 1 are banned (k < 3): eos -> runner-up 10; token 2 = 4; token 3 = eos stops
    assert out == [10, 10, 4]
    assert [p for _, p in f.calls][:3] == [10, 11, 12]


def test_greedy_stops_on_six_repeats():
    f = _FakeDecoder([5] * 20)
    out = f.decode_greedy(0, 20, 14, 15, ban_steps=0, batch=4)
    assert out == [5] * 6
    assert f.cache_len == 8  # two batches of 4 ran
