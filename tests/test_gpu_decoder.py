"""GPU parity of the CUDA decoder path against the CPU oracle (and, when the
reference build in oracle/_ref is present, against the reference itself).

Model: the Qwen3-ASR-1.7B geometry with full vocabulary and 2 layers (the
28-layer case is covered against golden vectors made by the reference build).

Tolerances. Greedy argmax must equal the oracle's wherever the oracle's top-2
margin is >= 2e-2. Logits: the north_star asks 2e-2 max-abs in bf16, but the
reference build itself differs from this oracle by up to 1.4e-2 (prefill) and
2.4e-2 (16 teacher-forced decode steps) max-abs on 2-layer cases like these
(bf16 rounding flips of activations under a different fp32 summation order;
tests/test_gpu_reference.py measures both implementations side by side), so
the bound here is 3e-2: the reference's own deviation plus 25 %.
"""
import numpy as np
import pytest

from oracle import decoder_oracle as D
from oracle import synth

pytestmark = pytest.mark.gpu

LOGIT_TOL = 3e-2
DECODE_TOL = 3e-2
MARGIN = 2e-2
LAYERS = 2
SEED = 1
VOCAB = 151936


def margin(logits):
    t = np.partition(logits, -2)[-2:]
    return float(t[1] - t[0])


@pytest.fixture(scope="module")
def weights():
    cfg = D.Config(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=512)
    return cfg, D.synthetic_weights(cfg, SEED)


@pytest.fixture(scope="module")
def dec(cuda, weights):
    from orator_b200 import AsrTextConfig, AsrTextDecoder
    cfg, _ = weights
    d = AsrTextDecoder(AsrTextConfig(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=512))
    d.init_synthetic(SEED)
    assert d.weights_complete()
    yield d
    d.close()


def oracle(weights):
    cfg, w = weights
    return D.OracleDecoder(cfg, w)


def prompt(T, n_audio):
    audio = synth.audio_rows(SEED, n_audio, 2048)
    toks = synth.token_ids(SEED, T - n_audio, VOCAB)
    return audio, toks


def test_synth_bit_exact(cuda):
    import torch
    from orator_b200 import synth_f32
    for tid, std, mean, rb in [(0, 0.02, 0.0, True), (17, 0.02, 1.0, True), (60000, 1.0, 0.0, False)]:
        n = 100003
        buf = torch.empty(n, dtype=torch.float32, device="cuda")
        synth_f32(buf.data_ptr(), n, SEED, tid, std, mean, rb)
        torch.cuda.synchronize()
        ref = synth.normal_f32(SEED, tid, n, std, mean)
        if rb:
            ref = synth.bf16_round(ref)
        assert np.array_equal(buf.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_embed_matches_table(dec, weights):
    _, w = weights
    for tok in [0, 1, 12345, VOCAB - 1]:
        np.testing.assert_array_equal(dec.Embed(tok), w["thinker.model.embed_tokens.weight"][tok])


def test_prefill_logits(dec, weights):
    audio, toks = prompt(40, 30)
    emb = np.concatenate([audio, weights[1]["thinker.model.embed_tokens.weight"][toks]], 0)
    o = oracle(weights)
    ref = o.prefill_at(emb, 0)
    dec.ResetCache()
    dec.Prefill(emb)
    got = dec.CopyLogits()
    assert dec.cache_len() == 40
    err = np.abs(got - ref).max()
    assert err <= LOGIT_TOL, err
    if margin(ref) >= MARGIN:
        assert dec.Argmax() == int(np.argmax(ref))


@pytest.mark.parametrize("T", [1, 15, 16, 17, 33])
def test_prefill_page_boundaries(dec, weights, T):
    audio, _ = prompt(T, T)
    o = oracle(weights)
    ref = o.prefill_at(audio, 0)
    dec.ResetCache()
    dec.Prefill(audio)
    assert np.abs(dec.CopyLogits() - ref).max() <= LOGIT_TOL


def test_split_prefill_and_truncate(dec, weights):
    """Reference T010 (test/unit/model/test_asr_decoder.cc:76-127)."""
    audio, _ = prompt(50, 50)
    dec.ResetCache()
    dec.Prefill(audio)
    single = dec.CopyLogits()
    am = dec.Argmax()
    dec.ResetCache()
    dec.PrefillAt(audio[:25], None, 0)
    dec.PrefillAt(audio[25:], None, 25)
    assert dec.cache_len() == 50
    inc = dec.CopyLogits()
    assert np.abs(inc - single).max() <= LOGIT_TOL
    assert dec.Argmax() == am
    dec.TruncateCache(25)
    assert dec.cache_len() == 25
    dec.PrefillAt(audio[25:], None, 25)
    assert dec.Argmax() == am


def test_teacher_forced_decode(cuda, dec, weights):
    """DecodeStepDevice at successive positions vs the oracle, fed the same tokens."""
    import torch
    audio, toks = prompt(24, 20)
    emb = np.concatenate([audio, weights[1]["thinker.model.embed_tokens.weight"][toks]], 0)
    o = oracle(weights)
    o.prefill_at(emb, 0)
    dec.ResetCache()
    dec.Prefill(emb)
    d_tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    worst = 0.0
    tok = int(np.argmax(o.logits))
    for step in range(40):  # crosses the 32-position page boundary
        pos = 24 + step
        ref = o.decode_step(tok, pos)
        d_tok.fill_(tok)
        torch.cuda.synchronize()
        dec.DecodeStepDevice(d_tok.data_ptr(), pos)
        got = dec.CopyLogits()
        worst = max(worst, float(np.abs(got - ref).max()))
        if margin(ref) >= MARGIN:
            assert dec.Argmax() == int(np.argmax(ref)), step
        tok = int(np.argmax(ref))
    assert worst <= DECODE_TOL, worst
    assert dec.device_error() == 0


def test_decode_greedy_matches_oracle(dec, weights):
    audio, toks = prompt(30, 26)
    emb = np.concatenate([audio, weights[1]["thinker.model.embed_tokens.weight"][toks]], 0)
    o = oracle(weights)
    o.prefill_at(emb, 0)
    rec = []
    eos0, eos1 = 151645, 151643
    ref = o.decode_greedy(30, 24, eos0, eos1, ban_steps=3, batch=4, record=rec)
    dec.ResetCache()
    dec.Prefill(emb)
    got = dec.DecodeGreedy(30, 24, eos0, eos1, ban_steps=3, batch=4)
    # identical up to the first oracle step with a near tie
    n = len(ref)
    for i, lg in enumerate(rec):
        if margin(lg) < MARGIN:
            n = min(n, i + 1)
            break
    assert got[:n] == ref[:n]
    if n == len(ref):
        assert dec.cache_len() == o.cache_len


def test_argmax_ban(dec, weights):
    audio, _ = prompt(8, 8)
    dec.ResetCache()
    dec.Prefill(audio)
    lg = dec.CopyLogits()
    top = np.argsort(lg)[::-1]
    assert dec.Argmax() == top[0]
    assert dec.Argmax(int(top[0])) == top[1]
    assert dec.Argmax(int(top[0]), int(top[1])) == top[2]


def test_errors_are_raised(dec):
    from orator_b200 import OrxError
    with pytest.raises(OrxError):
        dec.PrefillAt(np.zeros((4, 2048), np.float32), None, 510)  # past max_seq_len
    with pytest.raises(OrxError):
        dec.TruncateCache(-1)
    with pytest.raises(OrxError):
        dec.Embed(VOCAB)
