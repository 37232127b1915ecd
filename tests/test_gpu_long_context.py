"""Contexts past the persistent decode kernel's split table (max_seq_len >
4096 selects the per-kernel decode path: weight-streaming GEMV kernels and
flash-decoding attention replayed from CUDA graphs) and past the reference's
2048-position decode-attention cap: a 2-layer model prefilled with 2100 rows,
then teacher-forced decode steps and a greedy run, against the CPU oracle.
Bounds as in test_gpu_decoder.py (3e-2 max-abs, argmax equal where the
oracle's top-2 margin is at least 2e-2)."""
import numpy as np
import pytest

from oracle import decoder_oracle as D
from oracle import synth

pytestmark = pytest.mark.gpu

LAYERS, SEED, VOCAB = 2, 3, 151936
MAX_SEQ = 4400
TOL, MARGIN = 3e-2, 2e-2
T0 = 2100


def margin(lg):
    t = np.partition(lg, -2)[-2:]
    return float(t[1] - t[0])


def test_long_context_per_kernel_path(cuda):
    import torch
    from orator_b200 import AsrTextConfig, AsrTextDecoder
    cfg = D.Config(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=MAX_SEQ)
    o = D.OracleDecoder(cfg, D.synthetic_weights(cfg, SEED))
    dec = AsrTextDecoder(AsrTextConfig(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=MAX_SEQ))
    dec.init_synthetic(SEED)
    x = synth.audio_rows(SEED, T0, 2048)
    lo = o.prefill_at(x, 0)
    dec.Prefill(x)
    lg = dec.CopyLogits()
    assert np.abs(lg - lo).max() <= TOL
    tok = int(np.argmax(lo))
    d_tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    for s in range(6):
        ref = o.decode_step(tok, T0 + s)
        d_tok.fill_(tok)
        torch.cuda.synchronize()
        dec.DecodeStepDevice(d_tok.data_ptr(), T0 + s)
        got = dec.CopyLogits()
        assert np.abs(got - ref).max() <= TOL, s
        if margin(ref) >= MARGIN:
            assert int(np.argmax(got)) == int(np.argmax(ref)), s
        tok = int(np.argmax(ref))
    # greedy from the same prefix: tokens agree up to the oracle's first near tie
    dec.TruncateCache(T0)
    dec.Prefill(x)
    toks = dec.DecodeGreedy(T0, 8, -1, -1, ban_steps=0, batch=4)
    o.truncate(0)
    lg = o.prefill_at(x, 0)
    ref, pos = [], T0
    for _ in range(8):
        t = int(np.argmax(lg))
        if margin(lg) < MARGIN:
            break
        ref.append(t)
        lg = o.decode_step(t, pos)
        pos += 1
    assert list(toks[:len(ref)]) == ref
    assert dec.cache_len() == T0 + 8
    assert dec.device_error() == 0
    dec.close()
