"""fp32 single decoder layer on the GPU vs the fp32 oracle (no bf16 rounding).

The correctness configuration of the decoder: one Qwen3-1.7B-shaped layer,
fp32 weights N(0, 0.02) from the seeded generator (seed 0, unrounded), a KV
cache of 512 past positions produced by the layer itself from 512 hidden rows
N(0, 1) at positions 0..511, then one query row N(0, 1) at position 512.

Tolerance (fp32): max |gpu - oracle| <= 1e-4 * max |oracle| over every output
row, for the 512 cache-building rows and for the query.
"""
import numpy as np
import pytest

from oracle import decoder_oracle as D
from oracle import synth

pytestmark = pytest.mark.gpu

SEED, PAST = 0, 512
REL = 1e-4


@pytest.fixture(scope="module")
def pair(cuda):
    from orator_b200 import AsrTextConfig, Layer32
    cfg = D.Config(num_layers=1, vocab_size=16, max_seq_len=PAST + 64)
    orc = D.OracleDecoder(cfg, D.synthetic_weights(cfg, SEED, bf16=False), quantize=False)
    lay = Layer32(AsrTextConfig(num_layers=1, max_seq_len=PAST + 64))
    lay.init_synthetic(SEED, 0)
    yield orc, lay
    lay.close()


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def test_config1_layer(pair):
    orc, lay = pair
    past = synth.audio_rows(SEED + 100, PAST, 2048)
    query = synth.audio_rows(SEED + 101, 1, 2048)
    orc.forward(past, 0)
    ref_past = orc.last_hidden.copy()
    orc.forward(query, PAST)
    ref_q = orc.last_hidden.copy()
    got_past = lay.forward(past, 0)
    got_q = lay.forward(query, PAST)
    assert lay.cache_len() == PAST + 1
    assert rel_err(got_past, ref_past) <= REL, rel_err(got_past, ref_past)
    assert rel_err(got_q, ref_q) <= REL, rel_err(got_q, ref_q)


def test_truncate_and_replay(pair):
    """Truncating back to the 512 past rows and replaying the query gives the
    same output bit for bit (the cache rows before the cut are untouched)."""
    _, lay = pair
    past = synth.audio_rows(SEED + 100, PAST, 2048)
    query = synth.audio_rows(SEED + 101, 1, 2048)
    lay.truncate(0)
    lay.forward(past, 0)
    a = lay.forward(query, PAST)
    lay.truncate(PAST)
    b = lay.forward(query, PAST)
    assert np.array_equal(a, b)


def test_loaded_weights_match_generator(pair, cuda):
    """set_tensor with the oracle's fp32 arrays equals init_synthetic."""
    from orator_b200 import AsrTextConfig, Layer32
    cfg = D.Config(num_layers=1, vocab_size=16, max_seq_len=64)
    w = D.synthetic_weights(cfg, SEED, bf16=False)
    lay = Layer32(AsrTextConfig(num_layers=1, max_seq_len=64))
    for nm in synth.LAYER_TENSORS:
        lay.set_tensor(nm, w[f"thinker.model.layers.0.{nm}.weight"])
    other = Layer32(AsrTextConfig(num_layers=1, max_seq_len=64))
    other.init_synthetic(SEED, 0)
    x = synth.audio_rows(SEED + 7, 5, 2048)
    assert np.array_equal(lay.forward(x, 0), other.forward(x, 0))
    lay.close()
    other.close()


def test_errors(pair):
    from orator_b200 import OrxError
    _, lay = pair
    with pytest.raises(OrxError):
        lay.forward(np.zeros((1, 2048), np.float32), lay.cache_len() + 1)  # gap in the cache
    with pytest.raises(OrxError):
        lay.set_tensor("mlp.nope", np.zeros(4, np.float32))
