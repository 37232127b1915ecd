"""Continuous batching on the GPU: ragged sessions joining and leaving, each
session's greedy tokens checked against an independent oracle run of that
session alone (2-layer model, full vocabulary)."""
import numpy as np
import pytest

from oracle import decoder_oracle as D
from oracle import synth

pytestmark = pytest.mark.gpu

LAYERS, SEED, VOCAB = 2, 4, 151936
MARGIN = 2e-2


@pytest.fixture(scope="module")
def env(cuda):
    from orator_b200 import AsrTextConfig, AsrTextDecoder, BatchDecoder
    cfg = D.Config(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=256)
    w = D.synthetic_weights(cfg, SEED)
    dec = AsrTextDecoder(AsrTextConfig(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=256))
    dec.init_synthetic(SEED)
    bd = BatchDecoder(dec, max_sessions=8, max_batch=8, pool_pages=64, max_pages_per_session=16)
    yield cfg, w, dec, bd
    bd.close()
    dec.close()


def oracle_greedy(cfg, w, x, steps):
    """Greedy tokens of one session alone, with each step's top-2 margin."""
    o = D.OracleDecoder(cfg, w)
    lg = o.prefill_at(x, 0)
    toks, margins = [], []
    pos = x.shape[0]
    for _ in range(steps):
        t = int(np.argmax(lg))
        srt = np.sort(lg)
        toks.append(t)
        margins.append(float(srt[-1] - srt[-2]))
        lg = o.decode_step(t, pos)
        pos += 1
    return toks, margins


def agree(got, ref, margins):
    n = next((i for i, m in enumerate(margins) if m < MARGIN), len(margins))
    return got[:n] == ref[:n]  # identical up to the first near tie


def test_ragged_join_leave(env):
    cfg, w, dec, bd = env
    lens = [5, 17, 33, 16, 1]
    xs = [synth.audio_rows(SEED + 10 + i, L, 2048) for i, L in enumerate(lens)]
    sids = [bd.create_session() for _ in lens]
    # first decoded token of each session = argmax after its prefill
    bd.prefill(sids[:3], xs[:3])
    out = {s: [] for s in sids}
    active = list(sids[:3])
    for step in range(12):
        if step == 4:  # two sessions join mid-stream, batched in one prefill
            bd.prefill(sids[3:], xs[3:])
            active += sids[3:]
        if step == 8:  # one leaves
            bd.free_session(sids[1])
            active.remove(sids[1])
        toks = bd.step(active)
        for s, t in zip(active, toks):
            out[s].append(int(t))
    assert bd.device_error() == 0
    # The batch emits, per step, the token FOLLOWING the session's current one.
    # Oracle: greedy tokens t0 (after prefill), t1, ...; the batch's step k for
    # a session returns t_{k+1}.
    for i, s in enumerate(sids):
        n = len(out[s])
        ref, margins = oracle_greedy(cfg, w, xs[i], n + 1)
        assert agree(out[s], ref[1:], margins[1:]), (i, out[s], ref[1:])
    assert bd.cache_len(sids[0]) == lens[0] + 12


def test_pool_exhaustion_rejects_join(env):
    from orator_b200 import OrxError
    cfg, w, dec, bd = env
    free0 = bd.free_pages()
    sid = bd.create_session()
    big = synth.audio_rows(SEED, 16 * (free0 + 1), 2048)  # one page more than the pool has
    with pytest.raises(OrxError):
        bd.prefill([sid], [big])
    assert bd.free_pages() == free0 and bd.cache_len(sid) == 0
    bd.free_session(sid)


def test_truncate_returns_pages(env):
    cfg, w, dec, bd = env
    sid = bd.create_session()
    free0 = bd.free_pages()
    bd.prefill([sid], [synth.audio_rows(SEED, 40, 2048)])
    assert bd.free_pages() == free0 - 3
    bd.truncate(sid, 16)
    assert bd.free_pages() == free0 - 1 and bd.cache_len(sid) == 16
    bd.free_session(sid)
    assert bd.free_pages() == free0


def test_batch_sizes_return_to_earlier_sizes(env):
    """Regression for replaying a per-batch-size step graph after its buffers
    changed: batch sizes go 3 -> 8 -> 3 -> 5 -> 8 -> 1 with a 100-row join in
    between (which grows the prefill buffers and workspace), and every
    session's tokens still match the oracle run of that session alone."""
    from orator_b200 import BatchDecoder
    cfg, w, dec, _ = env
    bd = BatchDecoder(dec, max_sessions=9, max_batch=8, pool_pages=96, max_pages_per_session=12)
    try:
        lens = [3, 9, 20, 4, 7, 15, 2, 11, 100]
        xs = [synth.audio_rows(SEED + 40 + i, L, 2048) for i, L in enumerate(lens)]
        sids = [bd.create_session() for _ in lens]
        out = {s: [] for s in sids}

        def run(active, times):
            for _ in range(times):
                toks = bd.step(active)
                for s, t in zip(active, toks):
                    out[s].append(int(t))

        bd.prefill(sids[:3], xs[:3])
        run(sids[:3], 2)            # 3
        bd.prefill(sids[3:8], xs[3:8])
        run(sids[:8], 2)            # 8
        run(sids[:3], 2)            # back to 3
        bd.prefill([sids[8]], [xs[8]])  # a long join grows the prefill side
        run(sids[3:8], 2)           # 5
        run(sids[:8], 1)            # 8 again
        run([sids[8]], 3)           # 1
        run(sids[:3], 1)            # 3 again
        assert bd.device_error() == 0
        for i, s in enumerate(sids):
            n = len(out[s])
            ref, margins = oracle_greedy(cfg, w, xs[i], n + 1)
            assert agree(out[s], ref[1:], margins[1:]), (i, out[s], ref[1:])
            assert bd.cache_len(s) == lens[i] + n
    finally:
        bd.close()
