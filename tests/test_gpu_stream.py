"""Streaming front door on the GPU: three sessions opened, fed audio rows and
decoded together through AsrStreamPool over the batched engine, against the
same protocol run per session on the CPU oracle (prefix prefill, audio rows
after the checkpoint, suffix prefill, DecodeGreedy with the EOS ban window,
truncate to the checkpoint), two rounds of audio. Tokens must agree up to the
oracle's first near tie (top-2 margin < 2e-2, 2-layer model)."""
import numpy as np
import pytest

from oracle import decoder_oracle as D
from oracle import synth

pytestmark = pytest.mark.gpu

LAYERS, SEED, VOCAB = 2, 5, 151936
MARGIN = 2e-2
MAX_NEW, BAN = 10, 3


def oracle_protocol(o, prefix, audio_chunks, suffix, eos):
    """Returns per round (tokens, margins) of the oracle run of the protocol."""
    o.reset()
    o.prefill_at(o.embed.numpy()[prefix], 0)
    ckpt = len(prefix)
    rounds = []
    for rows in audio_chunks:
        o.truncate(ckpt)
        o.prefill_at(rows, ckpt)
        ckpt += len(rows)
        lg = o.prefill_at(o.embed.numpy()[suffix], ckpt)
        pos = ckpt + len(suffix)
        toks, margins = [], []
        for k in range(MAX_NEW):
            l = lg.copy()
            if k < BAN:
                l[list(eos)] = -np.inf
            t = int(np.argmax(l))
            s = np.sort(l)
            margins.append(float(s[-1] - s[-2]))
            if t in eos:
                break
            toks.append(t)
            if len(toks) >= 6 and len(set(toks[-6:])) == 1:
                break
            lg = o.decode_step(t, pos)
            pos += 1
        rounds.append((toks, margins))
        o.truncate(ckpt)
    return rounds


def test_stream_pool_vs_oracle(cuda):
    from orator_b200 import AsrTextConfig, AsrTextDecoder, BatchDecoder
    from orator_b200 import stream as S
    cfg = D.Config(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=512)
    o = D.OracleDecoder(cfg, D.synthetic_weights(cfg, SEED))
    dec = AsrTextDecoder(AsrTextConfig(num_layers=LAYERS, vocab_size=VOCAB, max_seq_len=512))
    dec.init_synthetic(SEED)
    bd = BatchDecoder(dec, max_sessions=4, max_batch=4, pool_pages=96, max_pages_per_session=24)
    pool = S.AsrStreamPool(dec, bd, max_new=MAX_NEW, ban_steps=BAN)
    systems = [[1000 + i, 2000 + i] for i in range(3)]
    sids = [pool.open(sy) for sy in systems]
    chunks = [[synth.audio_rows(SEED + 10 * i + r, 13 + 4 * i + r, 2048) for r in range(2)]
              for i in range(3)]
    suffix_req = ([3000], [4000, 4001])
    got = {s: [] for s in sids}
    for r in range(2):
        pool.append_audio(sids, [chunks[i][r] for i in range(3)])
        out = pool.decode({s: suffix_req for s in sids})
        for s in sids:
            got[s].append(out[s])
            assert bd.cache_len(s) == pool.ckpt[s]
    assert bd.device_error() == 0
    eos = (S.IM_END, S.END_OF_TEXT)
    suffix = S.suffix_ids(*suffix_req)
    for i, s in enumerate(sids):
        ref = oracle_protocol(o, S.prefix_ids(systems[i]), chunks[i], suffix, eos)
        for r in range(2):
            toks, margins = ref[r]
            n = next((k for k, m in enumerate(margins) if m < MARGIN), len(margins))
            assert got[s][r][:n] == toks[:n], (i, r, got[s][r], toks, margins)
    bd.close()
    dec.close()
