"""Generate golden vectors from the REFERENCE decoder itself (oracle/_ref build).

Run on a GPU machine from the repository root, after oracle/build_ref.sh:
    PYTHONPATH=. python tests/golden/make_ref_golden.py OUT_DIR
It writes the seeded synthetic checkpoint (oracle/st_writer.py) to a temporary
directory, drives the unmodified reference AsrTextDecoder through
oracle/ref_harness.cc and stores, per case, the prompt recipe, the reference's
greedy tokens and its logits at sampled vocabulary indices.

Cases:
  l2   : 2 layers, prompt = 40 audio rows (seed 1), 16 greedy steps
  cfg2 : 28 layers (benchmark config 2): 375 audio rows + 25 prompt token ids
         (seed 1), greedy decode of 128 tokens (no stop rule: the reference is
         stepped with DecodeStepDevice + its own argmax)
"""
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle import synth, st_writer  # noqa: E402
from refharness import RefDecoder  # noqa: E402

VOCAB = 151936
N_FIXED = 224
N_TOP = 32


def fixed_indices():
    return np.sort(np.random.default_rng(12345).choice(VOCAB, N_FIXED, replace=False)).astype(np.int32)


def sample(logits, fixed):
    top = np.argsort(logits)[::-1][:N_TOP].astype(np.int32)
    idx = np.concatenate([top, fixed])
    return idx, logits[idx].astype(np.float32)


def prompt(case):
    if case == "l2":
        return synth.audio_rows(1, 40, 2048), np.zeros(0, np.int32)
    return synth.audio_rows(1, 375, 2048), synth.token_ids(1, 25, VOCAB)


def run(case, layers, steps, out_dir):
    fixed = fixed_indices()
    with tempfile.TemporaryDirectory() as d:
        st_writer.write_synthetic_model(d, 1, layers, VOCAB)
        ref = RefDecoder(d, layers, VOCAB, 2048)
        audio, toks = prompt(case)
        emb = synth.make_tensor(1, synth.TID_EMBED, (VOCAB, 2048), False)[toks] if len(toks) else \
            np.zeros((0, 2048), np.float32)
        x = np.concatenate([audio, emb], 0)
        T = x.shape[0]
        lg = ref.prefill_at(x, 0)
        idx, val = [], []
        i0, v0 = sample(lg, fixed)
        idx.append(i0); val.append(v0)
        tokens = [int(np.argmax(lg))]
        margins = [float(np.diff(np.sort(lg)[-2:])[0])]
        for s in range(steps):
            lg = ref.decode_step(tokens[-1], T + s)
            i1, v1 = sample(lg, fixed)
            idx.append(i1); val.append(v1)
            tokens.append(int(np.argmax(lg)))
            margins.append(float(np.diff(np.sort(lg)[-2:])[0]))
        ref.close()
    np.savez_compressed(os.path.join(out_dir, f"ref_{case}.npz"), layers=layers, seed=1,
                        prompt_rows=T, audio_rows=audio.shape[0], prompt_tokens=toks,
                        tokens=np.array(tokens, np.int32), margins=np.array(margins, np.float32),
                        idx=np.stack(idx), val=np.stack(val))
    print(case, "tokens", tokens[:12], "min margin", min(margins), flush=True)


if __name__ == "__main__":
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__))
    os.makedirs(out, exist_ok=True)
    run("l2", 2, 16, out)
    run("cfg2", 28, 128, out)
