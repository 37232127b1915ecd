"""Benchmark config 2 on the GPU: the full 28-layer decoder against golden
vectors produced by the reference build itself (tests/golden/ref_cfg2.npz).

* teacher-forced: every one of the 128 steps is fed the reference's token;
  sampled logits (reference top-32 + 224 fixed ids) within TOL_DECODE and
  argmax equal wherever the reference's top-2 margin is >= MARGIN;
* free-running DecodeGreedy: the token sequence equals the reference's up to
  its first step with a top-2 margin below MARGIN (after such a near tie two
  correct bf16 implementations may legitimately diverge).

TOL_DECODE: the reference differs from the CPU oracle by up to 9.3e-2 max-abs
over decode steps at 28 layers; this build must agree with the reference to
the same order.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_cfg2.npz")
TOL_PREFILL = 0.08
TOL_DECODE = 0.15
MARGIN = 0.1


@pytest.fixture(scope="module")
def setup(cuda):
    from orator_b200 import AsrTextConfig, AsrTextDecoder, synth_f32
    torch = cuda
    z = np.load(GOLD)
    dec = AsrTextDecoder(AsrTextConfig(max_seq_len=2048))
    dec.init_synthetic(int(z["seed"]))
    na = int(z["audio_rows"])
    buf = torch.empty(na * 2048, dtype=torch.float32, device="cuda")
    synth_f32(buf.data_ptr(), buf.numel(), int(z["seed"]), 60000, 1.0)
    torch.cuda.synchronize()
    audio = buf.cpu().numpy().reshape(na, 2048)
    emb = np.stack([dec.Embed(int(t)) for t in z["prompt_tokens"]])
    x = np.concatenate([audio, emb], 0)
    yield dec, z, x
    dec.close()


def cmp(z, step, lg):
    idx, val = z["idx"][step], z["val"][step]
    return float(np.abs(lg[idx] - val).max())


def test_teacher_forced_128_steps(setup, cuda):
    torch = cuda
    dec, z, x = setup
    T = int(z["prompt_rows"])
    dec.ResetCache()
    dec.Prefill(x)
    lg = dec.CopyLogits()
    assert cmp(z, 0, lg) <= TOL_PREFILL, cmp(z, 0, lg)
    toks, margins = z["tokens"], z["margins"]
    d_tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    worst, mism = 0.0, []
    for s in range(len(toks) - 1):
        d_tok.fill_(int(toks[s]))
        torch.cuda.synchronize()
        dec.DecodeStepDevice(d_tok.data_ptr(), T + s)
        lg = dec.CopyLogits()
        worst = max(worst, cmp(z, s + 1, lg))
        if margins[s + 1] >= MARGIN and int(np.argmax(lg)) != int(toks[s + 1]):
            mism.append(s + 1)
    print(f"config2 teacher-forced: worst sampled-logit deviation {worst:.4f}")
    assert not mism, mism
    assert worst <= TOL_DECODE, worst
    assert dec.device_error() == 0


def test_free_running_greedy(setup):
    dec, z, x = setup
    T = int(z["prompt_rows"])
    dec.ResetCache()
    dec.Prefill(x)
    out = dec.DecodeGreedy(T, 128, -1, -1, ban_steps=0, batch=32)
    assert len(out) == 128 and dec.cache_len() == T + 128
    toks, margins = z["tokens"], z["margins"]
    n = next((i for i, m in enumerate(margins) if m < MARGIN), len(margins))
    same = next((i for i, (a, b) in enumerate(zip(out, toks)) if a != b), min(len(out), len(toks)))
    print(f"config2 greedy: {same} leading tokens identical to the reference (first near tie at {n})")
    assert out[:n] == [int(t) for t in toks[:n]]
