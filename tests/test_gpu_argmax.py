"""Every GPU argmax resolves exact ties as the reference's single-block
ArgmaxBannedKernel does (src/model/asr_ops.cu:300-325; restated step by step
in oracle/decoder_oracle.py argmax_banned): NaN and values <= -1e30 never
win, an input with nothing eligible gives 0, and equal maxima go by the
kernel's 256 thread slots and its reduction tree.

Two parts. (1) Planted logits, many exact ties: the scratch-free operator
(orx_argmax_banned), the allocation-free one (orx_argmax_banned_noalloc), the
decoder's multi-CTA argmax (orx_decoder_argmax over its logits buffer) and,
when oracle/_ref is present, the reference kernel itself. (2) The argmaxes
fused into the decode kernels (persistent decode kernel, per-kernel GEMV
lm_head, batched rows_argmax) on a model whose tied embedding table repeats
with period 300, so every logit has exact copies in other thread slots and
every greedy step is a tie: each emitted token must be the rule's pick
among the copies of its row."""
import ctypes as C
import os

import numpy as np
import pytest

import refharness
from oracle import decoder_oracle as D
from oracle import synth

pytestmark = pytest.mark.gpu

V = 151936


def _cudart():
    for name in ("libcudart.so", "libcudart.so.12"):
        try:
            return C.CDLL(name)
        except OSError:
            continue
    raise OSError("libcudart not found")


def tie_cases():
    rng = np.random.default_rng(7)
    cases = []
    x = np.zeros(V, np.float32)
    x[[10, 260, 300, 44, 4096 + 10]] = 5.0           # equal maxima in slots 10, 4, 44
    cases.append((x, -1, -1))
    cases.append((x, 260, -1))
    cases.append((x, 260, 10))
    y = np.full(V, -1e31, np.float32)                  # nothing beats -1e30
    cases.append((y, -1, -1))
    y2 = y.copy()
    y2[777] = np.float32(-1e30)                        # exactly -1e30 still loses
    y2[9] = np.nan
    cases.append((y2, -1, -1))
    z = np.zeros(V, np.float32)
    z[[128, 1, 129, 65]] = [-0.0, 0.0, 0.0, -0.0]      # signed zeros tie
    z[:] = np.where(z == 0, np.float32(-1.0), z)
    z[[128, 1, 129, 65]] = [-0.0, 0.0, 0.0, -0.0]
    cases.append((z, -1, -1))
    for t in range(12):                                # random small-integer logits
        w = rng.integers(-4, 5, V).astype(np.float32)
        if t % 3 == 0:
            w[rng.integers(0, V, 5000)] = np.nan
        b0 = int(np.argmax(w)) if t % 2 else -1
        cases.append((w, b0, int(rng.integers(0, V)) if t % 4 == 1 else -1))
    for n in (1, 255, 257, 70000):                     # short and ragged inputs
        w = rng.integers(0, 3, n).astype(np.float32)
        cases.append((w, -1, -1))
    return cases


def test_planted_ties_all_entry_points(cuda):
    torch = cuda
    from orator_b200 import AsrTextConfig, AsrTextDecoder, ops
    from orator_b200._lib import call
    rt = _cudart()
    dec = AsrTextDecoder(AsrTextConfig(num_layers=1, vocab_size=V, max_seq_len=32))
    dec.init_synthetic(1)
    lp = dec.logits_device_ptr()
    ref = refharness.RefOps() if refharness.available() else None
    out = torch.full((4,), -5, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream()
    for ci, (x, b0, b1) in enumerate(tie_cases()):
        want = D.argmax_banned(x, b0, b1)
        n = x.shape[0]
        dx = torch.from_numpy(x).cuda()
        ops.ArgmaxBanned(dx.data_ptr(), n, b0, b1, out.data_ptr(), s)
        call("orx_argmax_banned_noalloc", C.c_void_p(dx.data_ptr()), n, b0, b1,
             C.c_void_p(out.data_ptr() + 4), C.c_void_p(s.cuda_stream))
        if ref:
            ref.argmax_banned(dx.data_ptr(), n, b0, b1, out.data_ptr() + 8)
        torch.cuda.synchronize()
        got = out.tolist()
        assert got[0] == want and got[1] == want, (ci, got, want)
        if ref:
            assert got[2] == want, (ci, "reference build disagrees with the oracle", got[2], want)
        if n == V:  # the decoder's own argmax over its logits buffer
            host = np.ascontiguousarray(x)
            assert rt.cudaMemcpy(C.c_void_p(lp), host.ctypes.data_as(C.c_void_p),
                                 C.c_size_t(host.nbytes), 1) == 0
            assert dec.Argmax(b0, b1) == want, ci
    dec.close()


PERIOD = 300


def pick(tok, vocab, ban0=-1, ban1=-1):
    """The reference rule's choice among the exact copies of token tok's row."""
    onehot = np.zeros(vocab, np.float32)
    onehot[np.arange(tok % PERIOD, vocab, PERIOD)] = 1.0
    return D.argmax_banned(onehot, ban0, ban1)


def periodic_decoder(vocab, layers, no_mk=False, max_seq=256):
    from orator_b200 import AsrTextConfig, AsrTextDecoder
    cfg = D.Config(num_layers=layers, vocab_size=vocab, max_seq_len=max_seq)
    w = D.synthetic_weights(cfg, 5)
    e = w["thinker.model.embed_tokens.weight"]
    e = e[np.arange(vocab) % PERIOD]
    old = os.environ.get("ORX_NO_MK")
    if no_mk:
        os.environ["ORX_NO_MK"] = "1"
    try:
        dec = AsrTextDecoder(AsrTextConfig(num_layers=layers, vocab_size=vocab, max_seq_len=max_seq))
    finally:
        if no_mk:
            if old is None:
                del os.environ["ORX_NO_MK"]
            else:
                os.environ["ORX_NO_MK"] = old
    dec.init_synthetic(5)
    bits = (np.ascontiguousarray(e, np.float32).view(np.uint32) >> 16).astype(np.uint16)  # exact: e is bf16
    dec.set_tensor("thinker.model.embed_tokens.weight", bits)
    return dec


@pytest.mark.parametrize("no_mk", [False, True])
def test_fused_decode_argmax_ties(cuda, no_mk):
    vocab = 4096
    dec = periodic_decoder(vocab, 2, no_mk)
    x = synth.audio_rows(9, 10, 2048)
    dec.Prefill(x)
    toks = dec.DecodeGreedy(10, 24, -1, -1, ban_steps=0, batch=8)
    assert len(toks) >= 2, toks  # the six-repeat rule may stop early
    for k, t in enumerate(toks):
        assert t == pick(t, vocab), (no_mk, k, t, toks)
    # banned window: the first argmaxes exclude the ids the rule would pick
    dec.ResetCache()
    dec.Prefill(x)
    b0 = pick(toks[0], vocab)
    toks2 = dec.DecodeGreedy(10, 4, b0, -1, ban_steps=2, batch=1)
    assert toks2[0] == pick(toks2[0], vocab, b0, -1) and toks2[0] != b0
    assert dec.device_error() == 0
    dec.close()


def test_batched_argmax_ties(cuda):
    from orator_b200 import BatchDecoder
    vocab = 4096
    dec = periodic_decoder(vocab, 2)
    bd = BatchDecoder(dec, max_sessions=4, max_batch=4, pool_pages=32, max_pages_per_session=8)
    sids = [bd.create_session() for _ in range(3)]
    bd.prefill(sids, [synth.audio_rows(20 + i, 5 + 3 * i, 2048) for i in range(3)])
    first = bd.next_tokens(sids)
    for t in first:
        assert t == pick(int(t), vocab)
    for _ in range(10):
        for t in bd.step(sids):
            assert t == pick(int(t), vocab), t
    assert bd.device_error() == 0
    bd.close()
    dec.close()
