"""The batched speech detector (orx_vad_*, orator_b200/vad.py) on the GPU
against the CPU restatement (oracle/vad_oracle.py, itself pinned to the
reference's CPU detector) and against the reference's own GPU detector
(GpuVad from oracle/_ref, one stream at a time): per-window probabilities
within 1e-4 (fp32, summation order only), across chunk boundaries (LSTM state
and the 64-sample context carried), and the speech segments of the endpoint
state machine equal to GpuVad::DrainSegments on the same audio."""
import ctypes as C
import os

import numpy as np
import pytest

import refharness
from oracle import vad_oracle as V

pytestmark = pytest.mark.gpu
TOL = 1e-4


def pcm_for(S, steps):
    pcm = V.synthetic_pcm(4, S, steps * V.WINDOW)
    pcm[1::7] *= 0.01            # quiet streams
    pcm[2::7, :6000] = 0.0       # leading silence
    pcm[3::7, 9000:16000] = 0.0  # a pause in the middle
    return pcm


@pytest.fixture(scope="module")
def weights():
    return V.synthetic_weights(4)


def test_vs_oracle_with_chunks(cuda, weights):
    from orator_b200.vad import BatchVad
    S, steps = 64, 30
    pcm = pcm_for(S, steps)
    ref = V.BatchVadOracle(weights, S).run(pcm, steps)
    v = BatchVad(S)
    v.load(weights)
    a = v.run(pcm[:, :20 * V.WINDOW])
    b = v.run(pcm[:, 20 * V.WINDOW:])
    got = np.concatenate([a, b], 1)
    assert np.abs(got - ref).max() <= TOL, np.abs(got - ref).max()
    assert ref.min() < 0.5 < ref.max()
    v.reset()
    again = v.run(pcm)
    assert np.abs(again - ref).max() <= TOL
    v.close()


def test_synthetic_init_matches_oracle_weights(cuda, weights):
    from orator_b200.vad import BatchVad
    S, steps = 8, 6
    pcm = pcm_for(S, steps)
    v = BatchVad(S)
    v.init_synthetic(4)  # the GPU generator, bit-exact with oracle/synth.py
    got = v.run(pcm)
    ref = V.BatchVadOracle(weights, S).run(pcm, steps)
    assert np.abs(got - ref).max() <= TOL
    v.close()


def _ref_gpuvad(path):
    L = C.CDLL(refharness.LIB)
    L.ref_gpuvad_create.restype = C.c_void_p
    L.ref_gpuvad_create.argtypes = [C.c_char_p]
    L.ref_last_error.restype = C.c_char_p
    h = L.ref_gpuvad_create(path.encode())
    assert h, L.ref_last_error()
    return L, C.c_void_p(h)


def test_vs_reference_gpu_detector(cuda, weights, tmp_path):
    if not refharness.available():
        pytest.skip("reference build oracle/_ref not present")
    from orator_b200.vad import BatchVad, VadPool
    path = V.write_safetensors(str(tmp_path / "vad.safetensors"), weights)
    L, h = _ref_gpuvad(path)
    S, steps = 4, 40
    pcm = pcm_for(S, steps)
    v = BatchVad(S)
    v.load(weights)
    got = v.run(pcm)
    out = np.zeros(steps, np.float32)
    for s in range(S):
        n = L.ref_gpuvad_probs(h, pcm[s].ctypes.data_as(C.c_void_p), C.c_int(pcm.shape[1]),
                               out.ctypes.data_as(C.c_void_p))
        assert n == steps
        assert np.abs(out - got[s]).max() <= TOL, (s, np.abs(out - got[s]).max())
    # streaming segments: the same audio pushed in three pieces
    pool = VadPool(v)
    v.reset()
    cuts = [0, 7 * 512 + 100, 23 * 512, steps * 512]
    ours = [[] for _ in range(S)]
    for i in range(3):
        for s in range(S):
            pool.Push(s, pcm[s, cuts[i]:cuts[i + 1]])
        for s, segs in enumerate(pool.DrainSegments(finalize=(i == 2))):
            ours[s] += segs
    buf = (C.c_long * 64)()
    for s in range(S):
        L.ref_gpuvad_reset(h)
        theirs = []
        for i in range(3):
            piece = np.ascontiguousarray(pcm[s, cuts[i]:cuts[i + 1]])
            k = L.ref_gpuvad_push_drain(h, piece.ctypes.data_as(C.c_void_p), C.c_int(piece.size),
                                        C.c_int(i == 2), buf, 32)
            assert k >= 0
            theirs += [(buf[2 * j], buf[2 * j + 1]) for j in range(k)]
        assert ours[s] == theirs, (s, ours[s], theirs)
    L.ref_gpuvad_destroy(h)
    v.close()


def test_config5_shape_runs(cuda):
    torch = cuda
    from orator_b200.vad import BatchVad
    S, steps = 4096, 4
    v = BatchVad(S)
    v.init_synthetic(4)
    pcm = torch.rand(S, steps * 512, device="cuda") * 2 - 1
    probs = torch.empty(S, steps, device="cuda")
    v.run_device(pcm.data_ptr(), steps, probs.data_ptr())
    torch.cuda.synchronize()
    p = probs.cpu().numpy()
    assert np.isfinite(p).all() and (p > 0).all() and (p < 1).all()
    # spot-check a few streams against the restatement
    sel = [0, 1234, 4095]
    ref = V.BatchVadOracle(V.synthetic_weights(4), len(sel)).run(pcm[sel].cpu().numpy(), steps)
    assert np.abs(p[sel] - ref).max() <= TOL
    v.close()
