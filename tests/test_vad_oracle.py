"""The CPU restatement of the Silero-shaped detector (oracle/vad_oracle.py)
against the reference's own CPU detector (AsrSileroVad,
test/utils/asr_vad_cpu.cc, built from its sources by oracle/build_ref.sh into
oracle/_ref/libref_vad_cpu.so) on the same synthetic weights file and PCM:
per-window speech probabilities of several streams, 24 windows each, within
2e-5 (fp32 summation order only). Also the endpoint state machine on
scripted probabilities."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import vad_oracle as V

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref_vad_cpu.so")


@pytest.mark.skipif(not os.path.exists(LIB), reason="oracle/_ref/libref_vad_cpu.so not built")
def test_oracle_matches_reference_cpu_detector(tmp_path):
    w = V.synthetic_weights(4)
    path = V.write_safetensors(str(tmp_path / "vad.safetensors"), w)
    L = C.CDLL(LIB)
    L.ref_vadcpu_create.restype = C.c_void_p
    L.ref_vadcpu_create.argtypes = [C.c_char_p]
    L.ref_vadcpu_last_error.restype = C.c_char_p
    h = L.ref_vadcpu_create(path.encode())
    assert h, L.ref_vadcpu_last_error()
    h = C.c_void_p(h)
    S, steps = 6, 24
    pcm = V.synthetic_pcm(4, S, steps * V.WINDOW)
    pcm[1] *= 0.01           # a quiet stream
    pcm[2, :4000] = 0.0      # leading silence
    ours = V.BatchVadOracle(w, S).run(pcm, steps)
    out = np.zeros(steps, np.float32)
    for s in range(S):
        n = L.ref_vadcpu_probs(h, pcm[s].ctypes.data_as(C.c_void_p), C.c_int(pcm.shape[1]),
                               out.ctypes.data_as(C.c_void_p))
        assert n == steps
        assert np.abs(out - ours[s]).max() <= 2e-5, (s, np.abs(out - ours[s]).max())
    L.ref_vadcpu_destroy(h)
    # the synthetic model is not degenerate: probabilities on both sides of 0.5
    assert ours.min() < 0.5 < ours.max(), (ours.min(), ours.max())


def test_endpoint_state_machine():
    e = V.Endpoint()             # 16 kHz: min speech 4000 samples, min silence 1920, pad 960
    # 8 speech windows (4096 samples, onset after the 8th), 4 silence (2048 >= 1920 -> end)
    segs = e.push([0.9] * 8 + [0.1] * 4 + [0.2] * 4)
    assert segs == [(0 - 0 if False else 0, 8 * 512 + 960)] or segs == [(0, 8 * 512 + 960)]
    assert not e.in_speech
    # speech that never confirms (3 windows < 4000 samples) makes no segment
    assert e.push([0.9] * 3 + [0.1] * 5) == []
    # an open segment is flushed by finalize, clipped to the processed horizon
    e2 = V.Endpoint()
    e2.push([0.9] * 10)
    assert e2.in_speech
    assert e2.push([], finalize=True) == [(0, 10 * 512)]
