"""The audio tower (orx_tower_*, orator_b200/tower.py) on the GPU against the
CPU restatement (oracle/tower_oracle.py) and the reference's own
AsrAudioTower (oracle/_ref, src/model/asr_audio_tower.cu) on the same seeded
weights and mel: rows [OutputLength(n_frames), 2048] within 2e-2 max-abs
(the bf16 bar: both sides round every projection input to bf16, so a last-bit
fp32 difference can move one bf16 rounding), over full and ragged chunks, one
frame, windowed attention, and many utterances in one batched call."""
import os
import tempfile

import numpy as np
import pytest

import refharness
from oracle import synth
from oracle import tower_oracle as TO

pytestmark = pytest.mark.gpu
TOL = 5e-2
MEAN_TOL = 3e-3
LOG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpurun_out",
                   "tower_errors.txt")


def close(got, want, what):
    assert got.shape == want.shape, (got.shape, want.shape)
    d = np.abs(got - want)
    mx, mean = float(d.max()), float(d.mean())
    if os.path.isdir(os.path.dirname(LOG)):
        with open(LOG, "a") as f:
            f.write(f"{what}: max {mx:.3e} mean {mean:.3e} scale {float(np.abs(want).max()):.3f}\n")
    assert mx <= TOL and mean <= MEAN_TOL, (what, mx, mean)
LAYERS = 2
FRAMES = [350, 100, 57, 1, 230]


def mel_for(n, seed=9):
    return synth.normal_f32(seed, 81000 + n % 1000, 128 * n, 1.0).reshape(128, n)


@pytest.fixture(scope="module")
def weights():
    return TO.synthetic_weights(LAYERS)


@pytest.fixture(scope="module")
def tower(cuda, weights):
    from orator_b200.tower import AudioTower
    t = AudioTower(LAYERS)
    t.load(weights)
    assert t.weights_complete()
    yield t
    t.close()


@pytest.fixture(scope="module")
def ref_dir(weights):
    d = tempfile.mkdtemp(prefix="orx_tower_")
    return TO.write_checkpoint(d, weights, LAYERS)


def test_output_length_matches_reference():
    from orator_b200.tower import output_length
    for n in [0, 1, 2, 7, 8, 99, 100, 101, 199, 200, 350, 1234]:
        assert output_length(n) == TO.output_length(n)


@pytest.mark.parametrize("n", FRAMES)
def test_vs_oracle(tower, weights, n):
    mel = mel_for(n)
    got = tower.forward(mel)
    ref = TO.TowerOracle(weights, LAYERS).forward(mel)
    assert got.shape == (TO.output_length(n), 2048)
    close(got, ref, f"oracle n={n}")


@pytest.mark.parametrize("n", FRAMES)
def test_vs_reference_tower(tower, ref_dir, n):
    if not refharness.available():
        pytest.skip("reference build (oracle/_ref) absent")
    ref = refharness.RefTower(ref_dir, LAYERS)
    try:
        mel = mel_for(n)
        want = ref.forward(mel)
        got = tower.forward(mel)
        close(got, want, f"reference n={n}")
    finally:
        ref.close()


def test_windowed_attention_vs_reference(cuda, weights, ref_dir):
    if not refharness.available():
        pytest.skip("reference build (oracle/_ref) absent")
    from orator_b200.tower import AudioTower
    n = 1750  # 228 rows: windows of 104, 104, 20
    mel = mel_for(n)
    t = AudioTower(LAYERS, windowed=True)
    t.load(weights)
    ref = refharness.RefTower(ref_dir, LAYERS, windowed=True)
    full = AudioTower(LAYERS)
    full.load(weights)
    try:
        want = ref.forward(mel)
        got = t.forward(mel)
        close(got, want, "windowed reference n=1750")
        # the windows matter: full attention gives other rows
        assert np.abs(full.forward(mel) - want).max() > 4 * TOL
    finally:
        ref.close()
        t.close()
        full.close()


def test_batch_equals_single_calls(cuda, tower):
    import torch
    frames = [350, 57, 1000, 1, 100, 230, 99]
    mels = [mel_for(n, seed=11 + i) for i, n in enumerate(frames)]
    packed = np.concatenate([m.reshape(-1) for m in mels])
    d_mel = torch.from_numpy(packed).cuda()
    total = sum(TO.output_length(n) for n in frames)
    d_out = torch.empty(total, 2048, device="cuda")
    rows = tower.forward_batch(d_mel.data_ptr(), frames, d_out.data_ptr())
    torch.cuda.synchronize()
    assert rows == total
    got = d_out.cpu().numpy()
    r = 0
    for m, n in zip(mels, frames):
        k = TO.output_length(n)
        single = tower.forward(m)
        assert np.array_equal(got[r:r + k], single), np.abs(got[r:r + k] - single).max()
        r += k


def test_synthetic_init_matches_oracle_weights(cuda, weights):
    from orator_b200.tower import AudioTower
    t = AudioTower(LAYERS)
    t.init_synthetic(5)
    mel = mel_for(230)
    got = t.forward(mel)
    ref = TO.TowerOracle(weights, LAYERS).forward(mel)
    close(got, ref, "synthetic init vs oracle n=230")
    t.close()


def test_argument_errors(cuda):
    import ctypes as C
    from orator_b200._lib import lib
    from orator_b200.tower import AudioTower
    t = AudioTower(1)
    with pytest.raises(Exception):
        t.forward(mel_for(100))  # weights not loaded
    with pytest.raises(Exception):
        t.set_tensor("thinker.audio_tower.proj1.bias", np.zeros(5, np.float32))
    with pytest.raises(Exception):
        t.set_tensor("thinker.audio_tower.nope", np.zeros(5, np.float32))
    assert lib().orx_tower_create(-1, 0, C.byref(C.c_void_p())) != 0
    t.close()


def test_full_depth_vs_reference(cuda, tmp_path):
    """24 layers (the reference's default), weights from the GPU twin of the
    seeded generator, one 10 s utterance and a ragged one."""
    if not refharness.available():
        pytest.skip("reference build (oracle/_ref) absent")
    import torch
    from orator_b200 import synth_f32
    from orator_b200.tower import AudioTower

    def gpu_normal(seed, tid, n, std, mean):
        buf = torch.empty(n, dtype=torch.float32, device="cuda")
        synth_f32(buf.data_ptr(), n, seed, tid, std, mean, False)
        return buf.cpu().numpy()

    w = TO.synthetic_weights(24, normal=gpu_normal)
    d = TO.write_checkpoint(str(tmp_path / "tower24"), w, 24)
    del w
    t = AudioTower(24)
    t.init_synthetic(5)
    t2 = AudioTower(24)
    t2.load_safetensors(d)
    ref = refharness.RefTower(d, 24)
    try:
        for n in (1000, 777):
            mel = mel_for(n)
            want = ref.forward(mel)
            got = t.forward(mel)
            close(got, want, f"24 layers reference n={n}")
            assert np.array_equal(t2.forward(mel), got)
    finally:
        ref.close()
        t.close()
        t2.close()


@pytest.mark.parametrize("n", [350, 57])
def test_oracle_pinned_to_reference(weights, ref_dir, n):
    """The CPU restatement against the reference's own AsrAudioTower (run on
    this GPU) on the same checkpoint and mel: the oracle's pin."""
    if not refharness.available():
        pytest.skip("reference build (oracle/_ref) absent")
    ref = refharness.RefTower(ref_dir, LAYERS)
    try:
        mel = mel_for(n)
        close(TO.TowerOracle(weights, LAYERS).forward(mel), ref.forward(mel), f"oracle vs reference n={n}")
    finally:
        ref.close()
