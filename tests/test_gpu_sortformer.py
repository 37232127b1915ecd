"""The Sortformer network on B200 (orx_sf_*, orator_b200/sortformer.py)
against the CPU restatement (oracle/sortformer_oracle.py) and the reference's
own CUDA classes (oracle/_ref: ConformerPreEncode, ConformerLayer,
SortformerDecoder, assembled as ForwardEncoderDecoder) on the same seeded
weights and inputs.

Bars (fp32 model, the 1e-4 of fp32 parity): pre-encode rows within 1e-4 of
the row scale, relative (every Linear runs as three bf16 products of split
operands, about 2^-16 relative per product, against the reference's fp32
SGEMM; measured 2.6e-5); speaker probabilities within 1e-4 max-abs after the
whole stack (measured 1e-5 at 17 + 18 layers), identical zeros on padded
rows."""
import os
import tempfile

import numpy as np
import pytest

import refharness
from oracle import sortformer_oracle as SO

pytestmark = pytest.mark.gpu
LOG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpurun_out",
                   "sortformer_errors.txt")
CL, DL = 2, 2
PRED_TOL = 1e-4
EMB_TOL = 1e-4


def note(what, err):
    if os.path.isdir(os.path.dirname(LOG)):
        with open(LOG, "a") as f:
            f.write(f"{what}: {err:.3e}\n")


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def weights():
    return SO.synthetic_weights(CL, DL)


@pytest.fixture(scope="module")
def model(cuda, weights):
    from orator_b200.sortformer import Sortformer
    m = Sortformer(CL, DL)
    m.load(weights)
    assert m.weights_complete()
    yield m
    m.close()


@pytest.fixture(scope="module")
def ref(weights):
    if not refharness.available():
        pytest.skip("reference build (oracle/_ref) absent")
    d = tempfile.mkdtemp(prefix="orx_sf_")
    path = SO.write_safetensors(os.path.join(d, "sf.safetensors"), weights, CL, DL)
    r = refharness.RefSortformer(path, CL, DL)
    yield r
    r.close()


@pytest.mark.parametrize("n,valid", [(300, 300), (300, 250), (64, 40), (9, 9)])
def test_pre_encode(model, weights, ref, n, valid):
    mel = SO.synthetic_mel(3, n)
    got, v = model.pre_encode(mel, valid)
    want, T2, v2 = SO.SortformerOracle(weights, CL, DL).pre_encode(mel, valid)
    assert v == v2 and got.shape == want.shape
    note(f"pre_encode oracle n={n} valid={valid}", rel(got, want))
    assert rel(got, want) <= EMB_TOL
    r, rv = ref.pre_encode(mel, valid)
    assert rv == v
    note(f"pre_encode reference n={n} valid={valid}", rel(got, r))
    assert rel(got, r) <= EMB_TOL


@pytest.mark.parametrize("T,valid", [(90, 90), (90, 70), (33, 1), (200, 150)])
def test_encode_decode(model, weights, ref, T, valid):
    emb = SO.synth.normal_f32(3, 92000 + T, T * 512, 1.0).reshape(T, 512)
    got = model.forward(emb, valid)
    want = SO.SortformerOracle(weights, CL, DL).encode_decode(emb, valid)
    r = ref.encode_decode(emb, valid)
    note(f"encode_decode oracle T={T} valid={valid}", float(np.abs(got - want).max()))
    note(f"encode_decode reference T={T} valid={valid}", float(np.abs(got - r).max()))
    assert np.abs(got - want).max() <= PRED_TOL
    assert np.abs(got - r).max() <= PRED_TOL
    assert (got[valid:] == 0).all()
    assert want[:valid].min() < 0.5 < want[:valid].max() or valid < 4


def test_step_is_cache_plus_chunk(model, weights):
    mel = SO.synthetic_mel(4, 200)
    cache = SO.synth.normal_f32(4, 93000, 50 * 512, 1.0).reshape(50, 512)
    preds, v = model.step(mel, cache, valid=190)
    o = SO.SortformerOracle(weights, CL, DL)
    emb, T2, v2 = o.pre_encode(mel, 190)
    want = o.encode_decode(np.concatenate([cache, emb]), 50 + v2)
    assert v == 50 + v2 and preds.shape == want.shape
    assert np.abs(preds - want).max() <= PRED_TOL


def test_synthetic_init_matches_oracle_weights(cuda, weights):
    from orator_b200.sortformer import Sortformer
    m = Sortformer(CL, DL)
    m.init_synthetic(3)
    emb = SO.synth.normal_f32(3, 92090, 90 * 512, 1.0).reshape(90, 512)
    got = m.forward(emb, 80)
    want = SO.SortformerOracle(weights, CL, DL).encode_decode(emb, 80)
    assert np.abs(got - want).max() <= PRED_TOL
    m.close()


def test_full_size_step_vs_reference(cuda, tmp_path):
    """17 + 18 layers, weights from the GPU twin of the seeded generator; one
    config-4 step: 376 cache + FIFO rows and a 341-frame chunk (T = 717)."""
    if not refharness.available():
        pytest.skip("reference build (oracle/_ref) absent")
    import torch
    from orator_b200 import synth_f32
    from orator_b200.sortformer import Sortformer

    def gpu_normal(seed, tid, n, std, mean):
        buf = torch.empty(n, dtype=torch.float32, device="cuda")
        synth_f32(buf.data_ptr(), n, seed, tid, std, mean, False)
        return buf.cpu().numpy()

    w = SO.synthetic_weights(17, 18, normal=gpu_normal)
    path = SO.write_safetensors(str(tmp_path / "sf.safetensors"), w, 17, 18)
    del w
    m = Sortformer(17, 18)
    m.init_synthetic(3)
    m2 = Sortformer(17, 18)
    m2.load_safetensors(path)
    r = refharness.RefSortformer(path, 17, 18)
    try:
        mel = SO.synthetic_mel(5, 341 * 8)
        cache = SO.synth.normal_f32(5, 93001, 376 * 512, 1.0).reshape(376, 512)
        emb, v2 = r.pre_encode(mel, 341 * 8)
        want = r.encode_decode(np.concatenate([cache, emb]), 376 + v2)
        got, v = m.step(mel, cache)
        note("full step reference T=717", float(np.abs(got - want).max()))
        assert v == 376 + v2 == 717
        assert np.abs(got - want).max() <= PRED_TOL
        got2, _ = m2.step(mel, cache)
        assert np.array_equal(got, got2)
    finally:
        r.close()
        m.close()
        m2.close()


def test_oracle_pinned_to_reference(weights, ref):
    """The CPU restatement against the reference's own CUDA classes on the
    same weights and inputs: the oracle's pin."""
    o = SO.SortformerOracle(weights, CL, DL)
    mel = SO.synthetic_mel(6, 300)
    e_o, _, v_o = o.pre_encode(mel, 260)
    e_r, v_r = ref.pre_encode(mel, 260)
    assert v_o == v_r
    note("pre_encode oracle vs reference", rel(e_o, e_r))
    assert rel(e_o, e_r) <= EMB_TOL
    emb = SO.synth.normal_f32(6, 92500, 120 * 512, 1.0).reshape(120, 512)
    p_o, p_r = o.encode_decode(emb, 100), ref.encode_decode(emb, 100)
    note("encode_decode oracle vs reference", float(np.abs(p_o - p_r).max()))
    assert np.abs(p_o - p_r).max() <= PRED_TOL
