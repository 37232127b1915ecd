"""The Sortformer restatement (oracle/sortformer_oracle.py) on CPU: the
rel_shift gather it uses equals the reference's flat-index rel_shift
(RelShiftScoresKernel, src/model/conformer_layer.cu:121-145), the pre-encode
lengths follow ConvOutLen, and a small model gives finite probabilities with
the padded rows zeroed."""
import numpy as np
import torch

from oracle import sortformer_oracle as SO


def test_rel_shift_matches_reference_index_formula():
    T = 7
    P = 2 * T - 1
    bd_full = torch.randn(P, T).t().contiguous()  # [T, P] for one head
    ii = torch.arange(T)[:, None]
    jj = torch.arange(T)[None, :]
    ours = bd_full[ii, T - 1 - ii + jj]
    ref = torch.empty(T, T)
    for i in range(T):
        for j in range(T):
            idx = T + i * P + j
            ip, c2 = idx // (2 * T), idx % (2 * T)
            ref[i, j] = 0.0 if c2 == 0 else bd_full[ip, c2 - 1]
    assert torch.equal(ours, ref)


def test_pos_emb_rows():
    pe = SO.pos_emb(5)
    assert pe.shape == (9, SO.D)
    # row idx sits at position T - 1 - idx: the middle row is position 0
    assert torch.allclose(pe[4, 0::2], torch.zeros(SO.D // 2))
    assert torch.allclose(pe[4, 1::2], torch.ones(SO.D // 2))


def test_small_model_runs():
    w = SO.synthetic_weights(1, 1)
    o = SO.SortformerOracle(w, 1, 1)
    mel = SO.synthetic_mel(3, 200)
    emb, T2, v2 = o.pre_encode(mel, 180)
    assert (T2, v2) == (SO.conv_len(SO.conv_len(SO.conv_len(200))),
                        SO.conv_len(SO.conv_len(SO.conv_len(180))))
    preds = o.encode_decode(emb, v2)
    assert preds.shape == (T2, 4) and np.isfinite(preds).all()
    assert (preds[v2:] == 0).all() and (preds[:v2] > 0).all() and (preds[:v2] < 1).all()
