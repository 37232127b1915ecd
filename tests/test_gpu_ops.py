"""The free operators (orx_rms_norm, orx_rope_half / _interleaved, orx_swiglu,
orx_gqa_attention, orx_argmax_banned, orx_f32_to_bf16 / bf16_to_f32,
orx_linear / orx_linear_pre) against an independent f64 restatement and,
where the reference build in oracle/_ref is present, against the reference's
own asr_ops / asr_gemm kernels on the same device inputs.

Shapes follow the reference's op tests (test/unit/model/test_asr_ops.cc:73-169:
RMSNorm 8 x 2048, RoPE 12 tokens x 16 heads x 128, GQA T=24 Hq=16 Hkv=8 D=128
causal) and its f64 known-answer GEMM test (test/unit/model/test_asr_gemm.cc:
286-386: operands U(-1, 1), seed 20260627, the production (M, K, N) shape set,
act 0/1/2, max relative error <= 2e-2 against bf16-quantized operands
accumulated in f64)."""
import numpy as np
import pytest

import refharness

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env(cuda):
    from orator_b200 import ops
    ref = refharness.RefOps() if refharness.available() else None
    return cuda, ops, ref


def bf16_round(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def test_rms_norm(env):
    torch, ops, ref = env
    g = torch.Generator().manual_seed(1)
    for rows, dim in [(8, 2048), (3, 1024), (5, 130)]:  # 130: the scalar (unaligned-width) path
        x = torch.randn(rows, dim, generator=g)
        w = 1 + 0.1 * torch.randn(dim, generator=g)
        dx, dw = x.cuda(), w.cuda()
        out = torch.empty_like(dx)
        ops.RmsNorm(dx.data_ptr(), dw.data_ptr(), out.data_ptr(), rows, dim, 1e-6)
        torch.cuda.synchronize()
        x64 = x.double()
        want = x64 * torch.rsqrt((x64 * x64).mean(1, keepdim=True) + 1e-6) * w.double()
        got = out.cpu().double()
        assert (got - want).abs().max().item() <= 2e-6 * want.abs().max().item()
        if ref:
            r = torch.empty_like(dx)
            ref.rms_norm(dx.data_ptr(), dw.data_ptr(), r.data_ptr(), rows, dim, 1e-6)
            assert (r.cpu().double() - got).abs().max().item() <= 2e-6 * want.abs().max().item()
        # in place, as the reference allows
        ops.RmsNorm(dx.data_ptr(), dw.data_ptr(), dx.data_ptr(), rows, dim, 1e-6)
        torch.cuda.synchronize()
        assert torch.equal(dx.cpu(), out.cpu())


@pytest.mark.parametrize("half", [True, False])
def test_rope(env, half):
    torch, ops, ref = env
    T, H, D, base = 12, 16, 128, 1e6
    g = torch.Generator().manual_seed(2)
    x = torch.randn(T, H, D, generator=g)
    pos = torch.tensor([0, 1, 2, 5, 17, 100, 401, 527, 1000, 2047, 4000, 65535], dtype=torch.int32)
    dx, dp = x.cuda(), pos.cuda()
    fn = ops.RopeHalf if half else ops.RopeInterleaved
    fn(dx.data_ptr(), dp.data_ptr(), T, H, D, base)
    torch.cuda.synchronize()
    got = dx.cpu().double()
    j = torch.arange(D // 2, dtype=torch.float64)
    ang = pos.double()[:, None] * base ** (-2.0 * j / D)
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    x64 = x.double()
    if half:
        a, b = x64[..., : D // 2], x64[..., D // 2:]
        want = torch.cat([a * c - b * s, b * c + a * s], -1)
    else:
        a, b = x64[..., 0::2], x64[..., 1::2]
        want = torch.stack([a * c - b * s, a * s + b * c], -1).reshape(T, H, D)
    # fp32 angle rounding at position 65535 dominates: |pos| * ulp(inv_freq)
    assert (got - want).abs().max().item() <= 5e-2
    assert (got - want)[:8].abs().max().item() <= 1e-4
    if ref:
        r = x.cuda()
        (ref.rope_half if half else ref.rope_interleaved)(r.data_ptr(), dp.data_ptr(), T, H, D, base)
        # same angle formula and the same libm calls: bit-identical
        assert torch.equal(r.cpu(), dx.cpu())


def test_swiglu(env):
    torch, ops, ref = env
    g = torch.Generator().manual_seed(3)
    for n in [6144, 1, 100003]:
        a, b = torch.randn(n, generator=g) * 4, torch.randn(n, generator=g)
        da, db = a.cuda(), b.cuda()
        out = torch.empty_like(da)
        ops.SwiGLU(da.data_ptr(), db.data_ptr(), out.data_ptr(), n)
        torch.cuda.synchronize()
        a64 = a.double()
        want = a64 / (1 + torch.exp(-a64)) * b.double()
        assert (out.cpu().double() - want).abs().max().item() <= 1e-6 * max(1.0, want.abs().max().item())
        if ref:
            r = torch.empty_like(da)
            ref.swiglu(da.data_ptr(), db.data_ptr(), r.data_ptr(), n)
            assert torch.equal(r.cpu(), out.cpu())


@pytest.mark.parametrize("T,hq,hkv,D,causal", [(24, 16, 8, 128, True), (24, 16, 8, 128, False),
                                               (77, 16, 8, 128, True), (5, 4, 1, 64, True),
                                               (33, 6, 2, 256, False), (9, 2, 2, 48, True),
                                               (1, 16, 8, 128, True)])
def test_gqa_attention(env, T, hq, hkv, D, causal):
    torch, ops, ref = env
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(T, h, D, generator=g) for h in (hq, hkv, hkv))
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    out = torch.empty_like(dq)
    scale = 1.0 / D ** 0.5
    ops.GqaAttention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), T, hq, hkv, D,
                     scale, causal)
    torch.cuda.synchronize()
    grp = hq // hkv
    k64 = k.double().repeat_interleave(grp, 1)
    v64 = v.double().repeat_interleave(grp, 1)
    s = torch.einsum("thd,jhd->htj", q.double(), k64) * scale
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    want = torch.einsum("htj,jhd->thd", torch.softmax(s, -1), v64)
    got = out.cpu().double()
    assert (got - want).abs().max().item() <= 2e-5
    if ref and (D & (D - 1)) == 0:
        r = torch.empty_like(dq)
        ref.gqa(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), r.data_ptr(), T, hq, hkv, D, scale,
                causal)
        assert (r.cpu().double() - got).abs().max().item() <= 2e-5


def test_casts(env):
    torch, ops, ref = env
    x = torch.randn(100003) * 100
    x[:4] = torch.tensor([0.0, -0.0, 1e-40, 3.0e38])
    dx = x.cuda()
    b = torch.empty(x.numel(), dtype=torch.int16, device="cuda")
    ops.F32ToBf16(dx.data_ptr(), b.data_ptr(), x.numel())
    back = torch.empty_like(dx)
    ops.Bf16ToF32(b.data_ptr(), back.data_ptr(), x.numel())
    torch.cuda.synchronize()
    want = bf16_round(x.numpy())
    assert np.array_equal(back.cpu().numpy().view(np.uint32), want.view(np.uint32))
    if ref:
        r = torch.empty_like(b)
        ref.f32_to_bf16(dx.data_ptr(), r.data_ptr(), x.numel())
        assert torch.equal(r.cpu(), b.cpu())


# the reference test's production shapes (its default and ORATOR_GEMM_FULL sets) ...
REF_SHAPES = [(1, 1024, 1024), (1, 1024, 2048), (4, 1024, 1024), (4, 1024, 2048), (2, 1024, 1024),
              (1, 6144, 1024), (1, 1024, 6144), (6, 1024, 3072), (6, 3072, 1024), (4, 7680, 1024),
              (4, 1024, 5000), (8, 1024, 2048)]
# ... plus a full prefill tile, ragged N and K (K % 64 != 0 through the tensor
# maps' zero fill) and K % 8 != 0 (the CUDA-core path); the reference build is
# run only on its own shape set
SHAPES = REF_SHAPES + [(400, 2048, 2048), (37, 200, 300), (3, 100, 70), (5, 7, 9)]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_linear_vs_f64(env, M, K, N):
    torch, ops, ref = env
    rng = np.random.default_rng(20260627)
    x = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    w = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    xq, wq = bf16_round(x).astype(np.float64), bf16_round(w).astype(np.float64)
    pre = (xq @ wq.T).astype(np.float32) + bias
    dx, dwf, db = (torch.from_numpy(a).cuda() for a in (x, w, bias))
    dw = torch.empty(N * K, dtype=torch.int16, device="cuda")
    ops.F32ToBf16(dwf.data_ptr(), dw.data_ptr(), N * K)
    out = torch.empty(M, N, device="cuda")
    import math
    erf = np.vectorize(math.erf)
    for act in (0, 1, 2):
        ops.Linear(dx.data_ptr(), dw.data_ptr(), db.data_ptr(), out.data_ptr(), M, K, N, act)
        torch.cuda.synchronize()
        want = pre.astype(np.float64)
        if act == 1:
            want = 0.5 * want * (1 + erf(want / np.sqrt(2)))
        elif act == 2:
            want = np.maximum(want, 0)
        got = out.cpu().numpy().astype(np.float64)
        rel = np.abs(got - want) / np.maximum(1e-3, np.abs(want))
        if (M, K, N) in REF_SHAPES:  # the reference test's own bar, on its own shapes
            assert rel.max() <= 2e-2, (act, rel.max())
        # fp32 accumulation of exact products: far inside the 2e-2 bar
        assert np.abs(got - want).max() <= 1e-4 * np.sqrt(K), (act, np.abs(got - want).max())
        if ref and (M, K, N) in REF_SHAPES:
            r = torch.empty_like(out)
            ref.linear(dx.data_ptr(), dw.data_ptr(), db.data_ptr(), r.data_ptr(), M, K, N, act)
            assert np.abs(r.cpu().numpy() - got).max() <= 1e-4 * np.sqrt(K)
    # no bias, LinearPre on pre-cast activations
    xb = torch.empty(M * K, dtype=torch.int16, device="cuda")
    ops.F32ToBf16(dx.data_ptr(), xb.data_ptr(), M * K)
    ops.LinearPre(xb.data_ptr(), dw.data_ptr(), None, out.data_ptr(), M, K, N, 0)
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - (xq @ wq.T)).max() <= 1e-4 * np.sqrt(K)


def test_ops_reject_bad_arguments(env):
    torch, ops, ref = env
    from orator_b200 import OrxError
    buf = torch.zeros(64, device="cuda")
    p = buf.data_ptr()
    with pytest.raises(OrxError):
        ops.GqaAttention(p, p, p, p, 2, 3, 2, 8, 1.0, True)   # Hq not a multiple of Hkv
    with pytest.raises(OrxError):
        ops.RopeHalf(p, p, 1, 1, 7, 1e6)                      # odd head dim
    with pytest.raises(OrxError):
        ops.Linear(p, p, None, p, 1, 8, 8, 3)                 # unknown activation
    ops.RmsNorm(0, 0, 0, 0, 2048, 1e-6)                       # empty: no-op
