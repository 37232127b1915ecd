"""tcgen05 GEMM (orx_linear_pre, the asr_gemm::LinearPre equivalent) against
an fp64 reference over bf16-quantised operands, the scheme of the reference's
own known-answer test (test/unit/model/test_asr_gemm.cc:286-386, seed
20260627, uniform [-1, 1)); here the max-abs error against fp64 must stay below 5e-4 of the
output's RMS for K up to 6144 (tensor-core fp32 accumulation; the reference's
own test allows 2e-2 elementwise-relative)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def run(torch, M, K, N, seed=20260627):
    from orator_b200._lib import call
    g = np.random.default_rng(seed)
    x = torch.from_numpy(g.uniform(-1, 1, (M, K)).astype(np.float32)).to(torch.bfloat16).cuda()
    w = torch.from_numpy(g.uniform(-1, 1, (N, K)).astype(np.float32)).to(torch.bfloat16).cuda()
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    call("orx_linear_pre", C.c_void_p(x.data_ptr()), C.c_void_p(w.data_ptr()), None,
         C.c_void_p(out.data_ptr()), M, K, N, 0, None)
    torch.cuda.synchronize()
    ref = (x.double() @ w.double().T).cpu().numpy()
    got = out.cpu().numpy()
    return float(np.abs(got - ref).max() / np.sqrt(np.mean(ref * ref)))


@pytest.mark.parametrize("M,K,N", [(1, 1024, 1024), (1, 1024, 2048), (4, 1024, 1024),
                                   (4, 1024, 2048), (2, 1024, 1024),
                                   (64, 2048, 4096), (64, 6144, 2048), (17, 2048, 128),
                                   (400, 2048, 2048), (200, 2048, 12288), (256, 4096, 256)])
def test_tc_gemm_vs_f64(cuda, M, K, N):
    assert run(cuda, M, K, N) < 5e-4


def test_tc_gemm_rejects_bad_arguments(cuda):
    """Argument errors are caught on the host, before any launch."""
    import torch
    from orator_b200._lib import OrxError, call
    x = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(128, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(4, 128, device="cuda")
    args = [C.c_void_p(x.data_ptr()), C.c_void_p(w.data_ptr()), None, C.c_void_p(out.data_ptr())]
    with pytest.raises(OrxError):  # activation code out of range
        call("orx_linear_pre", *args, 4, 128, 128, 7, None)
    with pytest.raises(OrxError):  # null weight
        call("orx_linear_pre", args[0], None, None, args[3], 4, 128, 128, 0, None)
    with pytest.raises(OrxError):  # odd address for a bf16 operand
        call("orx_linear_pre", C.c_void_p(x.data_ptr() + 1), args[1], None, args[3], 4, 128, 128, 0,
             None)
    torch.cuda.synchronize()


def test_gemm_deterministic(cuda):
    """Repeated launches give bit-identical results."""
    import torch
    from orator_b200._lib import call
    g = np.random.default_rng(7)
    for M, K, N in [(64, 6144, 2048), (16, 2048, 2048), (1, 2048, 4096)]:
        x = torch.from_numpy(g.uniform(-1, 1, (M, K)).astype(np.float32)).to(torch.bfloat16).cuda()
        w = torch.from_numpy(g.uniform(-1, 1, (N, K)).astype(np.float32)).to(torch.bfloat16).cuda()
        outs = []
        for _ in range(2):
            out = torch.empty((M, N), dtype=torch.float32, device="cuda")
            call("orx_linear_pre", C.c_void_p(x.data_ptr()), C.c_void_p(w.data_ptr()), None,
                 C.c_void_p(out.data_ptr()), M, K, N, 0, None)
            outs.append(out)
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1])
        ref = x.double() @ w.double().T
        err = (outs[0].double() - ref).abs().max() / ref.pow(2).mean().sqrt()
        assert err < 5e-4
