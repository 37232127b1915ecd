"""The allocation-free argmax entry point (orx_argmax_banned_noalloc) against
the decoder's regular argmax entry point on the same device logits.

It exists for callers that cannot allocate device memory (inside a stream
capture they do not own, on real-time threads that must not take allocation
locks, or with device memory reserved by another allocator). This file is
collected last so a failing run has already run every other test; it also
passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_argmax_matches_regular_entry_point(cuda):
    torch = cuda
    from orator_b200 import AsrTextConfig, AsrTextDecoder
    from orator_b200._lib import OrxError, call

    V = 151936
    dec = AsrTextDecoder(AsrTextConfig(num_layers=1, vocab_size=V, max_seq_len=64))
    dec.init_synthetic(3)
    x = np.random.default_rng(5).standard_normal((6, 2048)).astype(np.float32)
    dec.Prefill(x)
    logits = dec.logits_device_ptr()
    host = dec.CopyLogits()
    top = [int(i) for i in np.argsort(host)[::-1][:3]]
    out = torch.full((2,), -7, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # two calls in a row each, with and without banned ids (tolerance: exact)
    for ban0, ban1 in [(-1, -1), (top[0], -1), (top[0], top[1]), (-1, -1)]:
        dec.ArgmaxToDevice(out.data_ptr(), ban0, ban1, s)
        call("orx_argmax_banned_noalloc", C.c_void_p(logits), V, ban0, ban1,
             C.c_void_p(out.data_ptr() + 4), C.c_void_p(s))
        torch.cuda.synchronize()
        a, b = out.tolist()
        assert a == b, (ban0, ban1, a, b)
    assert out.tolist()[1] == top[0]

    # a second, unrelated input through the same shared scratch
    y = torch.randn(300001, device="cuda")
    y[123457] = 50.0
    call("orx_argmax_banned_noalloc", C.c_void_p(y.data_ptr()), y.numel(), -1, -1,
         C.c_void_p(out.data_ptr()), C.c_void_p(s))
    torch.cuda.synchronize()
    assert out.tolist()[0] == 123457

    with pytest.raises(OrxError):
        call("orx_argmax_banned_noalloc", C.c_void_p(logits), 8388609, -1, -1,
             C.c_void_p(out.data_ptr()), C.c_void_p(s))
    dec.close()
