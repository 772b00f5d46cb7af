"""Device waits end in an error code, not a hang.

Every spin-wait in the library's kernels (mbarrier phases, stream-K partial
flags) gives up after a bounded time and records HSD_DEV_TIMEOUT | site in
the caller's status word.  ``hsd_selftest_bounded_wait`` runs that wait on a
device flag nothing sets; the test checks the status, the time it took, and
that the same context then runs a kernel of the library correctly.  No GPU
fault is involved.
"""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_that_cannot_finish_returns_timeout_status():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from hsd_b200 import _native as N
    lib = N.load()
    dev = torch.device("cuda:0")
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    N.check(lib.hsd_selftest_bounded_wait(N.ptr(flag), N.ptr(status), N.stream_handle()),
            "hsd_selftest_bounded_wait")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(status.item()) == N.HSD_DEV_TIMEOUT | 0x7F0
    assert 0.9 < dt < 10.0
    # the context is intact: a library kernel runs and is correct afterwards
    from hsd_b200.lm_head import lm_head_argmax
    g = torch.Generator(device=dev).manual_seed(0)
    h = torch.randn(64, 256, generator=g, device=dev).to(torch.bfloat16)
    w = torch.randn(1000, 256, generator=g, device=dev).to(torch.bfloat16)
    ids = lm_head_argmax(h, w)
    ref = (h.float() @ w.float().T).to(torch.bfloat16).argmax(-1)
    assert (ids == ref).float().mean().item() >= 0.99
