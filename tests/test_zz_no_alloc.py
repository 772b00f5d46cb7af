"""Attention through the entry point that allocates nothing.

``hsd_verify_attention_static_scratch`` runs the stream-K attention with its
scratch in a static device array; it must give the same output as
``hsd_verify_attention`` with a caller workspace, on consecutive calls (the
array keeps what the previous call left; each call clears the flags and
counters that must start at zero).  It is for callers that cannot allocate
device memory themselves.  Collected last so that it also runs after every
other GPU test in the same process; it passes alone as well.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from hsd_b200 import _native as N


def test_static_scratch_size_is_stated():
    lib = N.load()
    assert lib.hsd_attention_static_scratch_bytes() == 20 << 20
    # one CTA per SM needs a 33 KB partial record per head slot plus 32 bytes
    # of flags, and the whole scratch 256 bytes of counters: 148 SMs fit, and
    # so would 310
    per_sm = 2 * (128 * 64 + 256) * 4 + 32
    assert 310 * per_sm + 256 <= 20 << 20 < 311 * per_sm + 256
    assert lib.hsd_attention_workspace_bytes(1024, 12, 2) <= 20 << 20


def _call(lib, fn, q, k, v, plan, out, lse, scale, extra):
    hq, q_len, d = q.shape
    hkv, kv_len = k.shape[0], k.shape[1]
    return getattr(lib, fn)(
        N.ptr(q), q.stride(1), q.stride(0), N.ptr(k), k.stride(1), k.stride(0),
        N.ptr(v), v.stride(1), v.stride(0), N.ptr(out), N.ptr(lse), q_len, kv_len, hq, hkv,
        d, ctypes.c_float(scale), ctypes.byref(plan.struct), *extra, N.ptr(plan.status),
        N.stream_handle(None))


def _segments(q_len, kv_len, prefix, rng):
    """Causal prefix rows plus drafts that each see the prefix and themselves."""
    from oracle import masks as OM
    segs = [dict(q_start=0, q_len=prefix, kind=OM.CAUSAL, kv=np.zeros(kv_len, bool))]
    vis = np.zeros(kv_len, bool)
    vis[:prefix] = True
    qs = prefix
    while qs < q_len:
        n = int(min(q_len - qs, rng.integers(20, 200)))
        segs.append(dict(q_start=qs, q_len=n, kind=OM.CAUSAL, kv=vis.copy()))
        qs += n
    return segs


@pytest.mark.gpu
@pytest.mark.parametrize("q_len,prefix,hq,hkv", [(1536, 512, 12, 2), (700, 300, 8, 8)])
def test_static_scratch_matches_workspace_entry(q_len, prefix, hq, hkv):
    from hsd_b200.attention import attention_workspace
    from hsd_b200.plan import PackedMask

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    lib = N.load()
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(q_len)
    kv_len = q_len
    plan = PackedMask(q_len, kv_len, _segments(q_len, kv_len, prefix, rng), device=dev).plan()
    g = torch.Generator().manual_seed(q_len)
    q = (torch.randn(hq, q_len, 128, generator=g) / math.sqrt(128)).to(torch.bfloat16).to(dev)
    k = (torch.randn(hkv, kv_len, 128, generator=g) / math.sqrt(128)).to(torch.bfloat16).to(dev)
    v = torch.randn(hkv, kv_len, 128, generator=g).to(torch.bfloat16).to(dev)
    scale = 1.0 / math.sqrt(128)

    ws = attention_workspace(q_len, hq, hkv, dev)
    ref_out = torch.empty(q_len, hq, 128, dtype=torch.bfloat16, device=dev)
    ref_lse = torch.empty(hq, q_len, dtype=torch.float32, device=dev)
    N.check(_call(lib, "hsd_verify_attention", q, k, v, plan, ref_out, ref_lse, scale,
                  (ctypes.c_void_p(ws.base), ws.nbytes)), "hsd_verify_attention")
    torch.cuda.synchronize()
    plan.raise_on_device_error()

    for _ in range(2):  # the second call reuses the scratch the first one left behind
        out = torch.full_like(ref_out, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        N.check(_call(lib, "hsd_verify_attention_static_scratch", q, k, v, plan, out, lse,
                      scale, ()), "hsd_verify_attention_static_scratch")
        torch.cuda.synchronize()
        plan.raise_on_device_error()
        # same kernels and schedule: the results agree to within 0 (bit-identical)
        torch.testing.assert_close(out, ref_out, rtol=0, atol=0)
        torch.testing.assert_close(lse, ref_lse, rtol=0, atol=0)
