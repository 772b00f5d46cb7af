"""Next tokens from the final hidden states on the CPU (test infrastructure
only).

Restates what the reference does after the decoder stack: ``logits =
lm_head(hidden)`` in bf16 (a GEMM accumulated in fp32, its result rounded
to bf16) followed by ``logits.argmax(dim=-1)``
(hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py D:1057-1064); torch's
argmax returns the first maximal index.  Here the logits are summed exactly
(fp64 sums of products of bf16 inputs) and rounded once to bf16, so the
oracle is the exact-arithmetic form of that computation; a kernel that sums
in fp32 in another order can only differ on rows whose top logits lie
within one bf16 step of each other.
"""
from __future__ import annotations

import numpy as np
import torch


def round_bf16(x):
    """Round float64 values to the nearest bf16 (ties to even), returned as
    float64.  Normal range only (|x| >= 2^-126 or 0), as logits are."""
    x = np.asarray(x, dtype=np.float64)
    m, e = np.frexp(x)                       # x = m * 2^e, 0.5 <= |m| < 1
    return np.ldexp(np.rint(m * 256.0), e - 8)


def exact_logits(hidden, weight):
    """fp64 logits ``hidden @ weight^T`` of bf16 inputs ([Q, H], [V, H])."""
    h = torch.as_tensor(hidden).to(torch.bfloat16).double().numpy()
    w = torch.as_tensor(weight).to(torch.bfloat16).double().numpy()
    return h @ w.T


def lm_head_argmax(hidden, weight):
    """``(ids int64 [Q], max bf16 logit as float64 [Q], exact logits [Q, V])``."""
    exact = exact_logits(hidden, weight)
    rounded = round_bf16(exact)
    ids = rounded.argmax(axis=1)             # first maximal index, as torch
    return ids.astype(np.int64), rounded[np.arange(len(ids)), ids], exact


def near_tie(exact_row, got, want):
    """True when id ``got`` is an acceptable answer in place of ``want``: its
    exact logit is within one bf16 step (at the row maximum) of the best,
    so an fp32 sum in another order can round it to the same bf16 value."""
    best = exact_row[want]
    _, e = np.frexp(best)
    step = np.ldexp(1.0, int(e) - 8)
    return exact_row[got] >= best - step
