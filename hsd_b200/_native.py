"""ctypes binding of the in-tree C-ABI library ``libhsd_b200.so``.

The library is the product: there is no Python or PyTorch fallback for any
of its kernels.  Loading fails loudly (``HSDNativeError``) when the library is
missing, and every call raises ``HSDError`` with the library's message when an
entry point returns a non-zero status.  Structures mirror
``include/hsd_b200.h`` field for field.
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhsd_b200.so")

HSD_OK = 0
HSD_SEG_CAUSAL, HSD_SEG_TREE, HSD_SEG_SINGLE, HSD_SEG_NONE = 0, 1, 2, 3
HSD_MODE_NORMAL, HSD_MODE_SPEC, HSD_MODE_TREE, HSD_MODE_FINISHED = 0, 1, 2, 3
HSD_DEV_TIMEOUT = 0x10000
HSD_DEV_BAD_INDEX = 0x20000
HSD_DEV_CAPACITY = 0x40000


class HSDError(RuntimeError):
    """An hsd_b200 entry point rejected its arguments or CUDA failed."""


class HSDNativeError(ImportError):
    """The compiled library is missing or unusable."""


class Segment(C.Structure):
    _fields_ = [("q_start", C.c_int32), ("q_len", C.c_int32), ("kind", C.c_int32),
                ("tree_off", C.c_int32), ("tree_words", C.c_int32), ("reserved", C.c_int32)]


class Plan(C.Structure):
    _fields_ = [("q_len", C.c_int32), ("kv_len", C.c_int32), ("n_qtiles", C.c_int32),
                ("n_kv64", C.c_int32), ("n_kv128", C.c_int32), ("reserved", C.c_int32),
                ("mask_words", C.c_void_p), ("tile_class", C.c_void_p),
                ("kv_num_blocks", C.c_void_p), ("kv_indices", C.c_void_p),
                ("full_kv_num_blocks", C.c_void_p), ("full_kv_indices", C.c_void_p),
                ("blk_count", C.c_void_p), ("blk_list", C.c_void_p),
                ("tile_order", C.c_void_p), ("blk_prefix", C.c_void_p)]


class Block(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "mode", "q_start", "q_len", "valid_count", "gen_off", "gen_len", "gen_cap",
        "draft_off", "draft_len", "mws", "matches_len", "tree_off", "tree_nodes", "seg",
        "flags", "reserved")]


class BlockResult(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "finished", "increment", "pointer", "next_token", "match_count", "match_start",
        "slice_begin", "slice_end")]


class AcceptConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "n_blocks", "kv_len", "kv_base", "kv_words_stride", "match_window_size",
        "match_window_size_upper_bound", "max_spec_len", "repeat_sentinel", "n_eos")] + \
        [("eos_ids", C.c_int32 * 8)]


class AcceptLogits(C.Structure):
    _fields_ = [("max_logit", C.c_void_p), ("probe_logit", C.c_void_p),
                ("spec_thresh", C.c_float), ("tree_thresh", C.c_float),
                ("variant", C.c_int32), ("formula_tokens", C.c_int32 * 2),
                ("spec_mode", C.c_int32), ("spec_topk", C.c_int32), ("spec_margin", C.c_float),
                ("rank", C.c_void_p), ("second", C.c_void_p)]


HSD_ACCEPT_DOTS, HSD_ACCEPT_HUNYUAN = 0, 1
HSD_SPEC_FMST, HSD_SPEC_TOPK, HSD_SPEC_ADAPTIVE = 0, 1, 2
SPEC_MODES = {"fmst": HSD_SPEC_FMST, "topk": HSD_SPEC_TOPK, "adaptive": HSD_SPEC_ADAPTIVE}


# (name, restype, argtypes) of every entry point include/hsd_b200.h declares.
_P, _I32, _I64, _F, _SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t
SIGNATURES = [
    ("hsd_version", C.c_char_p, []),
    ("hsd_last_error", C.c_char_p, []),
    ("hsd_plan_workspace_bytes", _SZ, [_I32, _I32]),
    ("hsd_plan_init", C.c_int, [_P, _SZ, _I32, _I32, C.POINTER(Plan)]),
    ("hsd_build_plan_segments", C.c_int,
     [_P, _I32, _P, _P, _I32, _P, C.POINTER(Plan), _P, _P]),
    ("hsd_build_plan_dense", C.c_int, [_P, _I64, C.POINTER(Plan), _P, _P]),
    ("hsd_attention_workspace_bytes", _SZ, [_I32, _I32, _I32]),
    ("hsd_verify_attention", C.c_int,
     [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64, _P, _P, _I32, _I32, _I32, _I32,
      _I32, _F, C.POINTER(Plan), _P, _SZ, _P, _P]),
    ("hsd_attention_static_scratch_bytes", _SZ, []),
    ("hsd_verify_attention_static_scratch", C.c_int,
     [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64, _P, _P, _I32, _I32, _I32, _I32,
      _I32, _F, C.POINTER(Plan), _P, _P]),
    ("hsd_compact_kv", C.c_int, [_P, _I32, _I32, _P, _I32, _P, _P, _P]),
    ("hsd_kv_append", C.c_int, [_P, _P, _I32, _I32, _I32, _I32, _P]),
    ("hsd_keep_indices", C.c_int, [_P, _I32, _I32, _P, _I32, _P, _P, _P, _P]),
    ("hsd_compact_bits", C.c_int, [_P, _P, _I32, _I32, _P, _P, _I32, _P]),
    ("hsd_accept_kmp", C.c_int,
     [C.POINTER(AcceptConfig), _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    ("hsd_accept_kmp_logits", C.c_int,
     [C.POINTER(AcceptConfig), _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
      C.POINTER(AcceptLogits), _P, _P]),
    ("hsd_rope_append", C.c_int,
     [_P, _I64, _P, _P, _I64, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _I64, _P, _I64, _I64,
      _I32, _P]),
    ("hsd_continuation_trees", C.c_int,
     [_P, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P]),
    ("hsd_selftest_bounded_wait", C.c_int, [_P, _P, _P]),
    ("hsd_lm_head_argmax_workspace_bytes", _SZ, [_I32]),
    ("hsd_lm_head_argmax", C.c_int,
     [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _SZ, _P, _P]),
    ("hsd_lm_head_rank", C.c_int,
     [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    ("hsd_probe_logits", C.c_int,
     [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _P, _I32, _P, _P, _P]),
]

_lib = None


def load():
    """Load ``libhsd_b200.so`` once; raise ``HSDNativeError`` if unusable."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise HSDNativeError(
            f"{LIB_PATH} is missing: build it with `python -m hsd_b200.build` "
            "(there is no fallback path)")
    try:
        lib = C.CDLL(LIB_PATH)
    except OSError as e:  # pragma: no cover - depends on the machine
        raise HSDNativeError(f"cannot load {LIB_PATH}: {e}") from e
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str):
    if rc != HSD_OK:
        msg = load().hsd_last_error().decode(errors="replace")
        raise HSDError(f"{what} failed ({rc}): {msg}")


def stream_handle(stream=None):
    """Raw ``cudaStream_t`` of a torch stream (current stream by default)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def ptr(t):
    """Device address of a torch tensor (or None -> NULL)."""
    return None if t is None else C.c_void_p(t.data_ptr())
