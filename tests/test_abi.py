"""C-ABI library: loads, exports every declared entry point, validates arguments.

No compute call is made here: every call below is rejected on the host before
any CUDA work, so this runs without a GPU.
"""
import ctypes as C
import os
import re

import pytest

from hsd_b200 import _native as N

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "hsd_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hsd_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = N.load()
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == {s[0] for s in N.SIGNATURES}


def test_version_and_error_strings():
    lib = N.load()
    assert b"sm_100a" in lib.hsd_version()
    assert isinstance(lib.hsd_last_error(), bytes)


def test_struct_sizes_match_header():
    assert C.sizeof(N.Segment) == 24
    assert C.sizeof(N.Block) == 64
    assert C.sizeof(N.BlockResult) == 32
    assert C.sizeof(N.AcceptConfig) == 4 * 17
    assert C.sizeof(N.Plan) == 24 + 10 * 8


def test_plan_layout_host_only():
    lib = N.load()
    assert lib.hsd_plan_workspace_bytes(0, 10) == 0
    n = lib.hsd_plan_workspace_bytes(1512, 1512)
    # mask words dominate: 12 q tiles x 24 kv tiles x 128 rows x 8 bytes
    assert n >= 12 * 24 * 128 * 8
    buf = C.create_string_buffer(n + 512)
    base = (C.addressof(buf) + 255) & ~255
    plan = N.Plan()
    assert lib.hsd_plan_init(C.c_void_p(base), n, 1512, 1512, C.byref(plan)) == 0
    assert (plan.n_qtiles, plan.n_kv64, plan.n_kv128) == (12, 24, 12)
    ptrs = [plan.mask_words, plan.tile_class, plan.kv_num_blocks, plan.kv_indices,
            plan.full_kv_num_blocks, plan.full_kv_indices, plan.blk_count, plan.blk_list,
            plan.tile_order, plan.blk_prefix]
    assert all(p % 256 == 0 for p in ptrs)
    assert ptrs == sorted(ptrs) and ptrs[-1] < base + n
    # too small / misaligned workspaces are rejected
    assert lib.hsd_plan_init(C.c_void_p(base), n - 1, 1512, 1512, C.byref(plan)) != 0
    assert lib.hsd_plan_init(C.c_void_p(base + 8), n, 1512, 1512, C.byref(plan)) != 0
    assert b"aligned" in lib.hsd_last_error()


def test_attention_rejects_bad_head_dim_on_host():
    lib = N.load()
    plan = N.Plan()
    plan.q_len, plan.kv_len = 128, 128
    rc = lib.hsd_verify_attention(None, 64, 64, None, 64, 64, None, 64, 64, None, None,
                                  128, 128, 2, 1, 64, 0.1, C.byref(plan), None, 0, None, None)
    assert rc == N.HSD_OK + 2  # HSD_ERR_UNSUPPORTED
    assert b"head_dim" in lib.hsd_last_error()


def test_attention_workspace_size_host_only():
    lib = N.load()
    assert lib.hsd_attention_workspace_bytes(0, 12, 2) == 0
    assert lib.hsd_attention_workspace_bytes(128, 12, 5) == 0
    n = lib.hsd_attention_workspace_bytes(2176, 12, 2)
    # a partial-row record per head slot for every SM (148 on B200 when no
    # GPU is visible), plus their flags
    assert n >= 148 * 2 * (128 * 64 + 256) * 4


def test_other_entry_points_reject_null_arguments():
    lib = N.load()
    assert lib.hsd_compact_kv(None, 0, 256, None, 0, None, None, None) != 0
    assert lib.hsd_keep_indices(None, 0, 0, None, 0, None, None, None, None) != 0
    assert lib.hsd_compact_bits(None, None, 0, 0, None, None, 0, None) != 0
    cfg = N.AcceptConfig()
    assert lib.hsd_accept_kmp(C.byref(cfg), None, None, None, None, None, None, None,
                              None, None, None, None, None, None) != 0
    plan = N.Plan()
    assert lib.hsd_build_plan_segments(None, 0, None, None, 0, None, C.byref(plan),
                                       None, None) != 0
    assert lib.hsd_build_plan_dense(None, 0, C.byref(plan), None, None) != 0


def test_lm_head_argmax_host_checks():
    lib = N.load()
    assert lib.hsd_lm_head_argmax_workspace_bytes(0) == 0
    assert lib.hsd_lm_head_argmax_workspace_bytes(2176) == 2176 * 8 + 256
    # no id output / unaligned pointer / stride below hidden_dim: rejected on the host
    assert lib.hsd_lm_head_argmax(C.c_void_p(256), 1536, C.c_void_p(256), 1536, 4, 100, 1536,
                                  None, None, None, None, 0, None, None) != 0
    assert b"bad arguments" in lib.hsd_last_error()
    assert lib.hsd_lm_head_argmax(C.c_void_p(8), 1536, C.c_void_p(256), 1536, 4, 100, 1536,
                                  C.c_void_p(256), None, None, None, 0, None, None) != 0
    assert lib.hsd_lm_head_argmax(C.c_void_p(256), 1000, C.c_void_p(256), 1536, 4, 100, 1536,
                                  C.c_void_p(256), None, None, None, 0, None, None) != 0
    # too small a workspace
    assert lib.hsd_lm_head_argmax(C.c_void_p(256), 1536, C.c_void_p(256), 1536, 4, 100, 1536,
                                  C.c_void_p(256), None, None, C.c_void_p(256), 64, None,
                                  None) != 0
    assert b"workspace" in lib.hsd_last_error()


def test_lm_head_rank_host_checks():
    lib = N.load()
    a = C.c_void_p(256)
    # a missing per-row input / an unaligned hidden pointer / too small a workspace
    assert lib.hsd_lm_head_rank(a, 1536, a, 1536, 4, 100, 1536, None, a, a, a, a, a, 4096,
                                None, None) != 0
    assert b"bad arguments" in lib.hsd_last_error()
    assert lib.hsd_lm_head_rank(C.c_void_p(8), 1536, a, 1536, 4, 100, 1536, a, a, a, a, a, a,
                                4096, None, None) != 0
    assert b"bad arguments" in lib.hsd_last_error()
    assert lib.hsd_lm_head_rank(a, 1536, a, 1536, 4, 100, 1536, a, a, a, a, a, a, 64, None,
                                None) != 0
    assert b"workspace" in lib.hsd_last_error()


def test_rope_append_host_checks():
    lib = N.load()
    a = C.c_void_p(256)
    # head_dim other than 128
    assert lib.hsd_rope_append(a, 1536, a, a, 256, a, a, 128, 4, 12, 2, 64, a, 4096, a, 4096,
                               128, 0, None) == N.HSD_OK + 2
    # unaligned key pointer, then a row stride too small for the heads
    assert lib.hsd_rope_append(a, 1536, C.c_void_p(258), a, 256, a, a, 128, 4, 12, 2, 128, a,
                               4096, a, 4096, 128, 0, None) != 0
    assert lib.hsd_rope_append(a, 1000, a, a, 256, a, a, 128, 4, 12, 2, 128, a, 4096, a, 4096,
                               128, 0, None) != 0
    assert b"bad arguments" in lib.hsd_last_error()
    # zero rows: nothing to do, no launch
    assert lib.hsd_rope_append(a, 1536, a, a, 256, a, a, 128, 0, 12, 2, 128, a, 4096, a, 4096,
                               128, 0, None) == 0


def test_continuation_trees_host_checks():
    lib = N.load()
    a = C.c_void_p(256)
    args = [a, a, a, a, 3, 15]
    assert lib.hsd_continuation_trees(*args, 0, a, a, a, a, a, None, None) != 0      # cap 0
    assert lib.hsd_continuation_trees(*args, 1025, a, a, a, a, a, None, None) != 0   # cap > 1024
    assert b"cap" in lib.hsd_last_error()
    assert lib.hsd_continuation_trees(None, None, None, None, 0, 15, 256, None, None, None, None,
                                      None, None, None) == 0                        # nothing to do
