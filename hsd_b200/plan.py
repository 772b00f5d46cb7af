"""Packed verification masks and their tile plans (host side of subsystem 4).

The reference hands its attention a dense float mask ``[1, 1, Q, KV]`` and
converts it per step with ``create_block_mask(make_mask_mod(mask), ...,
BLOCK_SIZE=(128, 64))`` (hsd/dots_ocr_pipeline/modeling_dots_ocr_hsd.py
D:94-106, D:148-153).  Here a mask is either

* :class:`PackedMask` -- segment descriptors (row ranges, one KV visibility
  bitset per segment, an intra-segment pattern) that never materialise the
  dense matrix, or
* a dense float tensor, accepted for drop-in use,

and :class:`TilePlan` is the device-built plan the attention kernel consumes
(the BlockMask equivalent).  Both are built once per step and shared by all
decoder layers, as the reference caches its BlockMask per step (D:83-106).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native as N

SEG_CAUSAL, SEG_TREE, SEG_SINGLE, SEG_NONE = (N.HSD_SEG_CAUSAL, N.HSD_SEG_TREE,
                                              N.HSD_SEG_SINGLE, N.HSD_SEG_NONE)


def _dev_status(device):
    return torch.zeros(1, dtype=torch.int32, device=device)


class TilePlan:
    """Device tile plan for one (q_len, kv_len) mask (BlockMask equivalent)."""

    def __init__(self, q_len: int, kv_len: int, device):
        lib = N.load()
        self.q_len, self.kv_len = int(q_len), int(kv_len)
        nbytes = lib.hsd_plan_workspace_bytes(self.q_len, self.kv_len)
        if nbytes == 0:
            raise N.HSDError(f"empty plan (q_len={q_len}, kv_len={kv_len})")
        self.workspace = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        base = (self.workspace.data_ptr() + 255) & ~255
        self.struct = N.Plan()
        N.check(lib.hsd_plan_init(C.c_void_p(base), nbytes, self.q_len, self.kv_len,
                                  C.byref(self.struct)), "hsd_plan_init")
        self.status = _dev_status(device)
        self.device = device

    # -- views of the plan arrays (for tests and diagnostics) -------------
    def _view(self, field, dtype, shape):
        addr = getattr(self.struct, field)
        base = self.workspace.data_ptr()
        off = addr - base
        n = int(np.prod(shape)) * torch.empty((), dtype=dtype).element_size()
        return self.workspace[off:off + n].view(dtype).view(*shape)

    @property
    def n_qtiles(self):
        return self.struct.n_qtiles

    def tile_class(self):
        return self._view("tile_class", torch.uint8, (self.n_qtiles, self.struct.n_kv64))

    def block_mask_lists(self):
        """(kv_num_blocks, kv_indices, full_kv_num_blocks, full_kv_indices) on the host."""
        nq, n64 = self.n_qtiles, self.struct.n_kv64
        kn = self._view("kv_num_blocks", torch.int32, (nq,)).cpu().tolist()
        fn = self._view("full_kv_num_blocks", torch.int32, (nq,)).cpu().tolist()
        ki = self._view("kv_indices", torch.int32, (nq, n64)).cpu()
        fi = self._view("full_kv_indices", torch.int32, (nq, n64)).cpu()
        return (kn, [ki[i, :n].tolist() for i, n in enumerate(kn)],
                fn, [fi[i, :n].tolist() for i, n in enumerate(fn)])

    def mask_words(self):
        return self._view("mask_words", torch.int64, (self.n_qtiles, self.struct.n_kv64, 128))

    def blocks(self):
        cnt = self._view("blk_count", torch.int32, (self.n_qtiles,))
        lst = self._view("blk_list", torch.int32, (self.n_qtiles, self.struct.n_kv128))
        return cnt, lst

    def dense_allowed(self):
        """Expand the stored row masks to a bool [q_len, kv_len] matrix (tests)."""
        w = self.mask_words().cpu().numpy().view(np.uint64)  # [nq, n64, 128]
        nq, n64 = w.shape[0], w.shape[1]
        bits = np.unpackbits(w.view(np.uint8).reshape(nq, n64, 128, 8), axis=-1,
                             bitorder="little").reshape(nq, n64, 128, 64)
        dense = bits.transpose(0, 2, 1, 3).reshape(nq * 128, n64 * 64)
        return dense[:self.q_len, :self.kv_len].astype(bool)

    def raise_on_device_error(self):
        code = int(self.status.item())
        if code:
            raise N.HSDError(f"device status 0x{code:x} while building the tile plan")


class PackedMask:
    """Segment-form verification mask (see module docstring).

    ``segments`` is a list of dicts with ``q_start``, ``q_len``, ``kind``
    (SEG_*), ``kv`` (bool array over ``kv_len`` columns: the columns every
    row of the segment sees besides its own pattern) and, for SEG_TREE,
    ``parents`` (parent node of each real node, -1 for the root).  Rows that
    no segment covers are fully masked.
    """

    def __init__(self, q_len, kv_len, segments, device="cuda", words_stride=None):
        self.q_len, self.kv_len = int(q_len), int(kv_len)
        n64 = (self.kv_len + 63) // 64
        self.stride = int(words_stride or n64)
        nseg = len(segments)
        segs = np.zeros((max(nseg, 1), 6), dtype=np.int32)
        row_seg = np.full(self.q_len, -1, dtype=np.int32)
        kv_bits = np.zeros((max(nseg, 1), self.stride), dtype=np.uint64)
        tree_rows = []
        tree_off = 0
        for i, s in enumerate(segments):
            qs, ql, kind = int(s["q_start"]), int(s["q_len"]), int(s["kind"])
            segs[i, :3] = (qs, ql, kind)
            row_seg[qs:qs + ql] = i
            kv = np.asarray(s.get("kv", np.zeros(self.kv_len, bool)), dtype=bool)
            if kv.shape[0] != self.kv_len:
                raise ValueError("segment kv visibility must cover kv_len columns")
            kv_bits[i, :n64] = pack_bits(kv)
            if kind == SEG_TREE:
                tw = (ql + 63) // 64
                anc = np.zeros((ql, tw * 64), dtype=bool)
                parents = list(s["parents"])
                for j in range(len(parents)):
                    a = j
                    while a >= 0:
                        anc[j, a] = True
                        a = parents[a]
                tree_rows.append(pack_bits(anc).reshape(ql, tw))
                segs[i, 3], segs[i, 4] = tree_off, tw
                tree_off += ql * tw
        tree = (np.concatenate([t.ravel() for t in tree_rows]) if tree_rows
                else np.zeros(1, dtype=np.uint64))
        self.n_segs = nseg
        self.device = device
        self.segs = torch.from_numpy(segs).to(device)
        self.row_seg = torch.from_numpy(row_seg).to(device)
        self.kv_bits = torch.from_numpy(kv_bits.view(np.int64)).to(device)
        self.tree_bits = torch.from_numpy(tree.view(np.int64)).to(device)
        self._plan = None

    @classmethod
    def from_bits(cls, q_len, kv_len, segs, row_seg, kv_bits, device="cuda", tree_bits=None):
        """A mask whose segment visibility rows are already in device memory.

        ``segs``: int32 ``[n, 6]`` rows of ``hsd_segment_t``; ``row_seg``:
        int32 ``[q_len]`` (-1: row fully masked); ``kv_bits``: device int64
        ``[n, stride]`` visibility rows (bit c of row i = column c), e.g. the
        rows the acceptance kernel writes.  Tree segments need ``tree_bits``.
        """
        self = cls.__new__(cls)
        self.q_len, self.kv_len = int(q_len), int(kv_len)
        self.stride = int(kv_bits.shape[-1])
        if self.stride * 64 < self.kv_len:
            raise ValueError("visibility rows shorter than kv_len")
        segs = np.asarray(segs, dtype=np.int32).reshape(-1, 6)
        self.n_segs = segs.shape[0]
        self.device = device
        self.segs = torch.from_numpy(segs).to(device)
        self.row_seg = torch.from_numpy(np.asarray(row_seg, dtype=np.int32)).to(device)
        self.kv_bits = kv_bits
        self.tree_bits = (tree_bits if tree_bits is not None
                          else torch.zeros(1, dtype=torch.int64, device=device))
        self._plan = None
        return self

    def plan(self, stream=None) -> TilePlan:
        """Build (once) the device tile plan of this mask."""
        if self._plan is None:
            lib = N.load()
            plan = TilePlan(self.q_len, self.kv_len, self.device)
            N.check(lib.hsd_build_plan_segments(
                N.ptr(self.segs), max(self.n_segs, 1), N.ptr(self.row_seg),
                N.ptr(self.kv_bits), self.stride, N.ptr(self.tree_bits),
                C.byref(plan.struct), N.ptr(plan.status), N.stream_handle(stream)),
                "hsd_build_plan_segments")
            self._plan = plan
        return self._plan


def pack_bits(b):
    """bool [..., n] -> uint64 [..., ceil(n/64)] (bit i of word w = element 64w+i)."""
    b = np.asarray(b, dtype=bool)
    n = b.shape[-1]
    pad = (-n) % 64
    if pad:
        b = np.concatenate([b, np.zeros(b.shape[:-1] + (pad,), bool)], axis=-1)
    by = np.packbits(b.reshape(b.shape[:-1] + (-1, 8)), axis=-1, bitorder="little")
    return by.reshape(b.shape[:-1] + (-1, 8)).copy().view(np.uint64)[..., 0]


def plan_from_dense(mask: torch.Tensor, kv_len: int | None = None, stream=None) -> TilePlan:
    """Tile plan of a dense float mask ``[..., Q, >=KV]`` (allowed: > -0.1)."""
    lib = N.load()
    m = mask
    while m.dim() > 2:
        m = m[0]
    if m.dtype != torch.float32:
        m = m.float()
    if m.stride(-1) != 1:
        m = m.contiguous()
    q_len = m.shape[0]
    kv = int(kv_len if kv_len is not None else m.shape[1])
    plan = TilePlan(q_len, kv, m.device)
    N.check(lib.hsd_build_plan_dense(N.ptr(m), m.stride(0), C.byref(plan.struct),
                                     N.ptr(plan.status), N.stream_handle(stream)),
            "hsd_build_plan_dense")
    plan._src = m  # keep the source alive while the launch may still read it
    return plan
