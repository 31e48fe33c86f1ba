"""Block-sparse attention masks (reference: src/pallas_flexattn/block_mask.py).

``BlockMask`` keeps the reference's five fields (``num_blocks_in_row``,
``col_indices``, ``block_size``, ``q_len``, ``kv_len``) and properties, and adds
the engine's FlexAttention-style tables (``tables``): partial and full kv lists
per q block plus their transpose for the backward pass, resident on the GPU.

``create_block_mask`` runs on the GPU (libflexattn ``fa_create_block_mask``):
one pass with the reference's 3x3 sampling rule produces the reference fields
bit for bit, one exact pass produces the tables the kernels walk.  The analytic
builders ``create_causal_block_mask`` / ``create_sliding_window_block_mask``
are host functions, as in the reference.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Optional

import torch

from . import _lib as L
from .mask_mod import MaskMod, MaskSpec, evaluate_mask, spec_of


@dataclass(frozen=True, eq=False)
class BlockTables:
    """Device-resident block tables for one (Tq, Tkv, block_q, block_kv) geometry."""

    block_q: int
    block_kv: int
    nq: int
    nkv: int
    num_b: int
    tile_class: torch.Tensor          # [num_b, nq, nkv] uint8: 0 skip, 1 partial, 2 full
    kv_num_blocks: torch.Tensor       # [num_b, nq] int32
    kv_indices: torch.Tensor          # [num_b, nq, nkv]
    full_kv_num_blocks: torch.Tensor
    full_kv_indices: torch.Tensor
    q_num_blocks: torch.Tensor        # [num_b, nkv]
    q_indices: torch.Tensor           # [num_b, nkv, nq]
    full_q_num_blocks: torch.Tensor
    full_q_indices: torch.Tensor

    def to_c(self) -> L.FaBlockTables:
        t = L.FaBlockTables()
        t.block_q, t.block_kv, t.nq, t.nkv = self.block_q, self.block_kv, self.nq, self.nkv
        t.num_b, t.num_h = self.num_b, 1
        t.kv_num_blocks = self.kv_num_blocks.data_ptr()
        t.kv_indices = self.kv_indices.data_ptr()
        t.full_kv_num_blocks = self.full_kv_num_blocks.data_ptr()
        t.full_kv_indices = self.full_kv_indices.data_ptr()
        t.kv_cap = self.nkv
        t.q_num_blocks = self.q_num_blocks.data_ptr()
        t.q_indices = self.q_indices.data_ptr()
        t.full_q_num_blocks = self.full_q_num_blocks.data_ptr()
        t.full_q_indices = self.full_q_indices.data_ptr()
        t.q_cap = self.nq
        return t

    def unmasked_tiles(self) -> tuple[int, int]:
        """(partial, full) tile counts summed over batch rows (one host sync)."""
        return int(self.kv_num_blocks.sum()), int(self.full_kv_num_blocks.sum())


def _alloc_tables(num_b: int, nq: int, nkv: int, bq: int, bkv: int, device) -> tuple[BlockTables, L.FaBlockMaskOut]:
    i32 = dict(dtype=torch.int32, device=device)
    bt = BlockTables(
        block_q=bq, block_kv=bkv, nq=nq, nkv=nkv, num_b=num_b,
        tile_class=torch.empty((num_b, nq, nkv), dtype=torch.uint8, device=device),
        kv_num_blocks=torch.empty((num_b, nq), **i32),
        kv_indices=torch.empty((num_b, nq, nkv), **i32),
        full_kv_num_blocks=torch.empty((num_b, nq), **i32),
        full_kv_indices=torch.empty((num_b, nq, nkv), **i32),
        q_num_blocks=torch.empty((num_b, nkv), **i32),
        q_indices=torch.empty((num_b, nkv, nq), **i32),
        full_q_num_blocks=torch.empty((num_b, nkv), **i32),
        full_q_indices=torch.empty((num_b, nkv, nq), **i32),
    )
    out = L.FaBlockMaskOut()
    out.num_b, out.nq, out.nkv = num_b, nq, nkv
    for name in ("tile_class", "kv_num_blocks", "kv_indices", "full_kv_num_blocks", "full_kv_indices",
                 "q_num_blocks", "q_indices", "full_q_num_blocks", "full_q_indices"):
        setattr(out, name, getattr(bt, name).data_ptr())
    return bt, out


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def build_tables_from_spec(spec: MaskSpec, B: int, Tq: int, Tkv: int, block_q: int, block_kv: int,
                           device, mode: int = L.FA_BLOCK_MASK_EXACT, offsets: tuple = (0, 0)) -> BlockTables:
    """Classify every tile of the mask on the GPU and build all tables.  `offsets` are the
    global positions of the first query and key (a block of a longer sequence)."""
    device = torch.device(device)
    nq, nkv = math.ceil(Tq / block_q), math.ceil(Tkv / block_kv)
    num_b = B if spec.depends_on_batch else 1
    bt, out = _alloc_tables(num_b, nq, nkv, block_q, block_kv, device)
    m = spec.to_c(device, Tq, Tkv, *offsets)
    with torch.cuda.device(device):
        L.check(L.lib().fa_create_block_mask(C.byref(m), B, Tq, Tkv, block_q, block_kv, mode, C.byref(out),
                                             _stream(device)))
    return bt


def build_tables_from_lists(kv_num_blocks: torch.Tensor, kv_indices: torch.Tensor, block_q: int, block_kv: int,
                            nkv: int, full_kv_num_blocks: Optional[torch.Tensor] = None,
                            full_kv_indices: Optional[torch.Tensor] = None, device=None) -> BlockTables:
    """Tables (including the transpose) from reference-style row lists ([nq] / [nq, cap])."""
    device = torch.device(device if device is not None else "cuda")
    i32 = dict(dtype=torch.int32, device=device)
    num = kv_num_blocks.to(**i32).reshape(-1, kv_num_blocks.shape[-1]).contiguous()
    num_b, nq = num.shape
    idx = kv_indices.to(**i32).reshape(num_b, nq, -1).contiguous()
    cap = max(idx.shape[-1], 1)
    if idx.shape[-1] == 0:
        idx = torch.full((num_b, nq, 1), -1, **i32)
    fnum = fidx = None
    if full_kv_num_blocks is not None:
        fnum = full_kv_num_blocks.to(**i32).reshape(num_b, nq).contiguous()
        fidx = full_kv_indices.to(**i32).reshape(num_b, nq, -1).contiguous()
        if fidx.shape[-1] != cap:
            pad = torch.full((num_b, nq, cap), -1, **i32)
            pad[..., : min(cap, fidx.shape[-1])] = fidx[..., :cap]
            fidx = pad
    bt, out = _alloc_tables(num_b, nq, nkv, block_q, block_kv, device)
    with torch.cuda.device(device):
        L.check(L.lib().fa_block_tables_from_lists(
            num_b, nq, nkv, num.data_ptr(), idx.data_ptr(),
            fnum.data_ptr() if fnum is not None else None, fidx.data_ptr() if fidx is not None else None,
            cap, C.byref(out), _stream(device)))
    return bt


@dataclass(frozen=True, eq=False)
class BlockMask:
    """Block-sparse mask data structure (reference block_mask.py:16-51).

    Attributes:
        num_blocks_in_row: (Q_BLOCKS,) int32 count of valid KV blocks per query block
        col_indices: (Q_BLOCKS, max_blocks_per_row) int32 KV block indices, padded with -1
        block_size: block size (same for Q and KV)
        q_len, kv_len: sequence lengths
        tables: engine tables (partial/full lists and their transpose), or None
        mask_mod: the mask_mod the tables were built from, if any
    """

    num_blocks_in_row: torch.Tensor
    col_indices: torch.Tensor
    block_size: int
    q_len: int
    kv_len: int
    tables: Optional[BlockTables] = None
    mask_mod: Optional[MaskMod] = None
    _dev: dict = field(default_factory=dict, repr=False, compare=False)

    @property
    def num_q_blocks(self) -> int:
        return int(math.ceil(self.q_len / self.block_size))

    @property
    def num_kv_blocks(self) -> int:
        return int(math.ceil(self.kv_len / self.block_size))

    @property
    def sparsity(self) -> float:
        """Sparsity ratio (0 = dense, 1 = fully sparse)."""
        total_possible = self.num_q_blocks * self.num_kv_blocks
        actual_blocks = int(self.num_blocks_in_row.sum())
        return 1.0 - (float(actual_blocks) / total_possible)

    def device_tables(self, device) -> BlockTables:
        """Engine tables on `device`; built from the reference fields when absent."""
        device = torch.device(device)
        if self.tables is not None and self.tables.tile_class.device == device:
            return self.tables
        k = str(device)
        if k not in self._dev:
            self._dev[k] = build_tables_from_lists(self.num_blocks_in_row, self.col_indices, self.block_size,
                                                   self.block_size, self.num_kv_blocks, device=device)
        return self._dev[k]


def create_block_mask(mask_mod: MaskMod, B: int, H: int, Q_LEN: int, KV_LEN: int, block_size: int = 128, *,
                      device=None) -> BlockMask:
    """Create a BlockMask from a mask_mod (reference block_mask.py:54-129).

    ``num_blocks_in_row`` / ``col_indices`` follow the reference's 3x3 sampling
    rule exactly, for registry masks and arbitrary callables alike (a callable is
    first evaluated on the GPU into per-tile bitmasks, which the classifier reads).  ``tables`` hold the exact classification (a tile is listed iff
    any element is unmasked, and marked full iff all are), which the attention
    kernels use.  B and H do not change the result, as in the reference; a
    document mask with per-batch ids yields per-batch tables and batch 0's
    reference fields.
    """
    del H
    if device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("create_block_mask runs on the GPU; no CUDA device is available")
        device = torch.device("cuda", torch.cuda.current_device())
    spec = spec_of(mask_mod)
    if spec is None:  # an arbitrary callable: evaluated on the GPU into per-tile bitmasks first
        spec = evaluate_mask(mask_mod, Q_LEN, KV_LEN, device)
    ref = build_tables_from_spec(spec, B, Q_LEN, KV_LEN, block_size, block_size, device, L.FA_BLOCK_MASK_REF9)
    exact = build_tables_from_spec(spec, B, Q_LEN, KV_LEN, block_size, block_size, device, L.FA_BLOCK_MASK_EXACT)
    counts = ref.kv_num_blocks[0].contiguous()
    max_row = int(counts.max()) if counts.numel() else 0
    cols = ref.kv_indices[0, :, :max_row].contiguous()
    return BlockMask(counts, cols, block_size, Q_LEN, KV_LEN, exact, mask_mod)


def _padded(rows: list[list[int]]) -> tuple[torch.Tensor, torch.Tensor]:
    counts = [len(r) for r in rows]
    max_row = max(counts) if counts else 0
    cols = [r + [-1] * (max_row - len(r)) for r in rows]
    return torch.tensor(counts, dtype=torch.int32), torch.tensor(cols, dtype=torch.int32).reshape(len(rows), max_row)


def create_causal_block_mask(seq_len: int, block_size: int = 128) -> BlockMask:
    """Causal BlockMask: query block i attends to kv blocks 0..i (block_mask.py:132-172)."""
    n = math.ceil(seq_len / block_size)
    counts, cols = _padded([list(range(i + 1)) for i in range(n)])
    return BlockMask(counts, cols, block_size, seq_len, seq_len)


def create_sliding_window_block_mask(seq_len: int, window_size: int, block_size: int = 128) -> BlockMask:
    """Symmetric sliding-window BlockMask (block_mask.py:175-218)."""
    n = math.ceil(seq_len / block_size)
    w = math.ceil(window_size / block_size)
    counts, cols = _padded([list(range(max(0, i - w), min(n, i + w + 1))) for i in range(n)])
    return BlockMask(counts, cols, block_size, seq_len, seq_len)
