"""Mask modification functions (reference: src/pallas_flexattn/mask_mod.py).

A mask_mod is a boolean function of ``(q_idx, kv_idx)`` index arrays (torch
tensors or numpy arrays) that is True where attention is allowed — the same
contract as the reference's ``MaskMod``.  Each mask_mod built here also carries
a ``MaskSpec`` (attribute ``__fa_spec__``): its entry in the compiled functor
registry of libflexattn, which the CUDA kernels evaluate in registers.  Specs
compose with ``and_masks``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import numpy as np
import torch

from . import _lib as L

MaskMod = Callable[[Any, Any], Any]


def _true_like(x):
    if isinstance(x, torch.Tensor):
        return torch.ones_like(x, dtype=torch.bool)
    return np.ones_like(x, dtype=np.bool_)


@dataclass(frozen=True, eq=False)
class MaskSpec:
    """Registry description of a mask: the AND of the enabled predicates."""

    flags: int = 0
    window_left: int = -1
    window_right: int = -1
    doc_ids: Optional[torch.Tensor] = None     # [T] or [B, T] int32
    doc_sorted: bool = False                   # ids non-decreasing along T (contiguous documents)
    tile_table: Optional[torch.Tensor] = None  # [rows, cols] uint8, nonzero = keep
    table_block: int = 0
    bit_index: Optional[torch.Tensor] = None   # BITMASK: [ceil(Tq/128), ceil(Tkv/128)] int32 (device)
    bits: Optional[torch.Tensor] = None        # BITMASK: [slots, 128, 4] int32 words (device)
    _dev: dict = field(default_factory=dict, repr=False, compare=False)

    def key(self) -> tuple:
        return (
            self.flags,
            self.window_left,
            self.window_right,
            None if self.doc_ids is None else id(self.doc_ids),
            None if self.tile_table is None else id(self.tile_table),
            self.table_block,
            None if self.bits is None else id(self.bits),
        )

    @property
    def depends_on_batch(self) -> bool:
        return self.doc_ids is not None and self.doc_ids.dim() == 2 and self.doc_ids.shape[0] > 1

    def device_tensors(self, device: torch.device) -> dict:
        """Copies of the auxiliary arrays on `device` (cached per device)."""
        k = str(device)
        if k not in self._dev:
            d = {}
            if self.doc_ids is not None:
                d["doc"] = self.doc_ids.to(device=device, dtype=torch.int32).contiguous()
            if self.tile_table is not None:
                d["table"] = self.tile_table.to(device=device, dtype=torch.uint8).contiguous()
            self._dev[k] = d
        return self._dev[k]

    def to_c(self, device: torch.device, Tq: int, Tkv: int, q_offset: int = 0, kv_offset: int = 0) -> L.FaMaskSpec:
        m = L.FaMaskSpec()
        m.flags = self.flags
        m.window_left = self.window_left
        m.window_right = self.window_right
        m.q_offset, m.kv_offset = int(q_offset), int(kv_offset)
        dev = self.device_tensors(device)
        if self.flags & L.FA_MASK_DOCUMENT:
            doc = dev["doc"]
            T = doc.shape[-1]
            if T < max(q_offset + Tq, kv_offset + Tkv):
                raise ValueError(f"document ids cover {T} positions, attention needs "
                                 f"{max(q_offset + Tq, kv_offset + Tkv)}")
            m.doc_q = doc.data_ptr()
            m.doc_kv = doc.data_ptr()
            m.doc_stride_b = T if (doc.dim() == 2 and doc.shape[0] > 1) else 0
            if self.doc_sorted:
                m.flags |= L.FA_MASK_DOC_SORTED
        if self.flags & L.FA_MASK_TILE_TABLE:
            t = dev["table"]
            m.tile_table = t.data_ptr()
            m.table_rows, m.table_cols = t.shape
            m.table_block = self.table_block
        if self.flags & L.FA_MASK_BITMASK:
            if self.bit_index.device != device:
                raise ValueError("a mask_mod evaluated on one device cannot run on another")
            m.bit_index, m.bits = self.bit_index.data_ptr(), self.bits.data_ptr()
            m.bit_rows, m.bit_cols = self.bit_index.shape
        return m


BIT_TILE = 128  # tile edge of the evaluated bitmask of an arbitrary mask_mod
_CALLABLE_SPECS: dict = {}
_CALLABLE_SPECS_MAX = 32


def _pack_bits(tiles: torch.Tensor) -> torch.Tensor:
    """[n, 128, 128] bool -> [n, 128, 4] int32 words (bit j of word w = column 32 w + j)."""
    n = tiles.shape[0]
    w = tiles.reshape(n, BIT_TILE, 4, 32).to(torch.int64)
    words = (w << torch.arange(32, device=tiles.device, dtype=torch.int64)).sum(-1)
    return (words - ((words >> 31) << 32)).to(torch.int32)  # two's complement view of the uint32


def evaluate_mask(mask_mod: MaskMod, Tq: int, Tkv: int, device, q_offset: int = 0, kv_offset: int = 0,
                  rows_per_chunk: int = 1024) -> MaskSpec:
    """Evaluate an arbitrary mask_mod (a callable of index tensors, no registry entry) on the
    GPU over the whole (Tq, Tkv) grid at global positions (q + q_offset, kv + kv_offset),
    in chunks of rows, into 128 x 128 tiles: each tile is classified fully masked, fully
    allowed or mixed, and mixed tiles keep their predicate as 128 x 128 bits.  The result is
    a BITMASK spec the kernels (and the block-table builder) test per element.  Cached per
    (callable, geometry, device) while the callable is alive."""
    device = torch.device(device)
    key = (id(mask_mod), Tq, Tkv, q_offset, kv_offset, str(device))
    hit = _CALLABLE_SPECS.get(key)
    if hit is not None and hit[0] is mask_mod:
        return hit[1]
    nbq, nbk = -(-Tq // BIT_TILE), -(-Tkv // BIT_TILE)
    index = torch.empty((nbq, nbk), dtype=torch.int32, device=device)
    slots = []
    n_slots = 0
    ki = torch.arange(nbk * BIT_TILE, device=device)
    kvalid = ki < Tkv
    step = max(BIT_TILE, rows_per_chunk // BIT_TILE * BIT_TILE)
    for r0 in range(0, nbq * BIT_TILE, step):
        r1 = min(r0 + step, nbq * BIT_TILE)
        qi = torch.arange(r0, r1, device=device)
        m = mask_mod((qi + q_offset)[:, None], (ki + kv_offset)[None, :])
        m = torch.as_tensor(m, device=device)
        m = torch.broadcast_to(m, (r1 - r0, nbk * BIT_TILE)).to(torch.bool)
        valid = (qi < Tq)[:, None] & kvalid[None, :]
        allowed = m & valid
        nr = (r1 - r0) // BIT_TILE
        tiles = allowed.reshape(nr, BIT_TILE, nbk, BIT_TILE).permute(0, 2, 1, 3)  # [nr, nbk, 128, 128]
        any_ = tiles.any(dim=(2, 3))
        all_ = (m | ~valid).reshape(nr, BIT_TILE, nbk, BIT_TILE).all(dim=3).all(dim=1)  # padding counts as allowed
        cls = torch.where(any_ & all_, -2, -1).to(torch.int32)
        mixed = any_ & ~all_
        nm = int(mixed.sum())
        if nm:
            cls[mixed] = torch.arange(n_slots, n_slots + nm, device=device, dtype=torch.int32)
            slots.append(_pack_bits(tiles[mixed]))
            n_slots += nm
        index[r0 // BIT_TILE:r1 // BIT_TILE] = cls
    bits = torch.cat(slots) if slots else torch.zeros((1, BIT_TILE, 4), dtype=torch.int32, device=device)
    spec = MaskSpec(flags=L.FA_MASK_BITMASK, bit_index=index.contiguous(), bits=bits.contiguous())
    _CALLABLE_SPECS[key] = (mask_mod, spec)
    while len(_CALLABLE_SPECS) > _CALLABLE_SPECS_MAX:
        _CALLABLE_SPECS.pop(next(iter(_CALLABLE_SPECS)))
    return spec


def spec_of(mask_mod: Optional[MaskMod]) -> Optional[MaskSpec]:
    """The registry spec of a mask_mod (an all-True spec for None), or None if unknown."""
    if mask_mod is None:
        return MaskSpec()
    return getattr(mask_mod, "__fa_spec__", None)


def _with_spec(fn, spec: MaskSpec):
    fn.__fa_spec__ = spec
    return fn


def causal_mask(q_idx, kv_idx):
    """Causal mask - query can only attend to keys at same or earlier positions."""
    return q_idx >= kv_idx


causal_mask.__fa_spec__ = MaskSpec(flags=L.FA_MASK_CAUSAL)


def bidirectional_mask(q_idx, kv_idx):
    """Full bidirectional attention - all positions can attend to all positions."""
    return _true_like(q_idx >= kv_idx)


bidirectional_mask.__fa_spec__ = MaskSpec()


def sliding_window_mask(left: int, right: int) -> MaskMod:
    """Sliding window: allowed iff ``q - kv <= left`` and ``kv - q <= right``.

    ``-1`` means unlimited on that side (reference mask_mod.py:25-43).
    """
    left, right = int(left), int(right)

    def mask(q_idx, kv_idx):
        delta = q_idx - kv_idx
        m = _true_like(delta)
        if left >= 0:
            m = m & (delta <= left)
        if right >= 0:
            m = m & (-delta <= right)
        return m

    flags = L.FA_MASK_WINDOW if (left >= 0 or right >= 0) else 0
    return _with_spec(mask, MaskSpec(flags=flags, window_left=left, window_right=right))


def document_mask(seq_lengths, block_size: int = 128) -> MaskMod:
    """Block attention across document boundaries of a packed sequence.

    ``seq_lengths`` lists the document lengths in order (or, 2-D, one list per
    batch row, each summing to the same total).  The reference declares this
    function and raises NotImplementedError (mask_mod.py:46-59); here it is the
    predicate ``doc[q_idx] == doc[kv_idx]``.  ``block_size`` is accepted for
    signature compatibility and unused.
    """
    del block_size

    def ids(lens) -> torch.Tensor:
        lens = torch.as_tensor(np.asarray(lens), dtype=torch.int64).reshape(-1)
        return torch.repeat_interleave(torch.arange(lens.numel(), dtype=torch.int32), lens)

    per_row = (isinstance(seq_lengths, (list, tuple)) and len(seq_lengths) > 0
               and np.ndim(seq_lengths[0]) == 1) or (np.ndim(seq_lengths) == 2 if not isinstance(
                   seq_lengths, (list, tuple)) else False)
    if not per_row:
        return document_ids_mask(ids(seq_lengths))
    rows = [ids(r) for r in seq_lengths]  # batch rows may hold different numbers of documents
    if len({r.numel() for r in rows}) != 1:
        raise ValueError("every batch row of seq_lengths must cover the same total length")
    return document_ids_mask(torch.stack(rows))


def document_ids_mask(doc_ids) -> MaskMod:
    """Same-document predicate from explicit per-position document ids ([T] or [B, T])."""
    doc = torch.as_tensor(doc_ids).to(torch.int32)
    doc_np = doc.numpy() if doc.dim() == 1 else None

    def mask(q_idx, kv_idx):
        if doc.dim() != 1:
            raise NotImplementedError("a batch-dependent document mask needs the b index; use mha_reference")
        if isinstance(q_idx, torch.Tensor):
            d = doc.to(q_idx.device)
            return d[q_idx.long()] == d[kv_idx.long()]
        return doc_np[np.asarray(q_idx)] == doc_np[np.asarray(kv_idx)]

    # Contiguous documents (non-decreasing ids) let the kernels use one interval per row.
    doc_sorted = bool((doc[..., 1:] >= doc[..., :-1]).all()) if doc.shape[-1] > 1 else True
    return _with_spec(mask, MaskSpec(flags=L.FA_MASK_DOCUMENT, doc_ids=doc, doc_sorted=doc_sorted))


def tile_mask(table, block_size: int) -> MaskMod:
    """Keep element (q, kv) iff ``table[q // block_size, kv // block_size]`` is nonzero."""
    t = torch.as_tensor(np.asarray(table)).to(torch.uint8)
    t_np = t.numpy()
    bs = int(block_size)

    def mask(q_idx, kv_idx):
        if isinstance(q_idx, torch.Tensor):
            tt = t.to(q_idx.device)
            return tt[(q_idx // bs).long(), (kv_idx // bs).long()] != 0
        return t_np[np.asarray(q_idx) // bs, np.asarray(kv_idx) // bs] != 0

    return _with_spec(mask, MaskSpec(flags=L.FA_MASK_TILE_TABLE, tile_table=t, table_block=bs))


def _and_window(a: int, b: int) -> int:
    if a < 0:
        return b
    if b < 0:
        return a
    return min(a, b)


def and_masks(*mods: MaskMod) -> MaskMod:
    """Conjunction of mask_mods; the result keeps a registry spec when every part has one."""
    specs = [spec_of(m) for m in mods]

    def mask(q_idx, kv_idx):
        out = _true_like(q_idx >= kv_idx)
        for m in mods:
            out = out & m(q_idx, kv_idx)
        return out

    if any(s is None for s in specs):
        return mask
    flags, left, right, doc, table, tblock, doc_sorted = 0, -1, -1, None, None, 0, False
    for s in specs:
        flags |= s.flags
        if s.flags & L.FA_MASK_WINDOW:
            left, right = _and_window(left, s.window_left), _and_window(right, s.window_right)
        if s.doc_ids is not None:
            if doc is not None:
                raise NotImplementedError("and_masks: at most one document mask")
            doc, doc_sorted = s.doc_ids, s.doc_sorted
        if s.tile_table is not None:
            if table is not None:
                raise NotImplementedError("and_masks: at most one tile mask")
            table, tblock = s.tile_table, s.table_block
    return _with_spec(mask, MaskSpec(flags=flags, window_left=left, window_right=right, doc_ids=doc,
                                     doc_sorted=doc_sorted, tile_table=table, table_block=tblock))
