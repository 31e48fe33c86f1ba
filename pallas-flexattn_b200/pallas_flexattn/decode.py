"""Split-KV decode against a K/V cache (libflexattn ``fa_decode``).

The reference package has no decode entry point; this is the serving-side companion of
``flash_attention_fwd``: a few new query tokens per sequence attend to a cache of keys and
values that may be longer than the valid part of each sequence.  Masks and score mods are
the same registry objects the forward pass takes, evaluated at global positions: query row
``i`` of batch ``b`` sits at position ``kv_lens[b] - Tq + i`` and the cache row ``j`` at
position ``j``, so ``causal_mask`` lets each new token see the cache and the new tokens
before it.

The cache is cut into chunks handled by separate CTAs (one per chunk, batch and K/V head,
covering every query head of the group); a second kernel merges the chunks by
log-sum-exp.  bf16 runs on the tensor cores (tcgen05), fp32 on CUDA cores.  There is no
CPU path.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Optional, Sequence, Tuple, Union

import torch

from . import _lib as L
from .flash_attn import _DTYPES, _fa_tensor, _last_contig, device_status
from .mask_mod import MaskMod
from .mask_mod import spec_of as mask_spec_of
from .score_mod import ScoreMod
from .score_mod import spec_of as score_spec_of

MAX_QUERY_ROWS = {"bf16": 128, "fp32": 64}  # (H / H_kv) * Tq per K/V head


def flash_attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           kv_lens: Optional[Union[torch.Tensor, Sequence[int]]] = None,
                           mask_mod: Optional[MaskMod] = None, *, score_mod: Optional[ScoreMod] = None,
                           scale: Optional[float] = None, num_splits: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Attention of ``q`` [B, H, Tq, D] against ``k_cache`` / ``v_cache`` [B, H_kv, Tkv, D].

    ``kv_lens`` ([B] ints, ``Tq <= kv_lens[b] <= Tkv``) gives the valid cache length of each
    sequence; None means all ``Tkv`` rows.  ``mask_mod`` may be None, ``causal_mask``,
    ``sliding_window_mask`` or their ``and_masks``; ``score_mod`` may be ALiBi, softcap or
    both.  ``num_splits`` = 0 picks the chunking from the shape.  Returns ``(o, lse)`` with
    ``o`` like ``q`` and ``lse`` [B, H, Tq] fp32 (natural log); a row with no visible key
    gives ``o = 0`` and ``lse = -inf``.
    """
    if q.dim() != 4 or k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError("q, k_cache, v_cache must be (B, H, T, D)")
    if not (q.is_cuda and k_cache.is_cuda and v_cache.is_cuda):
        raise ValueError("flash_attention_decode runs on CUDA tensors only (there is no CPU path)")
    if q.dtype not in _DTYPES or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise ValueError(f"q/k/v must share dtype bf16 or fp32, got {q.dtype}/{k_cache.dtype}/{v_cache.dtype}")
    B, H, Tq, D = q.shape
    Bk, Hkv, Tkv, Dk = k_cache.shape
    if Bk != B or Dk != D or tuple(v_cache.shape) != (B, Hkv, Tkv, D):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k_cache.shape)} v{tuple(v_cache.shape)}")
    if H % Hkv:
        raise ValueError(f"H={H} must be a multiple of the K/V heads {Hkv}")
    mspec = mask_spec_of(mask_mod)
    if mspec is None or mspec.flags & ~(L.FA_MASK_CAUSAL | L.FA_MASK_WINDOW):
        raise NotImplementedError("decode takes None, causal_mask, sliding_window_mask or their and_masks")
    sspec = score_spec_of(score_mod)
    if sspec is None or sspec.flags & ~(L.FA_SCORE_ALIBI | L.FA_SCORE_SOFTCAP):
        raise NotImplementedError("decode takes alibi_score_mod, softcap_score_mod or their composition")
    dev = q.device
    q, k_cache, v_cache = _last_contig(q), _last_contig(k_cache), _last_contig(v_cache)
    lens = None
    if kv_lens is not None:
        lens = torch.as_tensor(kv_lens, dtype=torch.int32).to(dev).contiguous()
        if lens.shape != (B,):
            raise ValueError(f"kv_lens must have shape ({B},), got {tuple(lens.shape)}")

    o = torch.empty(q.shape, dtype=q.dtype, device=dev)
    lse = torch.empty((B, H, Tq), dtype=torch.float32, device=dev)
    p = L.FaDecodeParams()
    p.dtype = _DTYPES[q.dtype]
    p.B, p.H, p.H_kv, p.Tq, p.Tkv, p.D = B, H, Hkv, Tq, Tkv, D
    p.q, p.k, p.v, p.o = _fa_tensor(q), _fa_tensor(k_cache), _fa_tensor(v_cache), _fa_tensor(o)
    p.lse = lse.data_ptr()
    p.kv_lens = lens.data_ptr() if lens is not None else None
    p.scale = float(scale) if scale is not None else 1.0 / math.sqrt(D)
    p.mask = mspec.to_c(dev, Tq, Tkv)
    p.score = sspec.to_c(dev, H, Tq, Tkv)
    p.num_splits = int(num_splits)
    p.status = device_status(dev).data_ptr()
    lib = L.lib()
    size = C.c_size_t(0)
    L.check(lib.fa_decode_workspace_size(C.byref(p), C.byref(size)))
    ws = torch.empty(size.value, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        L.check(lib.fa_decode(C.byref(p), ws.data_ptr(), size.value, torch.cuda.current_stream(dev).cuda_stream))
    return o, lse
