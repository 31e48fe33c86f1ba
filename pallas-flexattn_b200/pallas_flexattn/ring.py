"""Context-parallel (ring) attention forward for long sequences.

The sequence is cut into 2·W chunks of equal length (W = world size) and rank r
owns chunks r and 2W-1-r ("zig-zag", which balances causal work across ranks).
Each rank keeps its Q chunks and passes its K/V chunks around the ring:

    step s = 0 .. W-1:  hold the K/V of rank (r - s) mod W
                        send it to rank r+1, receive the next from rank r-1  (async P2P)
                        meanwhile, attend each own Q chunk to each held K/V chunk
                        whose (q, kv) window is not fully masked, with the mask and
                        score mods evaluated at global positions (FaMaskSpec offsets)
                        and merge the partial (o, lse) into fp32 accumulators
                        (log-sum-exp combine, ``fa_lse_merge``)

On GPUs the exchange is NCCL send/recv through ``torch.distributed`` (NVLink) on
NCCL's own stream, overlapped with the attention kernels on the compute stream.
The partial-attention and merge functions are injectable so the same schedule
runs on CPU ranks (gloo) in tests.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch

from . import _lib as L


def zigzag_chunks(rank: int, world: int) -> tuple[int, int]:
    """The two sequence chunks (of 2·world) rank `rank` owns."""
    return rank, 2 * world - 1 - rank


def split_zigzag(x: torch.Tensor, rank: int, world: int, dim: int = 2) -> torch.Tensor:
    """Rank `rank`'s zig-zag share of a full-sequence tensor (concatenation of its two chunks)."""
    chunks = x.chunk(2 * world, dim=dim)
    a, b = zigzag_chunks(rank, world)
    return torch.cat([chunks[a], chunks[b]], dim=dim)


def gather_zigzag(parts: list[torch.Tensor], world: int, dim: int = 2) -> torch.Tensor:
    """Inverse of split_zigzag over all ranks' parts."""
    out = [None] * (2 * world)
    for r, p in enumerate(parts):
        x, y = p.chunk(2, dim=dim)
        a, b = zigzag_chunks(r, world)
        out[a], out[b] = x, y
    return torch.cat(out, dim=dim)


@dataclass
class RingStats:
    steps: int = 0
    pairs_computed: int = 0
    pairs_skipped: int = 0


def _default_pair_is_empty(mask_mod, q0: int, q1: int, k0: int, k1: int) -> bool:
    """Cheap emptiness test for the (q, kv) window: exact for causal/window masks via the spec."""
    from .mask_mod import spec_of

    s = spec_of(mask_mod)
    if s is None:
        return False
    if s.flags & L.FA_MASK_CAUSAL and k0 > q1 - 1:
        return True
    if s.flags & L.FA_MASK_WINDOW:
        if s.window_left >= 0 and (q0 - (k1 - 1)) > s.window_left:
            return True
        if s.window_right >= 0 and (k0 - (q1 - 1)) > s.window_right:
            return True
    return False


def gpu_partial_attention(q, k, v, mask_mod, score_mod, q_offset: int, kv_offset: int):
    """(o, lse) of q against one K/V chunk with global-position masks, on the tcgen05 kernel."""
    from .flash_attn import _Plan, _run_fwd

    plan = _Plan(q, k, v, mask_mod, score_mod, None, 64, 64, 0, None, need_bwd=False,
                 offsets=(q_offset, kv_offset))
    return _run_fwd(plan, q, k, v)


def gpu_merge(o_acc: torch.Tensor, lse_acc: torch.Tensor, o_part: torch.Tensor, lse_part: torch.Tensor) -> None:
    """In-place log-sum-exp combine on the GPU (fa_lse_merge)."""
    D = o_acc.shape[-1]
    rows = o_acc.numel() // D
    op = o_part.reshape(rows, D)
    dt = L.FA_DTYPE_BF16 if op.dtype == torch.bfloat16 else L.FA_DTYPE_F32
    L.check(L.lib().fa_lse_merge(rows, D, o_acc.data_ptr(), lse_acc.data_ptr(), op.data_ptr(), op.stride(0), dt,
                                 lse_part.contiguous().data_ptr(), torch.cuda.current_stream(o_acc.device).cuda_stream))


def torch_merge(o_acc: torch.Tensor, lse_acc: torch.Tensor, o_part: torch.Tensor, lse_part: torch.Tensor) -> None:
    """The same combine in torch (CPU ranks)."""
    mx = torch.maximum(lse_acc, lse_part)
    safe = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    wa = torch.where(torch.isfinite(lse_acc), torch.exp(lse_acc - safe), torch.zeros_like(mx))
    wb = torch.where(torch.isfinite(lse_part), torch.exp(lse_part - safe), torch.zeros_like(mx))
    tot = wa + wb
    live = tot > 0
    o_new = (o_acc * wa[..., None] + o_part.float() * wb[..., None]) / torch.where(live, tot, 1.0)[..., None]
    o_acc.copy_(torch.where(live[..., None], o_new, o_acc))
    lse_acc.copy_(torch.where(live, safe + torch.log(torch.where(live, tot, 1.0)), lse_acc))


def ring_attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask_mod=None, score_mod=None, *,
                       group=None, attn_fn: Optional[Callable] = None, merge_fn: Optional[Callable] = None,
                       pair_is_empty: Optional[Callable] = None, stats: Optional[RingStats] = None):
    """Ring attention over the process group; q/k/v hold this rank's zig-zag share
    ([B, H, 2C, D], chunks (r, 2W-1-r) concatenated).  Returns (o, lse) for the
    rank's rows, o in q's dtype, lse fp32."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    attn_fn = attn_fn or gpu_partial_attention
    merge_fn = merge_fn or gpu_merge
    pair_is_empty = pair_is_empty or _default_pair_is_empty
    B, H, T2, D = q.shape
    Cl = T2 // 2
    if 2 * Cl != T2 or k.shape[2] != T2:
        raise ValueError("q/k/v must hold two equal chunks")
    my = zigzag_chunks(rank, world)
    q_parts = (q[:, :, :Cl], q[:, :, Cl:])
    o_acc = [torch.zeros((B, H, Cl, D), dtype=torch.float32, device=q.device) for _ in range(2)]
    lse_acc = [torch.full((B, H, Cl), -math.inf, dtype=torch.float32, device=q.device) for _ in range(2)]
    cur_k, cur_v = k.contiguous(), v.contiguous()
    nxt_k, nxt_v = torch.empty_like(cur_k), torch.empty_like(cur_v)
    nxt_rank, prv_rank = (rank + 1) % world, (rank - 1) % world
    g = dist.get_global_rank(group, nxt_rank) if group is not None else nxt_rank
    gp = dist.get_global_rank(group, prv_rank) if group is not None else prv_rank
    for s in range(world):
        works = []
        if s + 1 < world:
            ops = [dist.P2POp(dist.isend, cur_k, g, group), dist.P2POp(dist.isend, cur_v, g, group),
                   dist.P2POp(dist.irecv, nxt_k, gp, group), dist.P2POp(dist.irecv, nxt_v, gp, group)]
            works = dist.batch_isend_irecv(ops)
        holder = (rank - s) % world
        held = zigzag_chunks(holder, world)
        for qi, qc in enumerate(my):
            for ki, kc in enumerate(held):
                q0, k0 = qc * Cl, kc * Cl
                if pair_is_empty(mask_mod, q0, q0 + Cl, k0, k0 + Cl):
                    if stats:
                        stats.pairs_skipped += 1
                    continue
                kk = cur_k[:, :, ki * Cl:(ki + 1) * Cl]
                vv = cur_v[:, :, ki * Cl:(ki + 1) * Cl]
                o_p, lse_p = attn_fn(q_parts[qi], kk, vv, mask_mod, score_mod, q0, k0)
                merge_fn(o_acc[qi], lse_acc[qi], o_p, lse_p)
                if stats:
                    stats.pairs_computed += 1
        for w_ in works:
            w_.wait()
        if s + 1 < world:
            cur_k, nxt_k = nxt_k, cur_k
            cur_v, nxt_v = nxt_v, cur_v
        if stats:
            stats.steps += 1
    return torch.cat(o_acc, dim=2).to(q.dtype), torch.cat(lse_acc, dim=2)
