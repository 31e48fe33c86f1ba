"""Context-parallel (ring) attention for long sequences: forward, backward and autograd.

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

The backward (``ring_attention_bwd``) walks the same ring.  Each rank keeps its Q,
O, dO and the final logsumexp rows and accumulates dQ locally in fp32; the K/V
blocks travel as in the forward, and with each block travel its fp32 dK/dV
accumulators.  At step s a rank adds the contributions of its Q chunks to the
held block (one fused backward call per unmasked chunk pair, the mask and score
mods at global positions, P recomputed from the final logsumexp) into a local
buffer, adds the accumulators that arrive from the previous rank, and sends the
sum on to the next rank; after the last step the accumulators have gone round
the ring once and arrive back at the block's owner.  The accumulator exchange of
step s overlaps the compute of step s+1.

On GPUs the exchange is NCCL send/recv through ``torch.distributed`` (NVLink) on
NCCL's own stream, overlapped with the attention kernels on the compute stream.
The partial-attention, partial-gradient and merge functions are injectable so the
same schedule runs on CPU ranks (gloo) in tests.
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


_PLANS: dict = {}


def _pair_plan(q, k, v, mask_mod, score_mod, q_offset: int, kv_offset: int, need_bwd: bool):
    """The plan of one (q chunk, K/V chunk) pair, kept across ring steps and calls: a ring
    revisits the same few geometries every step, and building a plan is host work on the
    critical path of short chunks.  The key holds everything a plan depends on (shapes,
    strides, 16-byte alignment, dtype, device, the mods, the offsets); the entry keeps the mod
    objects alive so that their ids are not reused by others."""
    from .flash_attn import _Plan

    key = (tuple(q.shape), tuple(k.shape), q.stride(), k.stride(), v.stride(),
           tuple(t.data_ptr() & 15 for t in (q, k, v)), q.dtype, q.device, id(mask_mod), id(score_mod),
           q_offset, kv_offset, need_bwd)
    hit = _PLANS.get(key)
    if hit is not None and hit[1] is mask_mod and hit[2] is score_mod:
        return hit[0]
    if len(_PLANS) > 256:
        _PLANS.clear()
    plan = _Plan(q, k, v, mask_mod, score_mod, None, 64, 64, 0, None, need_bwd=need_bwd,
                 offsets=(q_offset, kv_offset))
    _PLANS[key] = (plan, mask_mod, score_mod)
    return plan


def gpu_partial_attention(q, k, v, mask_mod, score_mod, q_offset: int, kv_offset: int):
    """(o, lse) of q against one K/V chunk with global-position masks, on the tcgen05 kernel."""
    from .flash_attn import _run_fwd

    return _run_fwd(_pair_plan(q, k, v, mask_mod, score_mod, q_offset, kv_offset, False), q, k, v)


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
    # The caller's k/v are only read (sent at step 0); received blocks alternate between two
    # buffers of the ring's own, so no receive ever writes a caller tensor.
    cur_k, cur_v = k.contiguous(), v.contiguous()
    bufs = [(torch.empty_like(cur_k), torch.empty_like(cur_v)) for _ in range(2 if world > 2 else 1)]
    nxt_rank, prv_rank = (rank + 1) % world, (rank - 1) % world
    g = dist.get_global_rank(group, nxt_rank) if group is not None else nxt_rank
    gp = dist.get_global_rank(group, prv_rank) if group is not None else prv_rank
    for s in range(world):
        works = []
        if s + 1 < world:
            nxt_k, nxt_v = bufs[s % len(bufs)]
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
            cur_k, cur_v = nxt_k, nxt_v
        if stats:
            stats.steps += 1
    return torch.cat(o_acc, dim=2).to(q.dtype), torch.cat(lse_acc, dim=2)


def gpu_partial_attention_bwd(q, k, v, o, lse, do, mask_mod, score_mod, q_offset: int, kv_offset: int):
    """(dq, dk, dv) contributions of one (q chunk, K/V chunk) pair, on the fused tcgen05
    backward: P is recomputed from the final logsumexp `lse` and delta from the final `o`."""
    from .flash_attn import _run_bwd

    return _run_bwd(_pair_plan(q, k, v, mask_mod, score_mod, q_offset, kv_offset, True), q, k, v, o, lse, do)


def ring_attention_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, lse: torch.Tensor,
                       do: torch.Tensor, mask_mod=None, score_mod=None, *, group=None,
                       attn_bwd_fn: Optional[Callable] = None, pair_is_empty: Optional[Callable] = None,
                       stats: Optional[RingStats] = None):
    """Gradients of ring attention over the process group.  q, k, v, o and do hold this rank's
    zig-zag share ([B, H(_kv), 2C, D]), lse its fp32 logsumexp rows ([B, H, 2C]), both from
    ring_attention_fwd.  Returns (dq, dk, dv) for the rank's share, in the input dtypes."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    attn_bwd_fn = attn_bwd_fn or gpu_partial_attention_bwd
    pair_is_empty = pair_is_empty or _default_pair_is_empty
    B, H, T2, D = q.shape
    Cl = T2 // 2
    if 2 * Cl != T2 or k.shape[2] != T2 or tuple(o.shape) != tuple(q.shape) or tuple(do.shape) != tuple(q.shape):
        raise ValueError("q/k/v/o/do must hold two equal chunks")
    my = zigzag_chunks(rank, world)
    halves = lambda x: (x[:, :, :Cl], x[:, :, Cl:])  # noqa: E731
    q_p, o_p, do_p = halves(q), halves(o), halves(do)
    lse = lse.to(torch.float32)
    l_p = (lse[:, :, :Cl], lse[:, :, Cl:])
    dq_acc = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    cur_k, cur_v = k.contiguous(), v.contiguous()  # read only; received blocks go to the ring's buffers
    bufs = [(torch.empty_like(cur_k), torch.empty_like(cur_v)) for _ in range(2 if world > 2 else 1)]
    nxt_rank, prv_rank = (rank + 1) % world, (rank - 1) % world
    g = dist.get_global_rank(group, nxt_rank) if group is not None else nxt_rank
    gp = dist.get_global_rank(group, prv_rank) if group is not None else prv_rank
    acc_works, acc_send, acc_recv = [], None, None
    for s in range(world):
        kv_works = []
        if s + 1 < world:
            nxt_k, nxt_v = bufs[s % len(bufs)]
            ops = [dist.P2POp(dist.isend, cur_k, g, group), dist.P2POp(dist.isend, cur_v, g, group),
                   dist.P2POp(dist.irecv, nxt_k, gp, group), dist.P2POp(dist.irecv, nxt_v, gp, group)]
            kv_works = dist.batch_isend_irecv(ops)
        held = zigzag_chunks((rank - s) % world, world)
        dk_loc = torch.zeros(cur_k.shape, dtype=torch.float32, device=k.device)
        dv_loc = torch.zeros(cur_v.shape, dtype=torch.float32, device=v.device)
        for qi, qc in enumerate(my):
            for ki, kc in enumerate(held):
                q0, k0 = qc * Cl, kc * Cl
                if pair_is_empty(mask_mod, q0, q0 + Cl, k0, k0 + Cl):
                    if stats:
                        stats.pairs_skipped += 1
                    continue
                ks = slice(ki * Cl, (ki + 1) * Cl)
                dq_c, dk_c, dv_c = attn_bwd_fn(q_p[qi], cur_k[:, :, ks], cur_v[:, :, ks], o_p[qi], l_p[qi], do_p[qi],
                                               mask_mod, score_mod, q0, k0)
                # in-place adds cast the bf16 contributions inside the kernel (no fp32 temporaries)
                dq_acc[:, :, qi * Cl:(qi + 1) * Cl].add_(dq_c)
                dk_loc[:, :, ks].add_(dk_c)
                dv_loc[:, :, ks].add_(dv_c)
                if stats:
                    stats.pairs_computed += 1
        if world > 1:
            if s > 0:  # the held block's accumulators, sent on by the previous rank after its step s-1
                for w_ in acc_works:
                    w_.wait()
                dk_loc += acc_recv[0]
                dv_loc += acc_recv[1]
            acc_send = (dk_loc, dv_loc)  # referenced until the sends complete
            acc_recv = (torch.empty_like(dk_loc), torch.empty_like(dv_loc))
            # tag 1 keeps these apart from the K/V messages (tag 0) of the same step on backends
            # that match by tag (gloo); NCCL matches in posting order, which is the same on all ranks
            ops = [dist.P2POp(dist.isend, acc_send[0], g, group, tag=1),
                   dist.P2POp(dist.isend, acc_send[1], g, group, tag=1),
                   dist.P2POp(dist.irecv, acc_recv[0], gp, group, tag=1),
                   dist.P2POp(dist.irecv, acc_recv[1], gp, group, tag=1)]
            acc_works = dist.batch_isend_irecv(ops)
        else:
            acc_recv = (dk_loc, dv_loc)
        for w_ in kv_works:
            w_.wait()
        if s + 1 < world:
            cur_k, cur_v = nxt_k, nxt_v
        if stats:
            stats.steps += 1
    for w_ in acc_works:  # the own block's accumulators, back from the last holder
        w_.wait()
    del acc_send
    return dq_acc.to(q.dtype), acc_recv[0].to(k.dtype), acc_recv[1].to(v.dtype)


class _RingAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, mask_mod, score_mod, group):
        o, lse = ring_attention_fwd(q, k, v, mask_mod, score_mod, group=group)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.cfg = (mask_mod, score_mod, group)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        mask_mod, score_mod, group = ctx.cfg
        dq, dk, dv = ring_attention_bwd(q, k, v, o, lse, do.contiguous(), mask_mod, score_mod, group=group)
        return dq, dk, dv, None, None, None


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask_mod=None, score_mod=None, *,
                   group=None) -> torch.Tensor:
    """Differentiable context-parallel attention: this rank's zig-zag share of the output;
    the backward runs ring_attention_bwd."""
    return _RingAttentionFn.apply(q, k, v, mask_mod, score_mod, group)
