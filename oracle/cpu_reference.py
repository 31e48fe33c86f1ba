"""Timed CPU restatement of the reference's flash-attention path — TEST/BASELINE ONLY.

Used by bench.py's CPU-baseline leg and ``--impl reference`` arm (and by tests),
never by the product.  The reference (novastar53/pallas-flexattn) runs on CPU
through Pallas interpret mode, which needs jax (not installable here), so this
module restates its kernels with torch CPU fp32 ops, keeping the reference's
work pattern — every KV tile visited, no block skipping:

* ``fwd``  flash_attention_fwd_kernel (src/pallas_flexattn/flash_attn.py:59-108):
  per q tile, online softmax over all kv tiles, O /= l, lse = m + log l;
* ``bwd``  flash_attention_bwd (flash_attn.py:410-461): preprocess delta
  (:168-173), dK/dV kernel looping over all q tiles (:206-253), dQ kernel looping
  over all kv tiles (:313-356) — S and P recomputed in both.
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import torch


def _mask_tile(mask_mod, S, r0, c0):
    if mask_mod is None:
        return S
    qi = torch.arange(r0, r0 + S.shape[0])[:, None]
    ki = torch.arange(c0, c0 + S.shape[1])[None, :]
    return torch.where(mask_mod(qi, ki), S, torch.tensor(float("-inf")))


def _score(S, score_mod, h, r0, c0):
    if score_mod is None:
        return S
    qi = torch.arange(r0, r0 + S.shape[0])[:, None]
    ki = torch.arange(c0, c0 + S.shape[1])[None, :]
    return score_mod(S, 0, torch.tensor(h), qi, ki)


@torch.no_grad()
def fwd(q, k, v, mask_mod: Optional[Callable] = None, score_mod=None, h: int = 0, block_r: int = 64,
        block_c: int = 64):
    """One (T, D) head slice; returns (o, lse)."""
    T, D = q.shape
    scale = 1.0 / math.sqrt(D)
    o = torch.empty_like(q)
    lse = torch.empty(T, dtype=q.dtype)
    for r0 in range(0, T, block_r):
        Q = q[r0:r0 + block_r]
        m = torch.full((Q.shape[0],), float("-inf"))
        l = torch.zeros(Q.shape[0])
        acc = torch.zeros(Q.shape[0], D)
        for c0 in range(0, T, block_c):
            S = (Q @ k[c0:c0 + block_c].T) * scale
            S = _mask_tile(mask_mod, _score(S, score_mod, h, r0, c0), r0, c0)
            mn = torch.maximum(m, S.max(dim=-1).values)
            p = torch.exp(S - mn[:, None]).nan_to_num(0.0)
            alpha = torch.exp(m - mn).nan_to_num(0.0)
            acc = acc * alpha[:, None] + p @ v[c0:c0 + block_c]
            l = l * alpha + p.sum(-1)
            m = mn
        o[r0:r0 + block_r] = acc / l[:, None]
        lse[r0:r0 + block_r] = m + torch.log(l)
    return o, lse


@torch.no_grad()
def bwd(q, k, v, o, lse, do, mask_mod: Optional[Callable] = None, score_mod=None, h: int = 0,
        block_r: int = 64, block_c: int = 64):
    """One head slice; returns (dq, dk, dv) with the reference's three-kernel structure."""
    T, D = q.shape
    scale = 1.0 / math.sqrt(D)
    delta = (o * do).sum(-1)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    for c0 in range(0, T, block_c):  # dK/dV kernel: all q tiles
        K, V = k[c0:c0 + block_c], v[c0:c0 + block_c]
        dk_acc = torch.zeros_like(K)
        dv_acc = torch.zeros_like(V)
        for r0 in range(0, T, block_r):
            Q, dO = q[r0:r0 + block_r], do[r0:r0 + block_r]
            S = _mask_tile(mask_mod, _score((Q @ K.T) * scale, score_mod, h, r0, c0), r0, c0)
            P = torch.exp(S - lse[r0:r0 + block_r, None])
            dP = dO @ V.T
            dS = P * (dP - delta[r0:r0 + block_r, None]) * scale
            dv_acc += P.T @ dO
            dk_acc += dS.T @ Q
        dk[c0:c0 + block_c], dv[c0:c0 + block_c] = dk_acc, dv_acc
    dq = torch.empty_like(q)
    for r0 in range(0, T, block_r):  # dQ kernel: all kv tiles
        Q, dO = q[r0:r0 + block_r], do[r0:r0 + block_r]
        dq_acc = torch.zeros_like(Q)
        for c0 in range(0, T, block_c):
            K, V = k[c0:c0 + block_c], v[c0:c0 + block_c]
            S = _mask_tile(mask_mod, _score((Q @ K.T) * scale, score_mod, h, r0, c0), r0, c0)
            P = torch.exp(S - lse[r0:r0 + block_r, None])
            dS = P * ((dO @ V.T) - delta[r0:r0 + block_r, None]) * scale
            dq_acc += dS @ K
        dq[r0:r0 + block_r] = dq_acc
    return dq, dk, dv
