"""Chunked fp32 reference of attention and its gradients on the GPU, for full-length
checks where the numpy oracle would be too slow.  Same formulas as the oracle
(oracle/flexattn_oracle.py: materialised softmax, delta = rowsum(o * dO), dS = P (dP - delta)
times the score_mod's derivative), evaluated in row chunks; tests check it against the oracle.
"""
import math

import torch


def torch_reference(q, k, v, do, mask_fn, score_fn=None, chunk=1024):
    """Chunked fp32 reference on the GPU: o, lse, dq, dk, dv with the oracle's formulas."""
    B, H, T, D = q.shape
    s = 1.0 / math.sqrt(D)
    qf, kf, vf, dof = (t.float() for t in (q, k, v, do))
    o = torch.empty_like(qf)
    lse = torch.empty(q.shape[:3], device=q.device)
    kvi = torch.arange(k.shape[2], device=q.device)[None, :]
    hi = torch.arange(H, device=q.device)[None, :, None, None]

    def scores(r0, r1):
        raw = torch.einsum("bhqd,bhkd->bhqk", qf[:, :, r0:r1], kf) * s
        qi = torch.arange(r0, r1, device=q.device)[:, None]
        x, g = raw, torch.ones_like(raw)
        if score_fn is not None:
            x, g = score_fn(raw, hi, qi, kvi)
        m = mask_fn(qi, kvi) if mask_fn is not None else torch.ones_like(x, dtype=torch.bool)
        return torch.where(m, x, torch.tensor(-math.inf, device=q.device)), g

    for r0 in range(0, T, chunk):
        x, _ = scores(r0, min(r0 + chunk, T))
        l = torch.logsumexp(x, -1)
        p = torch.exp(x - l[..., None]).nan_to_num(0.0)
        o[:, :, r0:r0 + chunk] = p @ vf
        lse[:, :, r0:r0 + chunk] = l
    delta = (o * dof).sum(-1)
    dq, dk, dv = torch.zeros_like(qf), torch.zeros_like(kf), torch.zeros_like(vf)
    for r0 in range(0, T, chunk):
        r1 = min(r0 + chunk, T)
        x, g = scores(r0, r1)
        p = torch.exp(x - lse[:, :, r0:r1, None]).nan_to_num(0.0)
        dp = dof[:, :, r0:r1] @ vf.transpose(-1, -2)
        ds = p * (dp - delta[:, :, r0:r1, None]) * g
        dv += p.transpose(-1, -2) @ dof[:, :, r0:r1]
        dk += ds.transpose(-1, -2) @ qf[:, :, r0:r1] * s
        dq[:, :, r0:r1] = ds @ kf * s
    return o, lse, dq, dk, dv
