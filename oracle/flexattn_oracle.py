"""CPU oracle for the FlexAttention hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this module, and only as the checker / the timed CPU restatement.  The product
(pallas-flexattn_b200/) never calls it.

It restates, in numpy (float64 by default), the algorithm of
novastar53/pallas-flexattn (paths inside that project):

* ``mha_reference``             flash_attn.py:45-56 (materialised softmax attention),
                                extended with FlexAttention's score_mod, applied to the
                                scaled logit before the mask;
* ``decode_reference``          the same formula for the last Tq positions of each
                                sequence against a K/V cache of per-batch length
                                (no counterpart in the reference; checked against
                                mha_reference);
* ``flash_fwd_tiled``           flash_attn.py:59-108 (online-softmax tile recurrence,
                                including its NaN->0 guards at :92 and :96);
* ``attention_bwd``             flash_attn.py:168-173 (delta), :241-245 (dK/dV),
                                :346-349 (dQ), plus d(score_mod)/d(logit);
* ``block_mask_ref9``           block_mask.py:78-129 (3x3 sampling rule, -1 padding);
* ``block_mask_exact``          exact any/all tile classification (engine tables);
* ``causal_block_mask`` / ``sliding_window_block_mask``  block_mask.py:132-218;
* mask predicates               mask_mod.py:15-43.

Parity pin: block-mask and tuner outputs and the reference's own attention
kernels (run in Pallas-interpret emulation) are stored as golden vectors under
tests/golden/ by tests/golden/make_golden.py, which executes the reference
source with a numpy stand-in for jax; tests/test_oracle_golden.py checks this
module against them.
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import numpy as np

# ---------------------------------------------------------------------------- mask predicates
# Each predicate takes broadcastable integer arrays (q_idx, kv_idx) -> bool array.


def causal(q, kv):
    """mask_mod.py:15-17."""
    return q >= kv


def bidirectional(q, kv):
    """mask_mod.py:20-22."""
    return np.ones(np.broadcast(q, kv).shape, dtype=bool)


def sliding_window(left: int, right: int):
    """mask_mod.py:25-43: delta = q - kv; allowed iff delta <= left and -delta <= right (-1 = unlimited)."""

    def f(q, kv):
        d = q - kv
        m = np.ones(np.broadcast(q, kv).shape, dtype=bool)
        if left >= 0:
            m &= d <= left
        if right >= 0:
            m &= -d <= right
        return m

    return f


def document(doc_ids: np.ndarray):
    """Same-document predicate over per-position ids."""
    doc = np.asarray(doc_ids)

    def f(q, kv):
        return doc[q] == doc[kv]

    return f


def tile_table(table: np.ndarray, block: int):
    t = np.asarray(table)

    def f(q, kv):
        return t[q // block, kv // block] != 0

    return f


def and_(*fs):
    def f(q, kv):
        out = np.ones(np.broadcast(q, kv).shape, dtype=bool)
        for g in fs:
            out &= g(q, kv)
        return out

    return f


# ---------------------------------------------------------------------------- score mods
# (s, h, q, kv) -> modified s, on the scaled logit; h broadcast over heads.


def alibi(slopes: np.ndarray):
    sl = np.asarray(slopes, dtype=np.float64)

    def f(s, h, q, kv):
        return s + sl[h] * (kv - q)

    f.grad = None
    return f


def softcap(cap: float):
    def f(s, h, q, kv):
        return cap * np.tanh(s / cap)

    def g(s_raw, h, q, kv):
        t = np.tanh(s_raw / cap)
        return 1.0 - t * t

    f.grad = g
    return f


def alibi_slopes(H: int) -> np.ndarray:
    return np.array([2.0 ** (-8.0 * h / H) for h in range(1, H + 1)])


# ---------------------------------------------------------------------------- attention
def _idx(Tq, Tkv):
    return np.arange(Tq)[:, None], np.arange(Tkv)[None, :]


def logits(q, k, scale=None, score_mods=(), dtype=np.float64):
    """Scaled logits with score mods; returns (raw scaled logits, modified logits)."""
    B, H, Tq, D = q.shape
    Tkv = k.shape[2]
    s = 1.0 / math.sqrt(D) if scale is None else scale
    raw = np.einsum("bhqd,bhkd->bhqk", q.astype(dtype), k.astype(dtype)) * s
    qi, ki = _idx(Tq, Tkv)
    h = np.arange(H)[None, :, None, None]
    x = raw
    for f in score_mods:
        x = f(x, h, qi, ki)
    return raw, x


def mha_reference(q, k, v, mask: Optional[Callable] = None, score_mods=(), scale=None, dtype=np.float64,
                  empty_rows_zero: bool = True):
    """softmax(mask(score(QK^T*scale))) V  (flash_attn.py:45-56).

    With ``empty_rows_zero`` a row whose every key is masked yields 0 and
    lse = -inf (FlexAttention's convention, the engine's); otherwise NaN as the
    reference.  Returns (o, lse).
    """
    Tq, Tkv = q.shape[2], k.shape[2]
    _, x = logits(q, k, scale, score_mods, dtype)
    if mask is not None:
        qi, ki = _idx(Tq, Tkv)
        x = np.where(mask(qi, ki), x, -np.inf)
    m = x.max(axis=-1, keepdims=True)
    empty = ~np.isfinite(m)
    m_safe = np.where(empty, 0.0, m)
    p = np.exp(x - m_safe)
    l = p.sum(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        o = np.einsum("bhqk,bhkd->bhqd", p / l, v.astype(dtype))
        lse = (m_safe + np.log(l))[..., 0]
    if empty_rows_zero:
        o = np.where(empty, 0.0, o)
        lse = np.where(empty[..., 0], -np.inf, lse)
    return o, lse


def decode_reference(q, k, v, kv_lens=None, mask: Optional[Callable] = None, score_mods=(), scale=None,
                     dtype=np.float64):
    """Decode against a K/V cache: q [B, H, Tq, D], k / v [B, H_kv, Tkv, D] with H_kv | H.

    Batch b keeps its first kv_lens[b] cache rows (all Tkv when kv_lens is None); query row i
    sits at global position kv_lens[b] - Tq + i, so it is the last Tq rows of
    mha_reference (flash_attn.py:45-56) over that sequence, with each K/V head shared by
    H / H_kv consecutive query heads.  Rows with no visible key give o = 0, lse = -inf.
    Returns (o, lse).
    """
    B, H, Tq, D = q.shape
    Hkv, Tkv = k.shape[1], k.shape[2]
    G = H // Hkv
    s = 1.0 / math.sqrt(D) if scale is None else scale
    o = np.zeros((B, H, Tq, D), dtype)
    lse = np.full((B, H, Tq), -np.inf, dtype)
    for b in range(B):
        n = Tkv if kv_lens is None else int(kv_lens[b])
        qi = (np.arange(Tq) + n - Tq)[:, None]
        ki = np.arange(n)[None, :]
        kb = np.repeat(k[b, :, :n].astype(dtype), G, axis=0)
        vb = np.repeat(v[b, :, :n].astype(dtype), G, axis=0)
        x = np.einsum("hqd,hkd->hqk", q[b].astype(dtype), kb) * s
        h = np.arange(H)[:, None, None]
        for f in score_mods:
            x = f(x, h, qi, ki)
        if mask is not None:
            x = np.where(mask(qi, ki), x, -np.inf)
        if n == 0:
            continue
        m = x.max(axis=-1, keepdims=True)
        empty = ~np.isfinite(m)
        m_safe = np.where(empty, 0.0, m)
        p = np.exp(x - m_safe)
        l = p.sum(axis=-1, keepdims=True)
        with np.errstate(invalid="ignore", divide="ignore"):
            ob = np.einsum("hqk,hkd->hqd", p / l, vb)
            lb = (m_safe + np.log(l))[..., 0]
        o[b] = np.where(empty, 0.0, ob)
        lse[b] = np.where(empty[..., 0], -np.inf, lb)
    return o, lse


def flash_fwd_tiled(q, k, v, mask: Optional[Callable] = None, block_r: int = 64, block_c: int = 64,
                    scale=None, dtype=np.float32):
    """Tile-faithful restatement of flash_attention_fwd_kernel (flash_attn.py:59-108).

    Per q tile: running (max, l, o); for every kv tile (no skipping, as the
    reference): s = q k^T * scale, masked to -inf; max_new = max(max, rowmax(s));
    p = exp(s - max_new) with NaN -> 0; o = o*alpha + p v; l = l*alpha + rowsum(p),
    alpha = exp(max - max_new) with NaN -> 0.  Then o /= l, lse = max + log(l).
    Requires T to be a multiple of the block sizes, as the reference does.
    """
    B, H, T, D = q.shape
    s = 1.0 / math.sqrt(D) if scale is None else scale
    o = np.zeros(q.shape, dtype)
    lse = np.zeros(q.shape[:3], dtype)
    for bh in np.ndindex(B, H):
        Q, K, V = q[bh].astype(dtype), k[bh].astype(dtype), v[bh].astype(dtype)
        for r0 in range(0, T, block_r):
            qi = np.arange(r0, r0 + block_r)
            mx = np.full(block_r, -np.inf, dtype)
            l = np.zeros(block_r, dtype)
            acc = np.zeros((block_r, D), dtype)
            for c0 in range(0, T, block_c):
                ki = np.arange(c0, c0 + block_c)
                S = (Q[r0:r0 + block_r] @ K[c0:c0 + block_c].T) * s
                if mask is not None:
                    S = np.where(mask(qi[:, None], ki[None, :]), S, -np.inf)
                mnew = np.maximum(mx, S.max(axis=-1))
                with np.errstate(invalid="ignore"):
                    p = np.exp(S - mnew[:, None])
                    p = np.where(np.isnan(p), 0.0, p)
                    alpha = np.exp(mx - mnew)
                    alpha = np.where(np.isnan(alpha), 0.0, alpha)
                acc = acc * alpha[:, None] + p.astype(dtype) @ V[c0:c0 + block_c]
                l = l * alpha + p.sum(axis=-1)
                mx = mnew
            with np.errstate(invalid="ignore", divide="ignore"):
                o[bh][r0:r0 + block_r] = acc / l[:, None]
                lse[bh][r0:r0 + block_r] = mx + np.log(l)
    return o, lse


def attention_bwd(q, k, v, o, lse, do, mask: Optional[Callable] = None, score_mods=(), scale=None,
                  dtype=np.float64):
    """Analytic backward (flash_attn.py:168-173, 241-245, 346-349).

    delta = rowsum(o * do); P = exp(x - lse); dP = dO V^T; dS = P (dP - delta)
    times d(score)/d(logit); dV = P^T dO; dK = dS^T Q * scale; dQ = dS K * scale.
    Rows with lse = -inf contribute nothing.  Returns (dq, dk, dv).
    """
    B, H, Tq, D = q.shape
    Tkv = k.shape[2]
    s = 1.0 / math.sqrt(D) if scale is None else scale
    raw, x = logits(q, k, s, score_mods, dtype)
    qi, ki = _idx(Tq, Tkv)
    h = np.arange(H)[None, :, None, None]
    valid = np.ones(x.shape, dtype=bool) if mask is None else np.broadcast_to(mask(qi, ki), x.shape)
    L = lse.astype(dtype)[..., None]
    live = valid & np.isfinite(L)
    with np.errstate(invalid="ignore", over="ignore"):
        P = np.where(live, np.exp(np.where(live, x, 0.0) - np.where(np.isfinite(L), L, 0.0)), 0.0)
    do_, o_, v_, q_, k_ = (a.astype(dtype) for a in (do, o, v, q, k))
    delta = (o_ * do_).sum(-1)[..., None]
    dP = np.einsum("bhqd,bhkd->bhqk", do_, v_)
    dS = P * (dP - delta)
    # chain rule through the score mods, innermost last
    g = np.ones_like(dS)
    for f in score_mods:
        if getattr(f, "grad", None) is not None:
            g = g * f.grad(_pre_mod(raw, score_mods, f, h, qi, ki), h, qi, ki)
    dS = dS * g
    dv = np.einsum("bhqk,bhqd->bhkd", P, do_)
    dk = np.einsum("bhqk,bhqd->bhkd", dS, q_) * s
    dq = np.einsum("bhqk,bhkd->bhqd", dS, k_) * s
    return dq, dk, dv


def _pre_mod(raw, mods, target, h, qi, ki):
    """The logit fed into `target` when `mods` are applied in order."""
    x = raw
    for f in mods:
        if f is target:
            return x
        x = f(x, h, qi, ki)
    return x


# ---------------------------------------------------------------------------- block masks
def _tile_bounds(n_blocks: int, block: int, length: int):
    starts = np.arange(n_blocks) * block
    ends = np.minimum(starts + block, length)
    return starts, ends


def block_mask_ref9(mask: Callable, Q_LEN: int, KV_LEN: int, block_size: int = 128):
    """The reference create_block_mask rule (block_mask.py:78-129).

    Tile (i, j) is valid iff mask is True at any of the 3x3 samples
    q in {q0, (q0+q1)//2, q1-1}, kv in {k0, (k0+k1)//2, k1-1}.  Returns
    (num_blocks_in_row int32 (nq,), col_indices int32 (nq, max_row) padded -1).
    """
    nq, nkv = math.ceil(Q_LEN / block_size), math.ceil(KV_LEN / block_size)
    qs, qe = _tile_bounds(nq, block_size, Q_LEN)
    ks, ke = _tile_bounds(nkv, block_size, KV_LEN)
    qsamp = np.stack([qs, (qs + qe) // 2, qe - 1], axis=1)
    ksamp = np.stack([ks, (ks + ke) // 2, ke - 1], axis=1)
    m = np.broadcast_to(mask(qsamp[:, :, None, None], ksamp[None, None, :, :]), (nq, 3, nkv, 3))
    valid = m.any(axis=(1, 3))
    return lists_from_valid(valid)


def lists_from_valid(valid: np.ndarray):
    counts = valid.sum(axis=1).astype(np.int32)
    max_row = int(counts.max()) if counts.size else 0
    cols = np.full((valid.shape[0], max_row), -1, dtype=np.int32)
    for i in range(valid.shape[0]):
        idx = np.nonzero(valid[i])[0]
        cols[i, : idx.size] = idx
    return counts, cols


def block_mask_exact(mask: Callable, Q_LEN: int, KV_LEN: int, block_q: int = 128, block_kv: int = 128):
    """Exact tile classes: 0 skip, 1 partial, 2 full ((nq, nkv) int8).

    A tile is listed iff any element (q < Q_LEN, kv in the block_kv-wide tile)
    is unmasked; it is full iff every element is unmasked and kv < KV_LEN.
    """
    nq, nkv = math.ceil(Q_LEN / block_q), math.ceil(KV_LEN / block_kv)
    cls = np.zeros((nq, nkv), dtype=np.int8)
    for i in range(nq):
        qi = np.arange(i * block_q, min((i + 1) * block_q, Q_LEN))[:, None]
        for j in range(nkv):
            ki = np.arange(j * block_kv, (j + 1) * block_kv)[None, :]
            m = np.broadcast_to(mask(qi, np.minimum(ki, KV_LEN - 1)), (qi.shape[0], block_kv)) & (ki < KV_LEN)
            cls[i, j] = 0 if not m.any() else (2 if m.all() else 1)
    return cls


def tables_from_classes(cls: np.ndarray):
    """Row and column lists (partial and full, ascending, -1 padded to full width)."""
    nq, nkv = cls.shape

    def lists(mat, n_other):
        part_n = (mat == 1).sum(axis=1).astype(np.int32)
        full_n = (mat == 2).sum(axis=1).astype(np.int32)
        part = np.full((mat.shape[0], n_other), -1, np.int32)
        full = np.full((mat.shape[0], n_other), -1, np.int32)
        for r in range(mat.shape[0]):
            p = np.nonzero(mat[r] == 1)[0]
            f = np.nonzero(mat[r] == 2)[0]
            part[r, : p.size] = p
            full[r, : f.size] = f
        return part_n, part, full_n, full

    kv = lists(cls, nkv)
    qq = lists(cls.T, nq)
    return {
        "kv_num_blocks": kv[0], "kv_indices": kv[1], "full_kv_num_blocks": kv[2], "full_kv_indices": kv[3],
        "q_num_blocks": qq[0], "q_indices": qq[1], "full_q_num_blocks": qq[2], "full_q_indices": qq[3],
    }


def causal_block_mask(seq_len: int, block_size: int = 128):
    """block_mask.py:132-172."""
    n = math.ceil(seq_len / block_size)
    valid = np.tril(np.ones((n, n), dtype=bool))
    return lists_from_valid(valid)


def sliding_window_block_mask(seq_len: int, window_size: int, block_size: int = 128):
    """block_mask.py:175-218 (symmetric, superset-based)."""
    n = math.ceil(seq_len / block_size)
    w = math.ceil(window_size / block_size)
    i = np.arange(n)[:, None]
    j = np.arange(n)[None, :]
    valid = (j >= np.maximum(0, i - w)) & (j < np.minimum(n, i + w + 1))
    return lists_from_valid(valid)


def unmasked_pairs(mask: Optional[Callable], Tq: int, Tkv: int, chunk: int = 2048) -> int:
    """Exact count of unmasked (q, kv) pairs (for effective-FLOP accounting)."""
    if mask is None:
        return Tq * Tkv
    n = 0
    ki = np.arange(Tkv)[None, :]
    for r0 in range(0, Tq, chunk):
        qi = np.arange(r0, min(r0 + chunk, Tq))[:, None]
        n += int(np.broadcast_to(mask(qi, ki), (qi.shape[0], Tkv)).sum())
    return n
