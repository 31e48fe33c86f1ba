"""The CPU oracle against the reference's own outputs (golden vectors), on CPU.

Fixtures come from tests/golden/make_golden.py, which runs the reference source
(block_mask.py, kernel_tuner.py and the Pallas kernels of flash_attn.py in
interpret emulation).  These tests pin the oracle before any GPU test trusts it.
"""
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import flexattn_oracle as O

GOLD = Path(__file__).resolve().parent / "golden"
BM = np.load(GOLD / "block_masks.npz")
ATT = np.load(GOLD / "attention.npz")


def _doc_ids():
    return np.repeat(np.arange(len(BM["meta/doc_lengths"])), BM["meta/doc_lengths"])


def _tile_table():
    rng = np.random.default_rng(0)
    keep = rng.random((256, 256)) < 0.25
    np.fill_diagonal(keep, True)
    return keep.astype(np.uint8)


MASKS = {
    "causal_T256_b64": O.causal,
    "bidir_T256_b64": O.bidirectional,
    "window32_32_T256_b64": O.sliding_window(32, 32),
    "window64_64_T256_b64": O.sliding_window(64, 64),
    "causal_T300_b64": O.causal,
    "window16_16_T300_b64": O.sliding_window(16, 16),
    "causal_Q256_KV384_b64": O.causal,
    "causal_T64_b16": O.causal,
    "causal_T64_b128": O.causal,
    "cfg1_causal_T512_b128": O.causal,
    "cfg2_causal_T4096_b128": O.causal,
    "cfg3_window1024_0_T8192_b128": O.sliding_window(1024, 0),
    "cfg4_doc_causal_T16384_b128": O.and_(O.document(_doc_ids()), O.causal),
    "cfg5_causal_tiles_T32768_b128": O.and_(O.causal, O.tile_table(_tile_table(), 128)),
    "band100_110_T1024_b128": lambda q, kv: ((q - kv) >= 100) & ((q - kv) <= 110),
}


@pytest.mark.parametrize("name", sorted(MASKS))
def test_ref9_block_mask_matches_reference(name):
    ql, kl, bs = (int(x) for x in BM[f"{name}/geom"])
    num, cols = O.block_mask_ref9(MASKS[name], ql, kl, bs)
    np.testing.assert_array_equal(num, BM[f"{name}/num"])
    np.testing.assert_array_equal(cols, BM[f"{name}/cols"].reshape(cols.shape))
    assert num.dtype == np.int32 and cols.dtype == np.int32


@pytest.mark.parametrize("T,bs", [(256, 64), (300, 64), (64, 16), (64, 128), (1024, 128), (128, 64)])
def test_causal_builder_matches_reference(T, bs):
    num, cols = O.causal_block_mask(T, bs)
    np.testing.assert_array_equal(num, BM[f"causalbuilder_T{T}_b{bs}/num"])
    np.testing.assert_array_equal(cols, BM[f"causalbuilder_T{T}_b{bs}/cols"])


@pytest.mark.parametrize("T,w,bs", [(256, 64, 64), (1000, 100, 128), (512, 200, 64)])
def test_window_builder_matches_reference(T, w, bs):
    num, cols = O.sliding_window_block_mask(T, w, bs)
    np.testing.assert_array_equal(num, BM[f"windowbuilder_T{T}_w{w}_b{bs}/num"])
    np.testing.assert_array_equal(cols, BM[f"windowbuilder_T{T}_w{w}_b{bs}/cols"])


ATT_CASES = {
    "causal_B1H2T128D32": O.causal,
    "bidir_B1H2T128D32": O.bidirectional,
    "window32_B1H2T128D32": O.sliding_window(32, 32),
    "causal_B1H2T128D64": O.causal,
}


@pytest.mark.parametrize("name", sorted(ATT_CASES))
def test_oracle_forward_matches_reference_kernels(name):
    g = {k: ATT[f"{name}/{k}"] for k in ("q", "k", "v", "do", "o", "lse", "dq", "dk", "dv", "o_ref")}
    m = ATT_CASES[name]
    o, lse = O.mha_reference(g["q"], g["k"], g["v"], m)
    np.testing.assert_allclose(o, g["o_ref"], atol=2e-5, rtol=1e-4)   # reference mha_reference
    np.testing.assert_allclose(o, g["o"], atol=2e-5, rtol=1e-4)       # reference Pallas forward kernel
    np.testing.assert_allclose(lse, g["lse"], atol=2e-5, rtol=1e-5)
    ot, lt = O.flash_fwd_tiled(g["q"], g["k"], g["v"], m, 64, 64)
    np.testing.assert_allclose(ot, g["o"], atol=2e-6, rtol=1e-5)      # same recurrence, same tiles
    np.testing.assert_allclose(lt, g["lse"], atol=2e-6, rtol=1e-6)


@pytest.mark.parametrize("name", sorted(ATT_CASES))
def test_oracle_backward_matches_reference_kernels(name):
    g = {k: ATT[f"{name}/{k}"] for k in ("q", "k", "v", "do", "o", "lse", "dq", "dk", "dv")}
    dq, dk, dv = O.attention_bwd(g["q"], g["k"], g["v"], g["o"], g["lse"], g["do"], ATT_CASES[name])
    for got, key in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, g[key], atol=5e-5, rtol=1e-4)


def _torch_grads(q, k, v, do, mask, mods):
    import torch

    tq, tk, tv = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (q, k, v))
    D = q.shape[-1]
    s = torch.einsum("bhqd,bhkd->bhqk", tq, tk) / math.sqrt(D)
    Tq, Tkv = q.shape[2], k.shape[2]
    qi = torch.arange(Tq)[:, None]
    ki = torch.arange(Tkv)[None, :]
    h = torch.arange(q.shape[1])[None, :, None, None]
    for f in mods:
        s = f.torch(s, h, qi, ki)
    if mask is not None:
        s = torch.where(torch.as_tensor(mask(qi.numpy(), ki.numpy())), s, torch.tensor(-math.inf, dtype=s.dtype))
    o = torch.softmax(s, -1) @ tv
    o.backward(torch.tensor(do, dtype=torch.float64))
    return o.detach().numpy(), tq.grad.numpy(), tk.grad.numpy(), tv.grad.numpy()


def test_oracle_backward_matches_autograd_with_score_mods():
    import torch

    rng = np.random.default_rng(3)
    B, H, T, D = 1, 3, 48, 16
    q, k, v, do = (rng.standard_normal((B, H, T, D)) for _ in range(4))
    slopes = O.alibi_slopes(H)
    al = O.alibi(slopes)
    al.torch = lambda s, h, qi, ki: s + torch.tensor(slopes)[h] * (ki - qi)
    sc = O.softcap(2.0)
    sc.torch = lambda s, h, qi, ki: 2.0 * torch.tanh(s / 2.0)
    mask = O.sliding_window(20, 0)
    for mods in ((), (al,), (sc,), (al, sc)):
        o, lse = O.mha_reference(q, k, v, mask, mods)
        to, tdq, tdk, tdv = _torch_grads(q, k, v, do, mask, mods)
        np.testing.assert_allclose(o, to, atol=1e-10)
        dq, dk, dv = O.attention_bwd(q, k, v, o, lse, do, mask, mods)
        np.testing.assert_allclose(dq, tdq, atol=1e-9)
        np.testing.assert_allclose(dk, tdk, atol=1e-9)
        np.testing.assert_allclose(dv, tdv, atol=1e-9)


def test_fully_masked_rows_follow_flexattention_convention():
    rng = np.random.default_rng(4)
    q, k, v, do = (rng.standard_normal((1, 1, 16, 8)) for _ in range(4))
    mask = lambda qi, ki: (qi >= 4) & (qi >= ki)  # noqa: E731  rows 0..3 see nothing
    o, lse = O.mha_reference(q, k, v, mask)
    assert np.all(o[0, 0, :4] == 0) and np.all(np.isneginf(lse[0, 0, :4]))
    dq, dk, dv = O.attention_bwd(q, k, v, o, lse, do, mask)
    assert np.all(dq[0, 0, :4] == 0) and np.isfinite(dq).all() and np.isfinite(dk).all()


@pytest.mark.parametrize("mask_name", ["none", "causal", "window"])
def test_decode_reference_is_the_tail_of_full_attention(mask_name):
    """decode_reference for batch b equals the last Tq rows of mha_reference over that
    sequence's first kv_lens[b] positions, with grouped K/V heads expanded."""
    rng = np.random.default_rng(11)
    B, H, Hkv, Tq, Tkv, D = 3, 4, 2, 3, 40, 8
    lens = [40, 17, 3]
    q_full = rng.standard_normal((B, H, Tkv, D))
    k, v = (rng.standard_normal((B, Hkv, Tkv, D)) for _ in range(2))
    mask = {"none": None, "causal": O.causal, "window": O.and_(O.causal, O.sliding_window(5, 0))}[mask_name]
    mods = (O.alibi(O.alibi_slopes(H)), O.softcap(20.0))
    q = np.stack([q_full[b, :, n - Tq:n] for b, n in enumerate(lens)])
    o, lse = O.decode_reference(q, k, v, lens, mask, mods)
    for b, n in enumerate(lens):
        kk, vv = (np.repeat(x[b:b + 1, :, :n], H // Hkv, axis=1) for x in (k, v))
        ro, rl = O.mha_reference(q_full[b:b + 1, :, :n], kk, vv, mask, mods)
        np.testing.assert_allclose(o[b], ro[0, :, n - Tq:], atol=1e-12)
        np.testing.assert_allclose(lse[b], rl[0, :, n - Tq:], atol=1e-12)


# Exact classification on the benchmark masks: tile counts (full, partial).
EXACT_COUNTS = {
    "cfg1_causal_T512_b128": (6, 4),
    "cfg2_causal_T4096_b128": (496, 32),
    "cfg3_window1024_0_T8192_b128": (420, 120),
    "cfg4_doc_causal_T16384_b128": (1024, 324),
}


@pytest.mark.parametrize("name", sorted(EXACT_COUNTS))
def test_exact_classification_counts_and_agreement_with_ref9(name):
    ql, kl, bs = (int(x) for x in BM[f"{name}/geom"])
    cls = O.block_mask_exact(MASKS[name], ql, kl, bs, bs)
    full, part = int((cls == 2).sum()), int((cls == 1).sum())
    assert (full, part) == EXACT_COUNTS[name]
    num, cols = O.lists_from_valid(cls > 0)
    np.testing.assert_array_equal(num, BM[f"{name}/num"])  # sampling finds every tile on these masks


def test_ref9_misses_band_tiles_exact_does_not():
    m = MASKS["band100_110_T1024_b128"]
    cls = O.block_mask_exact(m, 1024, 1024, 128, 128)
    assert int((cls > 0).sum()) == 15 and int(BM["band100_110_T1024_b128/num"].sum()) == 0


def test_tables_from_classes_are_transposes():
    cls = O.block_mask_exact(O.sliding_window(100, 20), 700, 900, 128, 128)
    t = O.tables_from_classes(cls)
    for i in range(cls.shape[0]):
        assert list(t["kv_indices"][i, : t["kv_num_blocks"][i]]) == list(np.nonzero(cls[i] == 1)[0])
    for j in range(cls.shape[1]):
        assert list(t["full_q_indices"][j, : t["full_q_num_blocks"][j]]) == list(np.nonzero(cls[:, j] == 2)[0])
