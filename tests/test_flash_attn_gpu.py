"""GPU parity: the CUDA kernels through the public API against the CPU oracle.

Tolerance (tests/tolerance.py): bf16 results within 2e-2 + half an ulp of the bf16
output per element (the output's own rounding) and relative-L2 <= 5e-3, against an
fp32/fp64 reference on the same (bf16-rounded) inputs, for o and for dq/dk/dv; no
quantile anywhere.  fp32 inputs (generic kernels) are held to 2e-4 / 1e-5.  Small shapes
use the numpy oracle (oracle/flexattn_oracle.py); full-length benchmark shapes use a
chunked fp32 torch reference of the same formulas, itself checked against the oracle here.
"""
import math

import numpy as np
import pytest
import torch

import pallas_flexattn as pf
from oracle import flexattn_oracle as O
from pallas_flexattn import workloads as W
from pallas_flexattn.flash_attn import check_device_status
from tolerance import assert_close
from torch_reference import torch_reference

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def inputs(shape_q, shape_kv, dtype, seed=0, scale=1.0):
    rng = np.random.default_rng(seed)
    mk = lambda s: torch.from_numpy((rng.standard_normal(s) * scale).astype(np.float32)).to(DEV, dtype)  # noqa: E731
    return mk(shape_q), mk(shape_kv), mk(shape_kv), mk(shape_q)


def close(name, got, ref, dtype):
    got = got.detach().float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    ref = ref.detach().float().cpu().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref)
    assert_close(name, got, ref, bf16=dtype == torch.bfloat16)


def run_api(q, k, v, do, mask_mod=None, score_mod=None, block_mask=None, bwd=True, **kw):
    q, k, v = (t.detach().clone().requires_grad_(bwd) for t in (q, k, v))
    o = pf.flash_attention(q, k, v, mask_mod, score_mod=score_mod, block_mask=block_mask, **kw)
    grads = torch.autograd.grad(o, (q, k, v), do) if bwd else None
    torch.cuda.synchronize()
    check_device_status(DEV)
    return o, grads


def oracle(q, k, v, do, mask=None, mods=()):
    qf, kf, vf, dof = (t.detach().float().cpu().numpy().astype(np.float64) for t in (q, k, v, do))
    o, lse = O.mha_reference(qf, kf, vf, mask, mods)
    return o, lse, O.attention_bwd(qf, kf, vf, o, lse, dof, mask, mods)


def check_all(q, k, v, do, mask_mod, omask, score_mod=None, omods=(), bwd=True, block_mask=None, **kw):
    o, g = run_api(q, k, v, do, mask_mod, score_mod, block_mask=block_mask, bwd=bwd, **kw)
    ro, rlse, rg = oracle(q, k, v, do, omask, omods)
    close("o", o, ro, q.dtype)
    if bwd:
        for n, a, b in zip(("dq", "dk", "dv"), g, rg):
            close(n, a, b, q.dtype)


# ------------------------------------------------------------------------ the reference's test suite
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("mname", ["causal", "bidir", "window32"])
def test_reference_forward_and_gradients(dtype, mname):
    """tests/test_flash_attn.py:43-71,117-135 of the reference (B2 H4 T128 D64)."""
    mm, om = {"causal": (pf.causal_mask, O.causal), "bidir": (pf.bidirectional_mask, O.bidirectional),
              "window32": (pf.sliding_window_mask(32, 32), O.sliding_window(32, 32))}[mname]
    q, k, v, do = inputs((2, 4, 128, 64), (2, 4, 128, 64), dtype)
    check_all(q, k, v, do, mm, om)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B", [1, 2, 4])
def test_batch_sizes(dtype, B):
    q, k, v, do = inputs((B, 4, 64, 32), (B, 4, 64, 32), dtype, seed=B)
    check_all(q, k, v, do, None, None)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_head_dims(dtype, D):
    q, k, v, do = inputs((2, 4, 64, D), (2, 4, 64, D), dtype, seed=D)
    check_all(q, k, v, do, pf.causal_mask, O.causal)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_large_sequence_length(dtype):
    q, k, v, do = inputs((1, 2, 512, 64), (1, 2, 512, 64), dtype, seed=7)
    check_all(q, k, v, do, None, None)


def test_no_nan_no_inf_and_shapes():
    q, k, v, do = inputs((2, 4, 128, 64), (2, 4, 128, 64), torch.bfloat16)
    o, (dq, dk, dv) = run_api(q, k, v, do)
    assert o.shape == q.shape and dq.shape == q.shape and dk.shape == k.shape and dv.shape == v.shape
    for t in (o, dq, dk, dv):
        assert torch.isfinite(t).all()


# ------------------------------------------------------------------------ golden: the reference's own kernels
GOLD = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "attention.npz")
GMASK = {"causal_B1H2T128D32": pf.causal_mask, "bidir_B1H2T128D32": pf.bidirectional_mask,
         "window32_B1H2T128D32": pf.sliding_window_mask(32, 32), "causal_B1H2T128D64": pf.causal_mask}


@pytest.mark.parametrize("name", sorted(GMASK))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_matches_reference_kernel_outputs(name, dtype):
    g = {k: GOLD[f"{name}/{k}"] for k in ("q", "k", "v", "do", "o", "lse", "dq", "dk", "dv")}
    q, k, v, do = (torch.from_numpy(g[n]).to(DEV, dtype) for n in ("q", "k", "v", "do"))
    o, lse = pf.flash_attention_fwd(q, k, v, GMASK[name])
    dq, dk, dv = pf.flash_attention_bwd(q, k, v, o, lse, do, GMASK[name])
    torch.cuda.synchronize()
    if dtype == torch.float32:
        close("o", o, g["o"], dtype)
        close("lse", lse, g["lse"], dtype)
        for n, a in (("dq", dq), ("dk", dk), ("dv", dv)):
            close(n, a, g[n], dtype)
    else:  # bf16 inputs differ from the fp32 golden inputs: compare against the oracle on them
        check_all(q, k, v, do, GMASK[name], None if "bidir" in name else {
            "causal_B1H2T128D32": O.causal, "causal_B1H2T128D64": O.causal,
            "window32_B1H2T128D32": O.sliding_window(32, 32)}[name])


# ------------------------------------------------------------------------ score_mods
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("kind", ["alibi", "softcap", "relbias", "alibi+softcap"])
def test_score_mods(D, kind):
    H, T = 3, 384
    q, k, v, do = inputs((1, H, T, D), (1, H, T, D), torch.bfloat16, seed=11)
    slopes = O.alibi_slopes(H)
    bias = np.random.default_rng(5).standard_normal((H, 2 * T - 1)).astype(np.float32) * 0.5
    al, om_al = pf.alibi_score_mod(H), O.alibi(slopes)
    sc, om_sc = pf.softcap_score_mod(2.5), O.softcap(2.5)
    rb = pf.relative_bias_score_mod(bias)

    def om_rb(s, h, qi, ki):
        return s + bias.astype(np.float64)[h, qi - ki + T - 1]

    om_rb.grad = None
    sm, om = {"alibi": (al, (om_al,)), "softcap": (sc, (om_sc,)), "relbias": (rb, (om_rb,)),
              "alibi+softcap": (pf.compose_score_mods(sc, al), (om_al, om_sc))}[kind]
    check_all(q, k, v, do, pf.causal_mask, O.causal, sm, om)


# ------------------------------------------------------------------------ masks and shapes
@pytest.mark.parametrize("D", [64, 128])
def test_document_and_tile_masks(D):
    T = 640
    lens = [100, 250, 37, 253]
    doc = np.repeat(np.arange(4), lens)
    q, k, v, do = inputs((1, 2, T, D), (1, 2, T, D), torch.bfloat16, seed=3)
    check_all(q, k, v, do, pf.and_masks(pf.document_mask(lens), pf.causal_mask), O.and_(O.document(doc), O.causal))
    table = W.random_tile_table(5, 0.4, seed=2)
    check_all(q, k, v, do, pf.and_masks(pf.causal_mask, pf.tile_mask(table, 128)),
              O.and_(O.causal, O.tile_table(table, 128)))


@pytest.mark.parametrize("D", [64, 128])
def test_document_id_layouts(D):
    """Contiguous documents take the per-row interval path of the tcgen05 kernels (ids sorted),
    interleaved ids the per-element path; per-batch document lengths give 2-D ids."""
    T = 520
    q, k, v, do = inputs((1, 2, T, D), (1, 2, T, D), torch.bfloat16, seed=11)
    lens = [300, 20, 200]
    doc = np.repeat(np.arange(3), lens)
    check_all(q, k, v, do, pf.and_masks(pf.document_mask(lens), pf.sliding_window_mask(150, 0)),
              O.and_(O.document(doc), O.sliding_window(150, 0)))
    inter = (np.arange(T) // 37) % 3  # non-monotone ids: documents interleave
    assert not pf.document_ids_mask(inter).__fa_spec__.doc_sorted
    check_all(q, k, v, do, pf.and_masks(pf.document_ids_mask(inter), pf.causal_mask),
              O.and_(O.document(inter), O.causal))
    qb, kb, vb, dob = inputs((2, 2, T, D), (2, 2, T, D), torch.bfloat16, seed=12)
    lens2 = [[100, 420], [260, 130, 130]]
    mm = pf.and_masks(pf.document_mask(lens2), pf.causal_mask)
    assert mm.__fa_spec__.doc_sorted and mm.__fa_spec__.depends_on_batch
    o, g = run_api(qb, kb, vb, dob, mm)
    for bi in range(2):
        docb = np.repeat(np.arange(len(lens2[bi])), lens2[bi])
        ro, _, rg = oracle(qb[bi:bi + 1], kb[bi:bi + 1], vb[bi:bi + 1], dob[bi:bi + 1], O.and_(O.document(docb), O.causal))
        close("o", o[bi:bi + 1], ro, torch.bfloat16)
        for n, a_, b_ in zip(("dq", "dk", "dv"), g, rg):
            close(n, a_[bi:bi + 1], b_, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T", [1, 77, 200, 300, 129])
def test_ragged_lengths(dtype, T):
    q, k, v, do = inputs((1, 2, T, 64), (1, 2, T, 64), dtype, seed=T)
    check_all(q, k, v, do, pf.causal_mask, O.causal)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cross_attention_lengths(dtype):
    q, k, v, do = inputs((2, 2, 256, 128), (2, 2, 384, 128), dtype, seed=9)
    check_all(q, k, v, do, pf.causal_mask, O.causal)
    q, k, v, do = inputs((1, 2, 300, 64), (1, 2, 130, 64), dtype, seed=10)
    check_all(q, k, v, do, None, None)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Hkv", [1, 2])
def test_grouped_query_attention(dtype, D, Hkv):
    """GQA / MQA: 8 query heads share Hkv K/V heads; dK, dV sum over each group (the oracle
    runs on K/V repeated per query head and its gradients are summed back)."""
    G = 8 // Hkv
    q, k, v, do = inputs((2, 8, 300, D), (2, Hkv, 300, D), dtype, seed=12 + Hkv)
    al = pf.alibi_score_mod(8)
    o, (dq, dk, dv) = run_api(q, k, v, do, pf.causal_mask, al)
    kr, vr = k.repeat_interleave(G, dim=1), v.repeat_interleave(G, dim=1)
    ro, _, (rdq, rdk, rdv) = oracle(q, kr, vr, do, O.causal, (O.alibi(pf.alibi_slopes(8).numpy()),))
    close("o", o, ro, dtype)
    close("dq", dq, rdq, dtype)
    rdk = rdk.reshape(2, Hkv, G, 300, D).sum(axis=2)
    rdv = rdv.reshape(2, Hkv, G, 300, D).sum(axis=2)
    close("dk", dk, rdk, dtype)
    close("dv", dv, rdv, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fully_masked_rows_give_zero_output_and_gradients(dtype):
    table = np.array([[0, 0], [1, 1]], np.uint8)  # q block 0 sees nothing
    q, k, v, do = inputs((1, 2, 256, 64), (1, 2, 256, 64), dtype, seed=13)
    mm = pf.and_masks(pf.causal_mask, pf.tile_mask(table, 128))
    o, lse = pf.flash_attention_fwd(q, k, v, mm)
    assert torch.all(o[:, :, :128] == 0) and torch.all(torch.isneginf(lse[:, :, :128]))
    check_all(q, k, v, do, mm, O.and_(O.causal, O.tile_table(table, 128)))


def test_strided_layout_inputs():
    """(B, T, H, D) storage viewed as (B, H, T, D): strides pass through the C ABI."""
    rng = np.random.default_rng(14)
    base = [torch.from_numpy(rng.standard_normal((2, 256, 4, 128)).astype(np.float32)).to(DEV, torch.bfloat16)
            for _ in range(4)]
    q, k, v, do = (t.transpose(1, 2) for t in base)
    assert not q.is_contiguous()
    check_all(q, k, v, do, pf.causal_mask, O.causal)


def test_forward_is_deterministic():
    q, k, v, do = inputs((2, 4, 1024, 128), (2, 4, 1024, 128), torch.bfloat16, seed=15)
    o1, l1 = pf.flash_attention_fwd(q, k, v, pf.causal_mask)
    o2, l2 = pf.flash_attention_fwd(q, k, v, pf.causal_mask)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_block_mask_argument_and_reference_style_lists():
    T = 512
    q, k, v, do = inputs((1, 2, T, 128), (1, 2, T, 128), torch.bfloat16, seed=16)
    bm = pf.create_block_mask(pf.causal_mask, 1, 2, T, T, 128)
    check_all(q, k, v, do, None, O.causal, block_mask=bm)  # mask_mod taken from the block mask
    lists = pf.create_causal_block_mask(T, 128)  # host-built, reference fields only: all tiles partial
    check_all(q, k, v, do, pf.causal_mask, O.causal, block_mask=lists)


def test_lse_matches_oracle():
    q, k, v, do = inputs((1, 2, 300, 128), (1, 2, 300, 128), torch.bfloat16, seed=17)
    _, lse = pf.flash_attention_fwd(q, k, v, pf.sliding_window_mask(40, 3))
    _, rlse, _ = oracle(q, k, v, do, O.sliding_window(40, 3))
    np.testing.assert_allclose(lse.cpu().numpy(), rlse, atol=2e-3, rtol=1e-4)


# ------------------------------------------------------------------------ full-length benchmark shapes
def test_torch_reference_matches_oracle():
    q, k, v, do = inputs((1, 2, 256, 64), (1, 2, 256, 64), torch.float32, seed=18)

    def sc(raw, h, qi, ki):
        t = torch.tanh(raw / 3.0)
        return 3.0 * t, 1 - t * t

    ro, rlse, rg = oracle(q, k, v, do, O.causal, (O.softcap(3.0),))
    to, tlse, *tg = torch_reference(q, k, v, do, lambda qi, ki: qi >= ki, sc, chunk=100)
    np.testing.assert_allclose(to.cpu().numpy(), ro, atol=1e-5)
    for a, b in zip(tg, rg):
        np.testing.assert_allclose(a.cpu().numpy(), b, atol=1e-4)


@pytest.mark.parametrize("seed", [0, 1])
@pytest.mark.parametrize("cfg", [2, 3, 4, 5])
def test_benchmark_config_full_length(cfg, seed):
    """Each benchmark configuration at its full sequence length on four heads, every element
    of o, dq, dk and dv held to the bar (no quantile)."""
    w = W.get(cfg)
    H = 4
    g = torch.Generator(device=DEV).manual_seed(100 * seed + cfg)
    q, k, v, do = (torch.randn((1, H, w.S, w.D), generator=g, device=DEV) * w.input_scale for _ in range(4))
    q, k, v, do = (t.to(w.dtype) for t in (q, k, v, do))
    mm, sm = w.mask_mod, w.score_mod
    h0 = 4 * seed  # heads h0 .. h0+3 of the 32-head ALiBi slope set (the steepest first)
    slopes = pf.alibi_slopes(32)[h0:h0 + H]
    if cfg == 3:
        sm = pf.alibi_score_mod(slopes=slopes)
    o, (dq, dk, dv) = run_api(q, k, v, do, mm, sm)

    def score_fn(raw, hi, qi, ki):
        if cfg == 3:
            return raw + slopes.to(DEV)[hi] * (ki - qi), torch.ones_like(raw)
        if cfg == 5:
            t = torch.tanh(raw / 30.0)
            return 30.0 * t, 1 - t * t
        return raw, torch.ones_like(raw)

    ref = torch_reference(q, k, v, do, mm, score_fn if cfg in (3, 5) else None, chunk=512 if w.S > 8192 else 1024)
    for n, a, b in zip(("o", "lse", "dq", "dk", "dv"), (o, None, dq, dk, dv), ref):
        if a is not None:
            close(n, a, b, torch.bfloat16)


@pytest.mark.parametrize("D,T", [(128, 1000), (64, 4097), (96, 300)])
def test_bwd_preprocess_entry_point(D, T):
    """fa_bwd_preprocess: delta = rowsum(o * dO) in fp32 for every row, and the dQ accumulator
    [B*H, T, D] zeroed (it starts full of garbage here)."""
    import ctypes as C

    from pallas_flexattn import _lib as L
    from pallas_flexattn import flash_attn as FA

    q, k, v, do = inputs((2, 3, T, D), (2, 3, T, D), torch.bfloat16, seed=T)
    o = torch.randn_like(q.float()).to(torch.bfloat16)
    lse = torch.zeros(q.shape[:3], dtype=torch.float32, device=DEV)
    plan = FA._Plan(q, k, v, pf.causal_mask, None, None, 64, 64, 3, None, True)
    p = L.FaBwdParams()
    plan._fill(p)
    p.q, p.k, p.v, p.o, p.dout = (FA._fa_tensor(t) for t in (q, k, v, o, do))
    p.dq, p.dk, p.dv = (FA._fa_tensor(torch.empty_like(t)) for t in (q, k, v))
    p.lse = lse.data_ptr()
    delta = torch.full((2 * 3 * T,), float("nan"), dtype=torch.float32, device=DEV)
    acc = torch.full((2 * 3 * T * D,), 7.0, dtype=torch.float32, device=DEV)
    L.check(L.lib().fa_bwd_preprocess(C.byref(p), delta.data_ptr(), acc.data_ptr(),
                                      torch.cuda.current_stream(DEV).cuda_stream))
    torch.cuda.synchronize()
    ref = (o.float() * do.float()).sum(-1).flatten()
    torch.testing.assert_close(delta, ref, atol=1e-4, rtol=1e-5)
    assert int((acc != 0).sum()) == 0


LAMBDAS = {
    # a band 100..110 back (no registry entry; fully masked rows at the start)
    "band": lambda q, kv: ((q - kv) >= 100) & ((q - kv) <= 110),
    # scattered keys plus the diagonal, causal
    "scatter": lambda q, kv: (((q * 7 + kv * 3) % 11 < 4) | (q == kv)) & (q >= kv),
    # prefix-LM: a bidirectional prefix of 200 positions, causal after it
    "prefix_lm": lambda q, kv: (kv < 200) | (q >= kv),
}


@pytest.mark.parametrize("name", list(LAMBDAS))
@pytest.mark.parametrize("dtype,D,T", [(torch.bfloat16, 128, 1000), (torch.bfloat16, 64, 640),
                                       (torch.float32, 64, 300)])
def test_arbitrary_mask_callable(name, dtype, D, T):
    """A mask_mod with no registry entry: evaluated on the GPU into per-tile bitmasks and
    tested per element by the kernels (tcgen05 for bf16, generic for fp32)."""
    fn = LAMBDAS[name]
    q, k, v, do = inputs((1, 2, T, D), (1, 2, T, D), dtype, seed=T + D)
    check_all(q, k, v, do, fn, fn)


def test_arbitrary_callable_inside_and_masks_with_score_mod():
    mm = pf.and_masks(pf.sliding_window_mask(300, 0), lambda q, kv: (kv % 4) != 1)  # callable part -> callable
    om = O.and_(O.sliding_window(300, 0), lambda q, kv: (kv % 4) != 1)
    q, k, v, do = inputs((2, 2, 768, 128), (2, 2, 768, 128), torch.bfloat16, seed=5)
    check_all(q, k, v, do, mm, om, pf.softcap_score_mod(20.0), (O.softcap(20.0),))


def test_fresh_tile_masks_never_reuse_cached_tables():
    """Block tables are cached under the mask's tensors' ids; a mask built after an earlier one
    was freed (its tile table may get the same id) must still get its own tables."""
    import gc

    T = 640
    q, k, v, do = inputs((1, 2, T, 64), (1, 2, T, 64), torch.bfloat16, seed=3)
    qf, kf, vf = (t.float().cpu().numpy().astype(np.float64) for t in (q, k, v))
    for trial in range(6):
        rng = np.random.default_rng(100 + trial)
        table = (rng.random((5, 5)) < 0.5).astype(np.uint8)
        np.fill_diagonal(table, 1)
        mm = pf.and_masks(pf.causal_mask, pf.tile_mask(table, 128))
        o, _ = pf.flash_attention_fwd(q, k, v, mm)
        ro, _ = O.mha_reference(qf, kf, vf, O.and_(O.causal, O.tile_table(table, 128)))
        close(f"o (trial {trial})", o, ro, torch.bfloat16)
        del mm, o
        gc.collect()


@pytest.mark.parametrize("D", [64, 128])
def test_dense_block_lists_with_a_tile_table_mask(D):
    """Reference-style block lists that visit every tile, with a tile-table mask_mod: every
    listed tile is partial, so the kernels must apply the table to tiles whose cell is zero
    (tested once per tile when the cells cover whole 128 x 128 tiles)."""
    T = 768
    table = W.random_tile_table(6, 0.35, seed=9)
    mm = pf.and_masks(pf.causal_mask, pf.tile_mask(table, 128))
    n = T // 128
    bm = pf.BlockMask(torch.full((n,), n, dtype=torch.int32), torch.arange(n, dtype=torch.int32).repeat(n, 1),
                      128, T, T, None, mm)
    q, k, v, do = inputs((1, 2, T, D), (1, 2, T, D), torch.bfloat16, seed=D)
    check_all(q, k, v, do, mm, O.and_(O.causal, O.tile_table(table, 128)), block_mask=bm)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("tile_cfg", [33, 34, 35, 96, 17, 41, 37])
def test_every_forward_launch_shape(D, tile_cfg):
    """Each launch shape of the tcgen05 forward (two Q tiles, one, head pairs, kv halves, rows
    split over two warps, softmax turns or concurrent) against the oracle on a ragged length,
    so every epilogue (the per-sub-tile TMA store, the kv-halves merge) writes the tail rows
    right; causal, and bidirectional with ALiBi (which also takes softmax turns)."""
    from pallas_flexattn import flash_attn as FA

    q, k, v, do = inputs((2, 4, 333, D), (2, 4, 333, D), torch.bfloat16, seed=40 + tile_cfg)
    for mask_mod, omask, score_mod, omods in ((pf.causal_mask, O.causal, None, ()),
                                              (None, None, pf.alibi_score_mod(4), (O.alibi(O.alibi_slopes(4)),))):
        plan = FA._Plan(q, k, v, mask_mod, score_mod, None, 128, 128, 0, None, need_bwd=False)
        plan.fwd_tile_cfg = tile_cfg
        o2, lse = FA._run_fwd(plan, q, k, v)
        torch.cuda.synchronize()
        check_device_status(DEV)
        ro, rlse, _ = oracle(q, k, v, do, omask, omods)
        close("o", o2, ro, torch.bfloat16)
        np.testing.assert_allclose(lse.cpu().numpy(), rlse, rtol=0, atol=2e-3)
