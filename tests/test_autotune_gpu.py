"""The measured autotuner on the GPU: it times the forward's launch configurations (pipeline
depth x one or two Q tiles per CTA x softmax schedule) and the backward's depths, caches
the fastest, and flash_attention uses the cached choice when num_stages is not given.  The
tuned call gives the same forward output as an explicit call with the same configuration
and stays within the parity bar of the oracle."""
import json

import numpy as np
import pytest
import torch

import pallas_flexattn as pf
from oracle import flexattn_oracle as O
from pallas_flexattn import _lib as L
from pallas_flexattn import flash_attn as FA
from pallas_flexattn import kernel_tuner as KT
from tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


@pytest.mark.parametrize("D", [128, 64])
def test_autotune_caches_and_is_used(tmp_path, monkeypatch, D):
    monkeypatch.setenv("FLEXATTN_TUNE_CACHE", str(tmp_path / "tune.json"))
    KT.clear_memory_cache()
    rng = np.random.default_rng(D)
    q, k, v, do = (torch.from_numpy(rng.standard_normal((1, 4, 640, D)).astype(np.float32)).to(DEV, torch.bfloat16)
                   for _ in range(4))
    entry = pf.autotune(q, k, v, pf.causal_mask, iters=3)
    fwd_c = entry["candidates"]["fwd [num_stages, tile_cfg]"]
    assert len(fwd_c) >= 4 and entry["bwd"]["num_stages"] in (2, 3, 4)
    tiles = {cfg[1] & 3 for cfg in map(json.loads, fwd_c)}
    assert tiles == {L.FA_TILE_Q1, L.FA_TILE_Q2, L.FA_TILE_HEADS2, 0}  # every launch shape was measured
    assert any(cfg[1] & L.FA_TILE_KV_HALVES for cfg in map(json.loads, fwd_c))
    assert (tmp_path / "tune.json").exists()

    KT.clear_memory_cache()  # the planner reads the entry back from the file
    plan = FA._Plan(q, k, v, pf.causal_mask, None, None, 64, 64, None, None, True)
    assert plan.tuned["fwd"] == entry["fwd"] and plan.tuned["bwd"] == entry["bwd"]
    assert (plan.fwd_stages, plan.fwd_tile_cfg, plan.bwd_stages) == (
        entry["fwd"]["num_stages"], entry["fwd"]["tile_cfg"], entry["bwd"]["num_stages"])

    o_tuned, lse_tuned = pf.flash_attention_fwd(q, k, v, pf.causal_mask)
    explicit = FA._Plan(q, k, v, pf.causal_mask, None, None, 64, 64, 0, None, True)
    explicit.fwd_stages, explicit.fwd_tile_cfg = entry["fwd"]["num_stages"], entry["fwd"]["tile_cfg"]
    o_exp, lse_exp = FA._run_fwd(explicit, q, k, v)
    assert torch.equal(o_tuned, o_exp) and torch.equal(lse_tuned, lse_exp)

    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = pf.flash_attention(qq, kk, vv, pf.causal_mask)
    grads = torch.autograd.grad(o, (qq, kk, vv), do)
    torch.cuda.synchronize()
    FA.check_device_status(DEV)
    qf, kf, vf, dof = (t.float().cpu().numpy().astype(np.float64) for t in (q, k, v, do))
    ro, rl = O.mha_reference(qf, kf, vf, O.causal)
    rg = O.attention_bwd(qf, kf, vf, ro, rl, dof, O.causal)
    assert_close("o", o.detach().float().cpu().numpy(), ro)
    for n, a, b in zip(("dq", "dk", "dv"), grads, rg):
        assert_close(n, a.float().cpu().numpy(), b)


@pytest.mark.parametrize("tile_cfg", [1 | 4, 1 | 8, 2 | 4, 2, 3 | 4, 3 | 8, 3, 1 | 4 | 16, 1 | 8 | 16, 2 | 16, 3 | 8 | 16,
                                      64 | 4, 64 | 8, 64])
def test_forward_launch_shapes_agree(tile_cfg):
    """Every forward launch shape computes the same attention (ragged length; grouped
    queries with two query heads per K/V head, so head pairs share their K/V loads)."""
    rng = np.random.default_rng(tile_cfg)
    q = torch.from_numpy(rng.standard_normal((2, 4, 700, 128)).astype(np.float32)).to(DEV, torch.bfloat16)
    k, v = (torch.from_numpy(rng.standard_normal((2, 2, 700, 128)).astype(np.float32)).to(DEV, torch.bfloat16)
            for _ in range(2))
    plan = FA._Plan(q, k, v, pf.causal_mask, None, None, 64, 64, 0, None, False)
    plan.fwd_tile_cfg = tile_cfg
    o, lse = FA._run_fwd(plan, q, k, v)
    torch.cuda.synchronize()
    FA.check_device_status(DEV)
    qf = q.float().cpu().numpy().astype(np.float64)
    kf, vf = (np.repeat(t.float().cpu().numpy().astype(np.float64), 2, axis=1) for t in (k, v))
    ro, rl = O.mha_reference(qf, kf, vf, O.causal)
    assert_close("o", o.float().cpu().numpy(), ro)
    np.testing.assert_allclose(lse.cpu().numpy(), rl, atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("tile_cfg", [3 | 4, 3 | 8, 0, 3 | 4 | 16, 1 | 4 | 16, 1 | 8 | 16, 64 | 4, 64 | 8])
@pytest.mark.parametrize("case", ["tiles_softcap_d64", "lambda_d128", "causal_d128", "window_alibi_d128"])
def test_head_pair_launch_shape(tile_cfg, case):
    """One Q tile of two heads per CTA with two distinct K/V heads per entry (K0, K1, V0, V1
    in the ring): irregular tile tables, an evaluated lambda mask and plain causal, against
    the oracle (tile_cfg 0 lets the launcher choose; it picks head pairs for the first two)."""
    T, D = (1000, 64) if case == "tiles_softcap_d64" else (768, 128)
    rng = np.random.default_rng(T + tile_cfg)
    q, k, v = (torch.from_numpy(rng.standard_normal((1, 4, T, D)).astype(np.float32)).to(DEV, torch.bfloat16)
               for _ in range(3))
    score, omods = None, ()
    if case == "tiles_softcap_d64":
        table = (rng.random((8, 8)) < 0.4).astype(np.uint8)
        np.fill_diagonal(table, 1)
        mm = pf.and_masks(pf.causal_mask, pf.tile_mask(table, 128))
        om = O.and_(O.causal, O.tile_table(table, 128))
        score, omods = pf.softcap_score_mod(30.0), (O.softcap(30.0),)
    elif case == "window_alibi_d128":
        mm, om = pf.sliding_window_mask(300, 0), O.sliding_window(300, 0)
        score, omods = pf.alibi_score_mod(4), (O.alibi(O.alibi_slopes(4)),)
    elif case == "lambda_d128":
        mm = om = lambda qi, ki: (((qi * 7 + ki * 3) % 11 < 4) | (qi == ki)) & (qi >= ki)  # noqa: E731
    else:
        mm, om = pf.causal_mask, O.causal
    plan = FA._Plan(q, k, v, mm, score, None, 64, 64, 0, None, False)
    plan.fwd_tile_cfg = tile_cfg
    o, lse = FA._run_fwd(plan, q, k, v)
    torch.cuda.synchronize()
    FA.check_device_status(DEV)
    qf, kf, vf = (t.float().cpu().numpy().astype(np.float64) for t in (q, k, v))
    ro, rl = O.mha_reference(qf, kf, vf, om, omods)
    assert_close("o", o.float().cpu().numpy(), ro)
    fin = np.isfinite(rl)
    np.testing.assert_array_equal(np.isfinite(lse.cpu().numpy()), fin)
    np.testing.assert_allclose(lse.cpu().numpy()[fin], rl[fin], atol=2e-3, rtol=1e-4)
