"""Context-parallel ring schedule on CPU ranks (gloo), world sizes 2 and 3, forward and backward.

The ring (pallas_flexattn/ring.py) takes its partial-attention and merge functions as
arguments; here they are an fp64 torch reference with global-position masks and the torch
log-sum-exp merge, so the test covers the schedule itself: zig-zag ownership, the K/V
exchange, skipping of fully masked chunk pairs and the merge order.  The result is compared
with full-sequence attention; the backward (K/V and the travelling dK/dV accumulators)
with fp64 autograd through full-sequence attention.  A fault test makes one rank raise before the ring starts and
checks that its peer fails with an error (process-group timeout) instead of hanging.
"""
import datetime
import math
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import pallas_flexattn as pf
from pallas_flexattn import ring


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def ref_partial(q, k, v, mask_mod, score_mod, q_offset, kv_offset):
    """(o, lse) of q against k/v in fp64, masks at global positions; empty rows: o = 0, lse = -inf."""
    del score_mod
    qd, kd, vd = q.double(), k.double(), v.double()
    s = torch.einsum("bhqd,bhkd->bhqk", qd, kd) / math.sqrt(q.shape[-1])
    qi = torch.arange(q.shape[2])[:, None] + q_offset
    ki = torch.arange(k.shape[2])[None, :] + kv_offset
    allowed = torch.ones_like(qi >= ki) if mask_mod is None else torch.broadcast_to(mask_mod(qi, ki), s.shape[-2:])
    s = s.masked_fill(~allowed, -math.inf)
    lse = torch.logsumexp(s, dim=-1)
    p = torch.where(torch.isfinite(lse)[..., None], torch.exp(s - lse[..., None]), torch.zeros_like(s))
    o = torch.einsum("bhqk,bhkd->bhqd", p, vd)
    return o.float(), lse.float()


def ref_partial_bwd(q, k, v, o, lse, do, mask_mod, score_mod, q_offset, kv_offset):
    """(dq, dk, dv) of one chunk pair in fp64 from the final o and lse, masks at global positions."""
    del score_mod
    qd, kd, vd, od, dod = (t.double() for t in (q, k, v, o, do))
    sc = 1.0 / math.sqrt(q.shape[-1])
    s = torch.einsum("bhqd,bhkd->bhqk", qd, kd) * sc
    qi = torch.arange(q.shape[2])[:, None] + q_offset
    ki = torch.arange(k.shape[2])[None, :] + kv_offset
    allowed = torch.ones_like(qi >= ki) if mask_mod is None else torch.broadcast_to(mask_mod(qi, ki), s.shape[-2:])
    lse = lse.double()
    p = torch.where(allowed & torch.isfinite(lse)[..., None], torch.exp(s - lse[..., None]), torch.zeros_like(s))
    delta = (od * dod).sum(-1, keepdim=True)
    ds = p * (torch.einsum("bhqd,bhkd->bhqk", dod, vd) - delta)
    return ((ds @ kd) * sc).float(), ((ds.transpose(-1, -2) @ qd) * sc).float(), (p.transpose(-1, -2) @ dod).float()


def full_attention_fp64(q, k, v, mask_mod):
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) / math.sqrt(q.shape[-1])
    T = q.shape[2]
    if mask_mod is not None:
        s = s.masked_fill(~torch.broadcast_to(mask_mod(torch.arange(T)[:, None], torch.arange(T)[None, :]),
                                              s.shape[-2:]), -math.inf)
    return torch.softmax(s, -1).nan_to_num(0.0) @ v


MASKS = {
    "causal": lambda T: pf.causal_mask,
    "window": lambda T: pf.sliding_window_mask(5, 0),
    "document": lambda T: pf.and_masks(pf.document_mask([10, 7, T - 17]), pf.causal_mask),
}


def _worker(rank, world, port, mask_name, out_dir):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        T = 12 * world  # 2W chunks of 6 positions
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(1, 2, T, 8, generator=g) for _ in range(3))
        mask_mod = MASKS[mask_name](T)
        mine = [ring.split_zigzag(x, rank, world) for x in (q, k, v)]
        stats = ring.RingStats()
        o, lse = ring.ring_attention_fwd(*mine, mask_mod, attn_fn=ref_partial, merge_fn=ring.torch_merge, stats=stats)
        os_, ls_ = [torch.empty_like(o) for _ in range(world)], [torch.empty_like(lse) for _ in range(world)]
        dist.all_gather(os_, o)
        dist.all_gather(ls_, lse)
        if rank == 0:
            o_full = ring.gather_zigzag(os_, world)
            lse_full = ring.gather_zigzag([x[..., None] for x in ls_], world)[..., 0]
            o_ref, lse_ref = ref_partial(q, k, v, mask_mod, None, 0, 0)
            torch.save({"o": o_full, "lse": lse_full, "o_ref": o_ref, "lse_ref": lse_ref,
                        "computed": stats.pairs_computed, "skipped": stats.pairs_skipped, "steps": stats.steps},
                       os.path.join(out_dir, "result.pt"))
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"error{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("mask_name", ["causal", "window", "document"])
def test_ring_matches_full_attention(tmp_path, world, mask_name):
    mp.start_processes(_worker, args=(world, _free_port(), mask_name, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    r = torch.load(tmp_path / "result.pt")
    torch.testing.assert_close(r["o"], r["o_ref"], atol=1e-5, rtol=1e-5)
    fin = torch.isfinite(r["lse_ref"])
    assert torch.equal(fin, torch.isfinite(r["lse"]))
    torch.testing.assert_close(r["lse"][fin], r["lse_ref"][fin], atol=1e-5, rtol=1e-5)
    assert r["steps"] == world
    # rank 0 holds chunks (0, 2W-1); the pairs it visits are 2 own chunks x 2 held chunks x W steps
    assert r["computed"] + r["skipped"] == 4 * world
    if mask_name == "causal":
        assert r["skipped"] > 0  # kv chunks after both of rank 0's q chunks are never computed


def _bwd_worker(rank, world, port, mask_name, out_dir):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        T = 12 * world
        g = torch.Generator().manual_seed(1)
        q, k, v, do = (torch.randn(1, 2, T, 8, generator=g) for _ in range(4))
        mask_mod = MASKS[mask_name](T)
        mine = [ring.split_zigzag(x, rank, world) for x in (q, k, v, do)]
        before = [t.clone() for t in mine]
        o, lse = ring.ring_attention_fwd(*mine[:3], mask_mod, attn_fn=ref_partial, merge_fn=ring.torch_merge)
        stats = ring.RingStats()
        dq, dk, dv = ring.ring_attention_bwd(*mine[:3], o, lse, mine[3], mask_mod, attn_bwd_fn=ref_partial_bwd,
                                             stats=stats)
        # the exchange receives into the ring's own buffers: the caller's tensors are only read
        untouched = all(torch.equal(a, b) for a, b in zip(mine, before))
        parts = {}
        for name, t in (("dq", dq), ("dk", dk), ("dv", dv)):
            bufs = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(bufs, t)
            parts[name] = ring.gather_zigzag(bufs, world)
        if rank == 0:
            qd, kd, vd = (t.double().requires_grad_(True) for t in (q, k, v))
            ref = torch.autograd.grad(full_attention_fp64(qd, kd, vd, mask_mod), (qd, kd, vd), do.double())
            torch.save({**parts, "ref": [r.float() for r in ref], "steps": stats.steps,
                        "computed": stats.pairs_computed, "untouched": untouched},
                       os.path.join(out_dir, "result.pt"))
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"error{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("mask_name", ["causal", "window", "document"])
def test_ring_backward_matches_full_attention(tmp_path, world, mask_name):
    mp.start_processes(_bwd_worker, args=(world, _free_port(), mask_name, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    r = torch.load(tmp_path / "result.pt")
    for i, name in enumerate(("dq", "dk", "dv")):
        torch.testing.assert_close(r[name], r["ref"][i], atol=1e-5, rtol=1e-5, msg=name)
    assert r["steps"] == world and r["computed"] > 0
    assert r["untouched"], "the ring wrote into the caller's q/k/v/dO"


def test_zigzag_round_trip():
    x = torch.arange(2 * 3 * 24 * 4, dtype=torch.float32).reshape(2, 3, 24, 4)
    for world in (1, 2, 3, 4):
        parts = [ring.split_zigzag(x, r, world) for r in range(world)]
        assert all(p.shape[2] == 24 // world for p in parts)
        assert torch.equal(ring.gather_zigzag(parts, world), x)


def _fault_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise RuntimeError("injected failure on rank 1 before the ring")  # this rank never joins the exchange
    q = k = v = torch.randn(1, 1, 8, 4)
    try:
        ring.ring_attention_fwd(q, k, v, pf.causal_mask, attn_fn=ref_partial, merge_fn=ring.torch_merge)
        outcome = "completed"
    except Exception as e:  # the peer's exchange fails (closed connection or timeout)
        outcome = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(outcome)


def test_ring_peer_failure_surfaces_as_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    assert procs[1].exitcode != 0  # the injected failure
    outcome = (tmp_path / "rank0.txt").read_text()
    assert outcome.startswith("error"), outcome
