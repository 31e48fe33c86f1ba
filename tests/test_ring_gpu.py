"""Context-parallel ring on 2 GPUs (NCCL), forward and backward, against fp32.

Each rank holds its zig-zag share of q/k/v/dO; the ring exchanges K/V (and, in the
backward, the travelling fp32 dK/dV accumulators) with NCCL send/recv, merges partial
outputs with fa_lse_merge and runs one fused backward call per unmasked chunk pair.  Rank 0
gathers o, dq, dk and dv and compares them, every element, with the chunked fp32 reference
of the whole sequence (tests/torch_reference.py) under the suite's tolerance.  Needs at
least 2 GPUs; skipped otherwise.  NVLS is off (plain peer transfers only).
"""
import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import pallas_flexattn as pf
from pallas_flexattn import ring
from tolerance import stats
from torch_reference import torch_reference

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _softcap(raw, hi, qi, ki):
    t = torch.tanh(raw / 30.0)
    return 30.0 * t, 1 - t * t


CASES = {
    "causal_d128": dict(T=2048, D=128, mask=pf.causal_mask, score=None, ref_score=None),
    "softcap_window_d64": dict(T=4096, D=64, mask=pf.sliding_window_mask(700, 0), score=pf.softcap_score_mod(30.0),
                               ref_score=_softcap),
}


def _worker(rank, port, case, out_dir):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        c = CASES[case]
        g = torch.Generator(device="cpu").manual_seed(5)
        q, k, v, do = (torch.randn(1, 2, c["T"], c["D"], generator=g).to(dev, torch.bfloat16) for _ in range(4))
        mine = [ring.split_zigzag(x, rank, WORLD).contiguous() for x in (q, k, v, do)]
        qq, kk, vv = (t.clone().requires_grad_(True) for t in mine[:3])
        o = ring.ring_attention(qq, kk, vv, c["mask"], c["score"])
        grads = torch.autograd.grad(o, (qq, kk, vv), mine[3])
        torch.cuda.synchronize(dev)
        full = {}
        for name, t in zip(("o", "dq", "dk", "dv"), (o.detach(), *grads)):
            bufs = [torch.empty_like(t) for _ in range(WORLD)]
            dist.all_gather(bufs, t.contiguous())
            full[name] = ring.gather_zigzag(bufs, WORLD)
        if rank == 0:
            ref = torch_reference(q, k, v, do, c["mask"], c["ref_score"])
            res = {n: stats(full[n].float().cpu().numpy(), r.float().cpu().numpy())
                   for n, r in zip(("o", "dq", "dk", "dv"), (ref[0], *ref[2:]))}
            torch.save(res, os.path.join(out_dir, "result.pt"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"error{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("case", list(CASES))
def test_ring_nccl_forward_backward_against_fp32(tmp_path, case):
    mp.start_processes(_worker, args=(_free_port(), case, str(tmp_path)), nprocs=WORLD, start_method="spawn",
                       join=True)
    r = torch.load(tmp_path / "result.pt")
    for name in ("o", "dq", "dk", "dv"):
        assert r[name]["pass"], f"{name}: {r[name]}"
