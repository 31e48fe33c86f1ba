"""Context-parallel ring forward on 2 GPUs (NCCL) against single-GPU attention.

Each rank holds its zig-zag share of q/k/v; the ring exchanges K/V with NCCL send/recv
and merges partial results with fa_lse_merge.  Rank 0 compares the gathered output with
flash_attention_fwd over the whole sequence on one GPU (same kernels, so the only
difference is the split and the log-sum-exp merge).  Needs at least 2 GPUs; skipped
otherwise.
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

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CASES = {
    "causal_d128": dict(T=2048, D=128, mask=lambda T: pf.causal_mask, score=None),
    "softcap_window_d64": dict(T=4096, D=64, mask=lambda T: pf.sliding_window_mask(700, 0),
                               score=pf.softcap_score_mod(30.0)),
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
        q, k, v = (torch.randn(1, 2, c["T"], c["D"], generator=g).to(dev, torch.bfloat16) for _ in range(3))
        mask = c["mask"](c["T"])
        mine = [ring.split_zigzag(x, rank, WORLD).contiguous() for x in (q, k, v)]
        stats = ring.RingStats()
        o, lse = ring.ring_attention_fwd(*mine, mask, c["score"], stats=stats)
        torch.cuda.synchronize(dev)
        os_ = [torch.empty_like(o) for _ in range(WORLD)]
        ls_ = [torch.empty_like(lse) for _ in range(WORLD)]
        dist.all_gather(os_, o)
        dist.all_gather(ls_, lse)
        if rank == 0:
            o_ring = ring.gather_zigzag(os_, WORLD)
            lse_ring = ring.gather_zigzag([x[..., None] for x in ls_], WORLD)[..., 0]
            o_ref, lse_ref = pf.flash_attention_fwd(q, k, v, mask, score_mod=c["score"])
            torch.save({"o": o_ring.cpu(), "lse": lse_ring.cpu(), "o_ref": o_ref.cpu(), "lse_ref": lse_ref.cpu(),
                        "computed": stats.pairs_computed, "skipped": stats.pairs_skipped},
                       os.path.join(out_dir, "result.pt"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"error{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("case", list(CASES))
def test_ring_nccl_matches_single_gpu(tmp_path, case):
    mp.start_processes(_worker, args=(_free_port(), case, str(tmp_path)), nprocs=WORLD, start_method="spawn",
                       join=True)
    r = torch.load(tmp_path / "result.pt")
    o, o_ref = r["o"].float(), r["o_ref"].float()
    # bf16 outputs of two different summation orders: within a couple of bf16 ulps
    assert float((o - o_ref).abs().max()) <= 2e-2
    assert float((o - o_ref).norm() / o_ref.norm()) <= 5e-3
    fin = torch.isfinite(r["lse_ref"])
    assert torch.equal(fin, torch.isfinite(r["lse"]))
    assert float((r["lse"][fin] - r["lse_ref"][fin]).abs().max()) <= 1e-3
    assert r["computed"] > 0
