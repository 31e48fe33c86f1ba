"""The benchmark workloads: the five attention configurations, seeded synthetic inputs.

Each config fixes dtype, shape, mask_mod and score_mod, and draws
q/k/v/dO ~ N(0, 1) from a seed (cfg2 scales them by 1/sqrt(D)).  The document
lengths and the random tile table are drawn with numpy's default_rng(seed):

* cfg4: lengths ``rng.integers(256, 4097)`` until they reach S, the last one
  truncated (seed 0: 3523, 2702, 2219, 1292, 1438, 413, 544, 319, 929, 3005);
* cfg5: tile (qb, kb) kept when ``rng.random((nq, nkv)) < 0.25``, diagonal forced,
  then intersected with causal.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Callable, Optional

import numpy as np
import torch

from .mask_mod import and_masks, causal_mask, document_mask, sliding_window_mask, tile_mask
from .score_mod import alibi_score_mod, slice_heads, softcap_score_mod


def document_lengths(S: int, seed: int = 0, lo: int = 256, hi: int = 4096) -> list[int]:
    rng = np.random.default_rng(seed)
    out, tot = [], 0
    while tot < S:
        n = int(rng.integers(lo, hi + 1))
        n = min(n, S - tot)
        out.append(n)
        tot += n
    return out


def random_tile_table(n: int, density: float = 0.25, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    keep = rng.random((n, n)) < density
    np.fill_diagonal(keep, True)
    return keep.astype(np.uint8)


@dataclass
class Workload:
    name: str
    dtype: torch.dtype
    B: int
    H: int
    S: int
    D: int
    mask_mod: Optional[Callable] = None
    score_mod: Optional[Callable] = None
    input_scale: float = 1.0
    block_size: int = 128
    desc: str = ""
    extra: dict = field(default_factory=dict)

    def inputs(self, device, seed: int = 0, B: Optional[int] = None, H: Optional[int] = None):
        """q, k, v, dO on `device` (generated there with a seeded torch generator)."""
        B = B or self.B
        H = H or self.H
        g = torch.Generator(device=device).manual_seed(seed)
        shape = (B, H, self.S, self.D)
        out = []
        for _ in range(4):
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * self.input_scale
            out.append(t.to(self.dtype))
        return out

    def head_shard(self, rank: int, world: int) -> "Workload":
        """Rank `rank`'s share of the problem when its H heads are split evenly over `world`
        ranks (heads are independent: no exchange is needed).  Per-head score parameters
        (ALiBi slopes) follow their heads."""
        if self.H % world:
            raise ValueError(f"{self.name}: H={self.H} heads do not split over {world} ranks")
        n = self.H // world
        h0 = rank * n
        return replace(self, H=n, score_mod=slice_heads(self.score_mod, h0, h0 + n),
                       extra={**self.extra, "heads": (h0, h0 + n), "full_H": self.H})

    def fwd_flops(self, n_pairs: int, B: Optional[int] = None, H: Optional[int] = None) -> float:
        """Effective forward FLOPs: 4 * D * unmasked pairs per (b, h) * B * H."""
        return 4.0 * self.D * n_pairs * (B or self.B) * (H or self.H)


def count_pairs(mask_mod: Optional[Callable], Tq: int, Tkv: int, device="cpu", chunk: int = 1024) -> int:
    """Exact number of unmasked (q, kv) pairs of one (b, h), evaluated in row chunks."""
    if mask_mod is None:
        return Tq * Tkv
    kv = torch.arange(Tkv, device=device)[None, :]
    n = 0
    for r0 in range(0, Tq, chunk):
        q = torch.arange(r0, min(r0 + chunk, Tq), device=device)[:, None]
        n += int(torch.broadcast_to(mask_mod(q, kv), (q.shape[0], Tkv)).sum())
    return n


def get(cfg: int) -> Workload:
    if cfg == 1:
        return Workload("cfg1_causal_fp32_B1H4S512D64", torch.float32, 1, 4, 512, 64, causal_mask,
                        desc="causal, fp32, block 128")
    if cfg == 2:
        return Workload("cfg2_causal_bf16_B4H16S4096D128", torch.bfloat16, 4, 16, 4096, 128, causal_mask,
                        input_scale=1.0 / math.sqrt(128), desc="causal, inputs x 1/sqrt(D)")
    if cfg == 3:
        return Workload("cfg3_window1024_alibi_bf16_B2H32S8192D128", torch.bfloat16, 2, 32, 8192, 128,
                        sliding_window_mask(1024, 0), alibi_score_mod(32), desc="window 1024 causal + ALiBi")
    if cfg == 4:
        lens = document_lengths(16384, seed=0)
        return Workload("cfg4_document_causal_bf16_B1H32S16384D128", torch.bfloat16, 1, 32, 16384, 128,
                        and_masks(document_mask(lens), causal_mask), desc="document AND causal",
                        extra={"doc_lengths": lens})
    if cfg == 5:
        S, bs = 32768, 128
        table = random_tile_table(S // bs, 0.25, seed=0)
        return Workload("cfg5_softcap_sparse_bf16_B1H16S32768D64", torch.bfloat16, 1, 16, S, 64,
                        and_masks(causal_mask, tile_mask(table, bs)), softcap_score_mod(30.0),
                        desc="softcap 30, causal AND 25% random tiles", extra={"tile_table": table})
    raise ValueError(f"unknown config {cfg}")
