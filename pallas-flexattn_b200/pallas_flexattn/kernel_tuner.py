"""Kernel configuration and autotuning (reference: src/pallas_flexattn/kernel_tuner.py).

``get_optimal_params`` / ``get_kernel_config`` / ``print_kernel_config`` keep the
reference's contract and table (kernel_tuner.py:11-148): a cached pure function
of (seq_len, head_dim, use_block_sparsity) returning (block_r, block_c,
num_warps, num_stages).  On this engine the table's ``block_r``/``block_c``
size the tiles of the generic kernels; the tcgen05 kernels always use 128x128.

``autotune`` replaces the reference's static choice with measurement: it times
each candidate K/V pipeline depth of the tcgen05 forward with CUDA events on the
caller's inputs, keeps the fastest, and caches it in memory and in a JSON file
keyed by (GPU name, dtype, B, H, Tq, Tkv, D, mask key, score flags).
"""
from __future__ import annotations

import functools
import json
import os
from pathlib import Path
from typing import Dict, Optional, Sequence, Tuple

DEFAULT_BLOCK_R = 64
DEFAULT_BLOCK_C = 64
DEFAULT_NUM_WARPS = 4
DEFAULT_NUM_STAGES = 3


@functools.lru_cache(maxsize=128)
def get_optimal_params(seq_len: int, head_dim: int = 64, use_block_sparsity: bool = False) -> Tuple[int, int, int, int]:
    """(block_r, block_c, num_warps, num_stages) for a sequence length and head dim."""
    if seq_len <= 256:
        block_r, block_c, num_warps, num_stages = 32, 32, 4, 2
    elif seq_len <= 512:
        block_r, block_c, num_warps, num_stages = 64, 64, 4, 3
    elif seq_len <= 2048:
        block_r, block_c, num_warps, num_stages = 128, 64, 4, 3
    elif seq_len <= 4096:
        block_r, block_c, num_warps, num_stages = 128, 128, 8, 4
    else:
        block_r, block_c, num_warps, num_stages = 128, 128, 8, 5
    if head_dim > 128:
        block_r, block_c, num_stages = min(block_r, 64), min(block_c, 64), min(num_stages, 3)
    elif head_dim <= 32:
        num_stages = max(num_stages, 4)
    if use_block_sparsity:
        block_r, block_c = min(block_r, 64), min(block_c, 64)
    return block_r, block_c, num_warps, num_stages


def get_kernel_config(batch_size: int, num_heads: int, seq_len: int, head_dim: int,
                      mask_type: Optional[str] = None) -> Dict[str, int]:
    """Complete kernel configuration dictionary (kernel_tuner.py:68-101)."""
    use_block_sparsity = mask_type in ("causal", "sliding_window")
    block_r, block_c, num_warps, num_stages = get_optimal_params(seq_len, head_dim, use_block_sparsity)
    return {
        "batch_size": batch_size,
        "num_heads": num_heads,
        "seq_len": seq_len,
        "head_dim": head_dim,
        "block_r": block_r,
        "block_c": block_c,
        "num_warps": num_warps,
        "num_stages": num_stages,
    }


def print_kernel_config(batch_size: int, num_heads: int, seq_len: int, head_dim: int,
                        mask_type: Optional[str] = None) -> None:
    """Print the kernel configuration (kernel_tuner.py:104-148)."""
    c = get_kernel_config(batch_size, num_heads, seq_len, head_dim, mask_type)
    bar = "=" * 70
    lines = [bar, "FlexAttention (B200) Kernel Configuration", bar, "Input Configuration:",
             f"  Batch size (B):   {c['batch_size']}", f"  Num heads (H):    {c['num_heads']}",
             f"  Seq length (T):   {c['seq_len']}", f"  Head dim (D):     {c['head_dim']}"]
    if mask_type:
        lines.append(f"  Mask type:        {mask_type}")
    lines += ["", "Kernel Parameters:", f"  BLOCK_R (block_r):      {c['block_r']}",
              f"  BLOCK_C (block_c):      {c['block_c']}", f"  NUM_WARPS:              {c['num_warps']}",
              f"  NUM_STAGES:             {c['num_stages']}", "", "Usage:",
              "  from pallas_flexattn import flash_attention", "  out = flash_attention(", "      q, k, v,",
              f"      block_r={c['block_r']},", f"      block_c={c['block_c']},",
              f"      num_warps={c['num_warps']},", f"      num_stages={c['num_stages']},", "  )", bar]
    print("\n".join(lines))


# ---------------------------------------------------------------------------- measured autotuning
_CACHE: Dict[str, dict] = {}
CACHE_PATH = Path(os.environ.get("FLEXATTN_TUNE_CACHE", Path.home() / ".cache" / "flexattn_b200_tune.json"))


def _load_cache() -> None:
    if not _CACHE and CACHE_PATH.exists():
        try:
            _CACHE.update(json.loads(CACHE_PATH.read_text()))
        except (OSError, ValueError):
            pass


def _save_cache() -> None:
    try:
        CACHE_PATH.parent.mkdir(parents=True, exist_ok=True)
        CACHE_PATH.write_text(json.dumps(_CACHE, indent=1, sort_keys=True))
    except OSError:
        pass


def tune_key(q, k, mask_mod=None, score_mod=None) -> str:
    import torch

    from .mask_mod import spec_of as mspec
    from .score_mod import spec_of as sspec

    ms, ss = mspec(mask_mod), sspec(score_mod)
    mk = None if ms is None else (ms.flags, ms.window_left, ms.window_right)
    sk = None if ss is None else ss.flags
    name = torch.cuda.get_device_name(q.device)
    return json.dumps([name, str(q.dtype), *q.shape, k.shape[1], k.shape[2], mk, sk])


def lookup(q, k, mask_mod=None, score_mod=None) -> Optional[dict]:
    _load_cache()
    return _CACHE.get(tune_key(q, k, mask_mod, score_mod))


def autotune(q, k, v, mask_mod=None, score_mod=None, block_mask=None,
             stages: Sequence[int] = (2, 3, 4), iters: int = 10, persist: bool = True) -> dict:
    """Time each candidate pipeline depth of the forward and cache the fastest.

    Returns ``{"num_stages": n, "ms": t, "candidates": {n: ms, ...}}``.
    """
    import torch

    from .flash_attn import flash_attention_fwd

    key = tune_key(q, k, mask_mod, score_mod)
    res: Dict[int, float] = {}
    for ns in stages:
        def run():
            flash_attention_fwd(q, k, v, mask_mod, num_stages=ns, score_mod=score_mod, block_mask=block_mask)
        try:
            run()
        except Exception:  # a depth the kernel cannot fit is skipped
            continue
        torch.cuda.synchronize(q.device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            run()
        end.record()
        end.synchronize()
        res[ns] = start.elapsed_time(end) / iters
    if not res:
        raise RuntimeError("autotune: no candidate configuration ran")
    best = min(res, key=res.get)
    entry = {"num_stages": best, "ms": res[best], "candidates": {str(k_): v_ for k_, v_ in res.items()}}
    _CACHE[key] = entry
    if persist:
        _save_cache()
    return entry
