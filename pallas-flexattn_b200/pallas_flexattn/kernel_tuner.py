"""Kernel configuration and autotuning (reference: src/pallas_flexattn/kernel_tuner.py).

``get_optimal_params`` / ``get_kernel_config`` / ``print_kernel_config`` keep the
reference's contract and table (kernel_tuner.py:11-148): a cached pure function
of (seq_len, head_dim, use_block_sparsity) returning (block_r, block_c,
num_warps, num_stages).  On this engine the table's ``block_r``/``block_c``
size the tiles of the generic kernels; the tcgen05 kernels always use 128x128.

``autotune`` replaces the reference's static choice with measurement: it times
the launch configurations of the tcgen05 forward (K/V pipeline depth, one or two
128-row Q tiles per CTA, softmax schedule) and backward (Q/dO pipeline depth)
with CUDA events on the caller's inputs, keeps the fastest of each pass, and
caches them in memory and in a JSON file keyed by (GPU name, dtype, B, H, Tq,
H_kv, Tkv, D, mask flags, score flags).  The attention entry points consult that
cache whenever ``num_stages`` is not given.
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
_LOADED_FROM: Optional[Path] = None


def cache_path() -> Path:
    """JSON file of tuned configurations ($FLEXATTN_TUNE_CACHE, else ~/.cache/flexattn_b200_tune.json)."""
    return Path(os.environ.get("FLEXATTN_TUNE_CACHE", Path.home() / ".cache" / "flexattn_b200_tune.json"))


def _load_cache() -> None:
    global _LOADED_FROM
    path = cache_path()
    if _LOADED_FROM == path:
        return
    _CACHE.clear()
    _LOADED_FROM = path
    if path.exists():
        try:
            _CACHE.update(json.loads(path.read_text()))
        except (OSError, ValueError):
            pass


def _save_cache() -> None:
    path = cache_path()
    try:
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(_CACHE, indent=1, sort_keys=True))
    except OSError:
        pass


def clear_memory_cache() -> None:
    """Forget the in-memory copy; the next lookup reads the cache file again."""
    global _LOADED_FROM
    _CACHE.clear()
    _LOADED_FROM = None


@functools.lru_cache(maxsize=16)
def _device_name(index: int) -> str:
    import torch

    return torch.cuda.get_device_name(index)


def make_key(device_name: str, dtype: str, q_shape, k_shape, mask_spec, score_spec) -> str:
    """Cache key: GPU name, dtype, (B, H, Tq, D), (H_kv, Tkv), mask flags and window, score flags."""
    mk = None if mask_spec is None else [mask_spec.flags, mask_spec.window_left, mask_spec.window_right]
    sk = None if score_spec is None else score_spec.flags
    return json.dumps([device_name, dtype, *map(int, q_shape), int(k_shape[1]), int(k_shape[2]), mk, sk])


def tune_key(q, k, mask_mod=None, score_mod=None) -> str:
    from .mask_mod import spec_of as mspec
    from .score_mod import spec_of as sspec

    return make_key(_device_name(q.device.index or 0), str(q.dtype), q.shape, k.shape, mspec(mask_mod),
                    sspec(score_mod))


def lookup(q, k, mask_mod=None, score_mod=None) -> Optional[dict]:
    """The tuned entry for this problem, or None."""
    _load_cache()
    return _CACHE.get(tune_key(q, k, mask_mod, score_mod))


def lookup_key(key: str) -> Optional[dict]:
    _load_cache()
    return _CACHE.get(key)


def _time(fn, iters: int) -> float:
    import torch

    fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / iters


def autotune(q, k, v, mask_mod=None, score_mod=None, block_mask=None, *,
             fwd_stages: Sequence[int] = (0, 2, 3, 4), bwd_stages: Sequence[int] = (2, 3, 4),
             iters: int = 10, persist: bool = True) -> dict:
    """Measure the launch configurations of both passes on the caller's inputs and cache the
    fastest of each (replacing the reference's static choice, kernel_tuner.py:11-65).

    Forward candidates: K/V pipeline depth (``fwd_stages``, entries in flight; 0 = as deep as
    shared memory holds) x launch shape (two 128-row Q tiles of one head sharing each K/V
    load, one Q tile, one Q tile of two heads walking the same kv list, or one Q tile whose kv
    list is split over the two sub-tiles) x softmax schedule
    x softmax warps per row (one, or two sharing its 128 columns) (concurrent warpgroups, or strict turns when there is no score_mod).
    Backward candidates: Q/dO pipeline depth (``bwd_stages``).  Each is timed with CUDA events
    over ``iters`` calls; depths the kernel cannot fit are skipped.  The entry is keyed by
    (GPU, dtype, shapes, mask flags and window, score flags); ``flash_attention`` and friends
    use it whenever the caller does not pass ``num_stages``.

    Returns ``{"fwd": {"num_stages", "tile_cfg", "ms"}, "bwd": {"num_stages", "ms"},
    "candidates": {...}}``.
    """
    import torch

    from . import _lib as L
    from .flash_attn import _Plan, _run_bwd, _run_fwd

    plan = _Plan(q, k, v, mask_mod, score_mod, block_mask, DEFAULT_BLOCK_R, DEFAULT_BLOCK_C, 0, None, need_bwd=True)
    if not plan.tc:
        raise ValueError("autotune: only the tcgen05 kernels (bf16, D in {64, 128}) have launch choices")
    key = tune_key(q, k, mask_mod, score_mod)
    scheds = [L.FA_TILE_SOFTMAX_CONCURRENT] + (
        [L.FA_TILE_SOFTMAX_TURNS] if plan.sspec.flags in (0, L.FA_SCORE_ALIBI) else [])
    fwd_res: Dict[str, float] = {}
    for ns in fwd_stages:
        shapes = (L.FA_TILE_Q2, L.FA_TILE_Q1, L.FA_TILE_KV_HALVES) + (
            (L.FA_TILE_HEADS2,) if q.shape[1] % 2 == 0 else ())
        for tiles in shapes:
            for sch in (scheds if tiles != L.FA_TILE_Q1 else [L.FA_TILE_SOFTMAX_CONCURRENT]):
                rows_opts = (L.FA_TILE_ROWS_WHOLE,) if tiles == L.FA_TILE_KV_HALVES else (
                    L.FA_TILE_ROWS_WHOLE, L.FA_TILE_ROWS_SPLIT)
                for rows in rows_opts:
                    cfg = tiles | sch | rows
                    plan.fwd_stages, plan.fwd_tile_cfg = ns, cfg
                    try:
                        ms = _time(lambda: _run_fwd(plan, q, k, v), iters)
                    except L.FlexAttnError:
                        continue
                    fwd_res[json.dumps([ns, cfg])] = ms
    if not fwd_res:
        raise RuntimeError("autotune: no forward candidate ran")
    best_f = json.loads(min(fwd_res, key=fwd_res.get))
    plan.fwd_stages, plan.fwd_tile_cfg = best_f
    o, lse = _run_fwd(plan, q, k, v)
    do = torch.randn_like(o)
    bwd_res: Dict[str, float] = {}
    for ns in bwd_stages:
        plan.bwd_stages = ns
        try:
            bwd_res[str(ns)] = _time(lambda: _run_bwd(plan, q, k, v, o, lse, do), iters)
        except L.FlexAttnError:
            continue
    if not bwd_res:
        raise RuntimeError("autotune: no backward candidate ran")
    best_b = int(min(bwd_res, key=bwd_res.get))
    entry = {"fwd": {"num_stages": best_f[0], "tile_cfg": best_f[1], "ms": fwd_res[json.dumps(best_f)]},
             "bwd": {"num_stages": best_b, "ms": bwd_res[str(best_b)]},
             "candidates": {"fwd [num_stages, tile_cfg]": fwd_res, "bwd num_stages": bwd_res}}
    _load_cache()
    _CACHE[key] = entry
    if persist:
        _save_cache()
    return entry
