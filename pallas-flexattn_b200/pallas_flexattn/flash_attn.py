"""FlexAttention on B200 — the reference's Python API over libflexattn.

Reference: src/pallas_flexattn/flash_attn.py.  Same entry points and argument
meaning:

* ``flash_attention(q, k, v, mask_mod=None, block_r=64, block_c=64,
  num_warps=4, num_stages=None, interpret=False)`` -> o, differentiable
  (the reference's default num_stages=3 is a Pallas pipelining knob; here None
  means "the measured choice", see below)
  (``torch.autograd``; the reference uses ``jax.custom_vjp`` with residuals
  ``(q, k, v, o, lse)``, flash_attn.py:464-504);
* ``flash_attention_fwd(...)`` -> ``(o, lse)`` (flash_attn.py:111-165);
* ``flash_attention_bwd(q, k, v, o, logsumexp, do, mask_mod, ...)`` ->
  ``(dq, dk, dv)`` (flash_attn.py:410-461);
* ``mha_reference(q, k, v, mask_mod=None)`` — the materialised formula
  (flash_attn.py:33-56), never used by the kernels.

Keyword-only additions: ``score_mod``, ``block_mask`` and ``scale``.

Tensors are torch CUDA tensors shaped (B, H, T, D), bf16 or fp32; K/V may have
fewer heads (grouped-query, forward only) and another length (cross attention).
The logsumexp is fp32 (the reference returns it in the input dtype, :144).
Rows with no unmasked key give o = 0 and lse = -inf (the reference gives NaN).

Kernel choice: bf16 with D in {64, 128} runs the tcgen05 kernels on 128x128
tiles (the MMA-native tile; ``block_r``/``block_c`` are then not used); other
dtypes and head dims run the generic CUDA-core kernels on ``block_r x block_c``
tiles.  ``num_stages`` sets the pipeline depth of the tcgen05 kernels (K/V
entries in flight in the forward, Q/dO tiles in the backward); left at None, the
measured autotuner's cached choice for the problem is used when there is one
(``kernel_tuner.autotune``), else the kernels' defaults.
``num_warps`` and ``interpret`` are accepted for signature compatibility; there
is no interpreter and no CPU path.
"""
from __future__ import annotations

import ctypes as C
import math
from collections import OrderedDict
from typing import Optional, Tuple

import torch

from . import _lib as L
from .block_mask import BlockMask, BlockTables, build_tables_from_spec
from .mask_mod import MaskMod, MaskSpec, evaluate_mask
from .mask_mod import spec_of as mask_spec_of
from .score_mod import ScoreMod, ScoreSpec
from .score_mod import spec_of as score_spec_of

DEFAULT_BLOCK_R = 64
DEFAULT_BLOCK_C = 64
DEFAULT_NUM_WARPS = 4
DEFAULT_NUM_STAGES = 3
TC_TILE = 128

_TABLE_CACHE: "OrderedDict[tuple, tuple[MaskSpec, BlockTables]]" = OrderedDict()
_TABLE_CACHE_MAX = 64
_STATUS: dict = {}


def device_status(device) -> torch.Tensor:
    """Per-device int32 the kernels set when a bounded device-side wait gives up."""
    device = torch.device(device)
    k = str(device)
    if k not in _STATUS:
        _STATUS[k] = torch.zeros(1, dtype=torch.int32, device=device)
    return _STATUS[k]


def check_device_status(device=None) -> None:
    """Synchronise and raise if any kernel on `device` reported a timeout."""
    device = torch.device(device if device is not None else "cuda")
    st = device_status(device)
    v = int(st.item())
    if v:
        st.zero_()
        raise L.FlexAttnError(v, "a device-side wait timed out (kernel aborted its tile)")


def clear_table_cache() -> None:
    _TABLE_CACHE.clear()


def _tables_for(spec: MaskSpec, B: int, Tq: int, Tkv: int, bq: int, bkv: int, device,
                offsets: tuple = (0, 0)) -> BlockTables:
    # The key names the spec's tensors (document ids, tile table, bitmask) by id(); the entry
    # keeps the spec, and so those tensors, alive, so no new tensor can take a cached id while
    # the entry exists and hit tables built for another mask.
    key = (spec.key(), B if spec.depends_on_batch else 1, Tq, Tkv, bq, bkv, str(device), tuple(offsets))
    hit = _TABLE_CACHE.get(key)
    if hit is None:
        bt = build_tables_from_spec(spec, B, Tq, Tkv, bq, bkv, device, offsets=offsets)
        _TABLE_CACHE[key] = (spec, bt)
        while len(_TABLE_CACHE) > _TABLE_CACHE_MAX:
            _TABLE_CACHE.popitem(last=False)
        return bt
    _TABLE_CACHE.move_to_end(key)
    return hit[1]


_DTYPES = {torch.bfloat16: L.FA_DTYPE_BF16, torch.float32: L.FA_DTYPE_F32}


def _fa_tensor(t: torch.Tensor) -> L.FaTensor:
    ft = L.FaTensor()
    ft.ptr = t.data_ptr()
    ft.stride_b, ft.stride_h, ft.stride_t = t.stride(0), t.stride(1), t.stride(2)
    return ft


def _last_contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _tc_ok_tensor(t: torch.Tensor) -> bool:
    es = t.element_size()
    return t.data_ptr() % 16 == 0 and all((s * es) % 16 == 0 for s in t.stride()[:3])


class _Plan:
    """Everything one forward/backward call needs: resolved specs, tables, kernel choice."""

    def __init__(self, q, k, v, mask_mod, score_mod, block_mask, block_r, block_c, num_stages, scale, need_bwd,
                 offsets: tuple = (0, 0)):
        if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
            raise ValueError("q, k, v must be (B, H, T, D)")
        if not (q.is_cuda and k.is_cuda and v.is_cuda):
            raise ValueError("flash_attention runs on CUDA tensors only (there is no CPU path)")
        if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
            raise ValueError(f"q/k/v must share dtype bf16 or fp32, got {q.dtype}/{k.dtype}/{v.dtype}")
        B, H, Tq, D = q.shape
        Bk, Hkv, Tkv, Dk = k.shape
        if Bk != B or Dk != D or tuple(v.shape) != (B, Hkv, Tkv, D):
            raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
        if H % Hkv:
            raise ValueError(f"H={H} must be a multiple of the K/V heads {Hkv}")
        if D % 8 or D > 256:
            raise NotImplementedError(f"head dim {D}: need a multiple of 8 up to 256")
        self.device = q.device
        self.B, self.H, self.Hkv, self.Tq, self.Tkv, self.D = B, H, Hkv, Tq, Tkv, D
        self.dtype = _DTYPES[q.dtype]
        self.scale = float(scale) if scale is not None else 1.0 / math.sqrt(D)

        if mask_mod is None and block_mask is not None and block_mask.mask_mod is not None:
            mask_mod = block_mask.mask_mod
        mspec = mask_spec_of(mask_mod)
        if mspec is None:
            # an arbitrary callable: evaluated once per geometry on the GPU into per-tile bitmasks
            mspec = evaluate_mask(mask_mod, Tq, Tkv, self.device, *offsets)
        sspec = score_spec_of(score_mod)
        if sspec is None:
            raise NotImplementedError(
                "this score_mod has no registry entry; build it from alibi_score_mod, softcap_score_mod, "
                "relative_bias_score_mod or compose_score_mods")
        self.mspec, self.sspec = mspec, sspec

        tc = (self.dtype == L.FA_DTYPE_BF16 and D in (64, 128)
              and all(_tc_ok_tensor(t) for t in (q, k, v)))
        if block_mask is not None:
            bt = block_mask.device_tables(self.device)
            tc = tc and bt.block_q == TC_TILE and bt.block_kv == TC_TILE
        else:
            bq, bkv = (TC_TILE, TC_TILE) if tc else (int(block_r), int(block_c))
            bt = _tables_for(mspec, B, Tq, Tkv, bq, bkv, self.device, offsets)
        if bt.nq != math.ceil(Tq / bt.block_q) or bt.nkv != math.ceil(Tkv / bt.block_kv):
            raise ValueError(f"block mask for ({bt.nq} x {bt.nkv}) tiles does not match Tq={Tq}, Tkv={Tkv}")
        if bt.num_b not in (1, B):
            raise ValueError("block mask batch dimension does not match B")
        self.tables = bt
        # AUTO lets the library take the tcgen05 kernel of each pass when it applies.
        self.tc = tc
        self.kernel = L.FA_KERNEL_AUTO if tc else L.FA_KERNEL_SIMT
        # Launch configuration: an explicit num_stages sets the pipeline depth of both passes;
        # without one, the measured autotuner's entry for this problem (if any) supplies the
        # depth of each pass and the forward's launch shape, else the kernels' defaults.
        self.num_stages = int(num_stages) if num_stages else 0
        self.fwd_stages = self.bwd_stages = self.num_stages
        self.fwd_tile_cfg = 0
        self.tuned = None
        if num_stages is None and tc:
            from .kernel_tuner import make_key, lookup_key, _device_name

            self.tuned = lookup_key(make_key(_device_name(self.device.index or 0), str(q.dtype), q.shape, k.shape,
                                             mspec, sspec))
            if self.tuned is not None:
                self.fwd_stages = int(self.tuned["fwd"]["num_stages"])
                self.fwd_tile_cfg = int(self.tuned["fwd"]["tile_cfg"])
                self.bwd_stages = int(self.tuned["bwd"]["num_stages"])
        self.c_mask = mspec.to_c(self.device, Tq, Tkv, *offsets)
        self.c_score = sspec.to_c(self.device, H, Tq, Tkv)
        self.c_tables = bt.to_c()
        self.status = device_status(self.device)
        self._templates = {}  # parameter structs with everything but the tensors, per pass
        self._ws_bytes = None

    def template(self, cls):
        """A filled parameter struct of type `cls` (FaFwdParams / FaBwdParams) without tensors;
        each call copies it (a memcpy) instead of setting every field again."""
        t = self._templates.get(cls)
        if t is None:
            t = cls()
            self._fill(t)
            self._templates[cls] = t
        return cls.from_buffer_copy(t)

    def _fill(self, p):
        p.dtype = self.dtype
        p.B, p.H, p.H_kv, p.Tq, p.Tkv, p.D = self.B, self.H, self.Hkv, self.Tq, self.Tkv, self.D
        p.scale = self.scale
        p.mask = self.c_mask
        p.score = self.c_score
        p.blocks = self.c_tables
        p.kernel = self.kernel
        p.num_stages = self.num_stages
        p.tile_cfg = 0
        p.status = self.status.data_ptr()


def _run_fwd(plan: _Plan, q, k, v) -> Tuple[torch.Tensor, torch.Tensor]:
    o = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    p = plan.template(L.FaFwdParams)
    p.num_stages, p.tile_cfg = plan.fwd_stages, plan.fwd_tile_cfg
    p.q, p.k, p.v, p.o = _fa_tensor(q), _fa_tensor(k), _fa_tensor(v), _fa_tensor(o)
    p.lse = lse.data_ptr()
    with torch.cuda.device(q.device):
        L.check(L.lib().fa_fwd(C.byref(p), torch.cuda.current_stream(q.device).cuda_stream))
    return o, lse


def _run_bwd(plan: _Plan, q, k, v, o, lse, do) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    if not (_tc_ok_tensor(do) and _tc_ok_tensor(o)):
        o, do = o.contiguous(), do.contiguous()
    dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    lse = lse.to(torch.float32).contiguous()
    p = plan.template(L.FaBwdParams)
    p.num_stages = plan.bwd_stages
    p.q, p.k, p.v, p.o, p.dout = _fa_tensor(q), _fa_tensor(k), _fa_tensor(v), _fa_tensor(o), _fa_tensor(do)
    p.dq, p.dk, p.dv = _fa_tensor(dq), _fa_tensor(dk), _fa_tensor(dv)
    p.lse = lse.data_ptr()
    lib = L.lib()
    if plan._ws_bytes is None:  # a function of the shape alone
        nbytes = C.c_size_t(0)
        L.check(lib.fa_bwd_workspace_size(C.byref(p), C.byref(nbytes)))
        plan._ws_bytes = max(int(nbytes.value), 16)
    ws = torch.empty(plan._ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        L.check(lib.fa_bwd(C.byref(p), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(q.device).cuda_stream))
    return dq, dk, dv


def flash_attention_fwd(q, k, v, mask_mod: Optional[MaskMod] = None, block_r: int = DEFAULT_BLOCK_R,
                        block_c: int = DEFAULT_BLOCK_C, num_warps: int = DEFAULT_NUM_WARPS,
                        num_stages: Optional[int] = None, interpret: bool = False, *,
                        score_mod: Optional[ScoreMod] = None, block_mask: Optional[BlockMask] = None,
                        scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Flash attention forward pass: returns (o, lse)."""
    del num_warps, interpret
    q, k, v = _last_contig(q), _last_contig(k), _last_contig(v)
    plan = _Plan(q, k, v, mask_mod, score_mod, block_mask, block_r, block_c, num_stages, scale, need_bwd=False)
    return _run_fwd(plan, q, k, v)


def flash_attention_bwd(q, k, v, o, logsumexp, do, mask_mod: Optional[MaskMod] = None,
                        block_r: int = DEFAULT_BLOCK_R, block_c: int = DEFAULT_BLOCK_C,
                        num_warps: int = DEFAULT_NUM_WARPS, num_stages: Optional[int] = None,
                        interpret: bool = False, *, score_mod: Optional[ScoreMod] = None,
                        block_mask: Optional[BlockMask] = None,
                        scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Flash attention backward pass: returns (dq, dk, dv)."""
    del num_warps, interpret
    q, k, v, o, do = (_last_contig(t) for t in (q, k, v, o, do))
    plan = _Plan(q, k, v, mask_mod, score_mod, block_mask, block_r, block_c, num_stages, scale, need_bwd=True)
    return _run_bwd(plan, q, k, v, o, logsumexp, do)


class _FlashAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cfg):
        q, k, v = _last_contig(q), _last_contig(k), _last_contig(v)
        need_bwd = any(t.requires_grad for t in (q, k, v))
        plan = _Plan(q, k, v, *cfg, need_bwd=need_bwd)
        o, lse = _run_fwd(plan, q, k, v)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.plan = plan
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _run_bwd(ctx.plan, q, k, v, o, lse, _last_contig(do))
        return dq, dk, dv, None


def flash_attention(q, k, v, mask_mod: Optional[MaskMod] = None, block_r: int = DEFAULT_BLOCK_R,
                    block_c: int = DEFAULT_BLOCK_C, num_warps: int = DEFAULT_NUM_WARPS,
                    num_stages: Optional[int] = None, interpret: bool = False, *,
                    score_mod: Optional[ScoreMod] = None, block_mask: Optional[BlockMask] = None,
                    scale: Optional[float] = None) -> torch.Tensor:
    """Flash attention with a custom backward pass; returns o."""
    del num_warps, interpret
    cfg = (mask_mod, score_mod, block_mask, block_r, block_c, num_stages, scale)
    return _FlashAttentionFn.apply(q, k, v, cfg)


def mha_reference(q, k, v, mask_mod: Optional[MaskMod] = None, *, score_mod: Optional[ScoreMod] = None,
                  scale: Optional[float] = None) -> torch.Tensor:
    """Reference multi-head attention that materialises the T x T matrix.

    softmax(mask(score_mod(Q K^T * scale))) V in fp32, cast back to q's dtype.
    As in the reference (flash_attn.py:45-56), a fully masked row yields NaN.
    """
    B, H, Tq, D = q.shape
    Tkv = k.shape[2]
    if k.shape[1] != H:
        rep = H // k.shape[1]
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    s = 1.0 / math.sqrt(D) if scale is None else scale
    logits = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) * s
    dev = q.device
    q_idx = torch.arange(Tq, device=dev)[:, None]
    kv_idx = torch.arange(Tkv, device=dev)[None, :]
    if score_mod is not None:
        b_idx = torch.arange(B, device=dev)[:, None, None, None]
        h_idx = torch.arange(H, device=dev)[None, :, None, None]
        logits = score_mod(logits, b_idx, h_idx, q_idx, kv_idx)
    if mask_mod is not None:
        logits = torch.where(mask_mod(q_idx, kv_idx), logits, torch.tensor(-math.inf, device=dev))
    probs = torch.softmax(logits, dim=-1)
    return torch.einsum("bhqk,bhkd->bhqd", probs, v.float()).to(q.dtype)
