"""JAX front end of the B200 engine: the reference's ``flash_attention`` as XLA FFI calls.

Requires jax/jaxlib and libflexattn_jax.so (built from flexattn_jax_ffi.cc, see
its header).  Not importable in an environment without jax.  Mirrors the
reference's custom_vjp structure (src/pallas_flexattn/flash_attn.py:464-504):
the forward returns o and keeps residuals (q, k, v, o, lse); the backward calls
the fused backward kernel.  Block tables come from the GPU block-mask kernel.
"""
from __future__ import annotations

import ctypes
import math
from functools import partial
from pathlib import Path

import jax
import jax.numpy as jnp
import numpy as np

_LIB = ctypes.cdll.LoadLibrary(str(Path(__file__).resolve().parent / "libflexattn_jax.so"))
for _name, _sym in (("flexattn_fwd", _LIB.FlexAttnFwd), ("flexattn_bwd", _LIB.FlexAttnBwd),
                    ("flexattn_block_mask", _LIB.FlexAttnBlockMask)):
    jax.ffi.register_ffi_target(_name, jax.ffi.pycapsule(_sym), platform="CUDA")

MASK_CAUSAL, MASK_WINDOW, MASK_DOCUMENT, MASK_TILE_TABLE = 1, 2, 4, 8
SCORE_ALIBI, SCORE_SOFTCAP, SCORE_REL_BIAS = 1, 2, 4
TILE = 128


def block_tables(mask_flags: int, B: int, Tq: int, Tkv: int, window=(-1, -1), doc=None, table=None,
                 table_block: int = 0, mode: int = 0):
    """GPU create_block_mask: (tile_class, kv_num, kv_idx, full_kv_num, full_kv_idx, q_num, q_idx, full_q_num,
    full_q_idx) for 128x128 tiles."""
    nq, nkv = math.ceil(Tq / TILE), math.ceil(Tkv / TILE)
    nb = B if (doc is not None and doc.ndim == 2 and doc.shape[0] > 1) else 1
    i32 = jnp.int32
    out = [jax.ShapeDtypeStruct((nb, nq, nkv), jnp.uint8),
           jax.ShapeDtypeStruct((nb, nq), i32), jax.ShapeDtypeStruct((nb, nq, nkv), i32),
           jax.ShapeDtypeStruct((nb, nq), i32), jax.ShapeDtypeStruct((nb, nq, nkv), i32),
           jax.ShapeDtypeStruct((nb, nkv), i32), jax.ShapeDtypeStruct((nb, nkv, nq), i32),
           jax.ShapeDtypeStruct((nb, nkv), i32), jax.ShapeDtypeStruct((nb, nkv, nq), i32)]
    doc = jnp.zeros((1,), i32) if doc is None else doc.astype(i32)
    table = jnp.zeros((1, 1), jnp.uint8) if table is None else table.astype(jnp.uint8)
    return jax.ffi.ffi_call("flexattn_block_mask", out)(
        doc, table, mask_flags=np.int32(mask_flags), window_left=np.int32(window[0]),
        window_right=np.int32(window[1]), table_block=np.int32(table_block), B=np.int32(B), Tq=np.int32(Tq),
        Tkv=np.int32(Tkv), block_size=np.int32(TILE), mode=np.int32(mode))


def _attrs(spec):
    return dict(mask_flags=np.int32(spec["mask_flags"]), window_left=np.int32(spec.get("window_left", -1)),
                window_right=np.int32(spec.get("window_right", -1)), table_block=np.int32(spec.get("table_block", 0)),
                score_flags=np.int32(spec.get("score_flags", 0)), softcap=np.float32(spec.get("softcap", 0.0)),
                scale=np.float32(spec["scale"]), block_size=np.int32(TILE), kernel=np.int32(0),
                num_stages=np.int32(spec.get("num_stages", 0)))


def _aux(spec):
    z32, z8, zf = jnp.zeros((1,), jnp.int32), jnp.zeros((1, 1), jnp.uint8), jnp.zeros((1,), jnp.float32)
    return (spec.get("doc", z32), spec.get("table", z8), spec.get("slopes", zf), spec.get("rel_bias", zf[None]))


@partial(jax.custom_vjp, nondiff_argnums=(3,))
def flash_attention(q, k, v, spec):
    """Attention with the registry mask/score described by `spec` (a dict of static parameters)."""
    return _fwd(q, k, v, spec)[0]


def _fwd(q, k, v, spec):
    B, H, Tq, D = q.shape
    tables = spec["tables"]
    out = [jax.ShapeDtypeStruct(q.shape, q.dtype), jax.ShapeDtypeStruct((B, H, Tq), jnp.float32)]
    return jax.ffi.ffi_call("flexattn_fwd", out)(q, k, v, *_aux(spec), *tables[1:], **_attrs(spec))


def _fwd_rule(q, k, v, spec):
    o, lse = _fwd(q, k, v, spec)
    return o, (q, k, v, o, lse)


def _bwd_rule(spec, res, do):
    q, k, v, o, lse = res
    B, H, Tq, D = q.shape
    pad = math.ceil(Tq / TILE) * TILE
    ws = 2 * ((B * H * pad * 4 + 255) // 256 * 256) + (B * H * Tq * D * 4 + 255) // 256 * 256
    out = [jax.ShapeDtypeStruct(q.shape, q.dtype), jax.ShapeDtypeStruct(k.shape, k.dtype),
           jax.ShapeDtypeStruct(v.shape, v.dtype), jax.ShapeDtypeStruct((ws,), jnp.uint8)]
    dq, dk, dv, _ = jax.ffi.ffi_call("flexattn_bwd", out)(q, k, v, o, lse, do, *_aux(spec), *spec["tables"][1:],
                                                          **_attrs(spec))
    return dq, dk, dv


flash_attention.defvjp(_fwd_rule, _bwd_rule)
