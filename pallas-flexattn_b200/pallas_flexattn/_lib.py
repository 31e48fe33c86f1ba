"""ctypes binding of libflexattn.so (the C ABI declared in include/flexattn.h).

The structures below mirror the header field for field.  Every call raises
``FlexAttnError`` with the library's message on a non-zero status.  The library
is required: there is no fallback implementation, so importing a compute entry
point without the built ``libflexattn.so`` fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

FA_OK, FA_ERR_INVALID, FA_ERR_UNSUPPORTED, FA_ERR_CUDA, FA_ERR_TIMEOUT = 0, 1, 2, 3, 4
FA_DTYPE_F32, FA_DTYPE_BF16 = 0, 1
FA_KERNEL_AUTO, FA_KERNEL_TC, FA_KERNEL_SIMT = 0, 1, 2
FA_MASK_CAUSAL, FA_MASK_WINDOW, FA_MASK_DOCUMENT, FA_MASK_TILE_TABLE, FA_MASK_DOC_SORTED = 1, 2, 4, 8, 16
FA_MASK_BITMASK = 32
FA_SCORE_ALIBI, FA_SCORE_SOFTCAP, FA_SCORE_REL_BIAS = 1, 2, 4
FA_BLOCK_MASK_EXACT, FA_BLOCK_MASK_REF9 = 0, 1
FA_NOALLOC_SCRATCH_BYTES = 64 << 20  # static scratch of fa_bwd_noalloc
FA_TILE_Q2, FA_TILE_Q1, FA_TILE_HEADS2, FA_TILE_SOFTMAX_CONCURRENT, FA_TILE_SOFTMAX_TURNS = 1, 2, 3, 4, 8
FA_TILE_ROWS_SPLIT, FA_TILE_ROWS_WHOLE, FA_TILE_KV_HALVES = 16, 32, 64

_i32p = C.POINTER(C.c_int32)


class FaMaskSpec(C.Structure):
    _fields_ = [
        ("flags", C.c_int32),
        ("window_left", C.c_int32),
        ("window_right", C.c_int32),
        ("doc_q", C.c_void_p),
        ("doc_kv", C.c_void_p),
        ("doc_stride_b", C.c_int64),
        ("tile_table", C.c_void_p),
        ("table_rows", C.c_int32),
        ("table_cols", C.c_int32),
        ("table_block", C.c_int32),
        ("q_offset", C.c_int32),
        ("kv_offset", C.c_int32),
        ("bit_index", C.c_void_p),
        ("bits", C.c_void_p),
        ("bit_rows", C.c_int32),
        ("bit_cols", C.c_int32),
    ]


class FaScoreSpec(C.Structure):
    _fields_ = [
        ("flags", C.c_int32),
        ("softcap", C.c_float),
        ("alibi_slopes", C.c_void_p),
        ("rel_bias", C.c_void_p),
        ("rel_bias_stride_h", C.c_int64),
        ("rel_bias_center", C.c_int32),
    ]


class FaBlockTables(C.Structure):
    _fields_ = [
        ("block_q", C.c_int32),
        ("block_kv", C.c_int32),
        ("nq", C.c_int32),
        ("nkv", C.c_int32),
        ("num_b", C.c_int32),
        ("num_h", C.c_int32),
        ("kv_num_blocks", C.c_void_p),
        ("kv_indices", C.c_void_p),
        ("full_kv_num_blocks", C.c_void_p),
        ("full_kv_indices", C.c_void_p),
        ("kv_cap", C.c_int32),
        ("q_num_blocks", C.c_void_p),
        ("q_indices", C.c_void_p),
        ("full_q_num_blocks", C.c_void_p),
        ("full_q_indices", C.c_void_p),
        ("q_cap", C.c_int32),
    ]


class FaTensor(C.Structure):
    _fields_ = [
        ("ptr", C.c_void_p),
        ("stride_b", C.c_int64),
        ("stride_h", C.c_int64),
        ("stride_t", C.c_int64),
    ]


class FaFwdParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int32),
        ("B", C.c_int32),
        ("H", C.c_int32),
        ("H_kv", C.c_int32),
        ("Tq", C.c_int32),
        ("Tkv", C.c_int32),
        ("D", C.c_int32),
        ("q", FaTensor),
        ("k", FaTensor),
        ("v", FaTensor),
        ("o", FaTensor),
        ("lse", C.c_void_p),
        ("scale", C.c_float),
        ("mask", FaMaskSpec),
        ("score", FaScoreSpec),
        ("blocks", FaBlockTables),
        ("kernel", C.c_int32),
        ("num_stages", C.c_int32),
        ("status", C.c_void_p),
        ("tile_cfg", C.c_int32),
    ]


class FaBwdParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int32),
        ("B", C.c_int32),
        ("H", C.c_int32),
        ("H_kv", C.c_int32),
        ("Tq", C.c_int32),
        ("Tkv", C.c_int32),
        ("D", C.c_int32),
        ("q", FaTensor),
        ("k", FaTensor),
        ("v", FaTensor),
        ("o", FaTensor),
        ("dout", FaTensor),
        ("dq", FaTensor),
        ("dk", FaTensor),
        ("dv", FaTensor),
        ("lse", C.c_void_p),
        ("scale", C.c_float),
        ("mask", FaMaskSpec),
        ("score", FaScoreSpec),
        ("blocks", FaBlockTables),
        ("kernel", C.c_int32),
        ("num_stages", C.c_int32),
        ("status", C.c_void_p),
        ("tile_cfg", C.c_int32),
    ]


class FaDecodeParams(C.Structure):
    _fields_ = [
        ("dtype", C.c_int32),
        ("B", C.c_int32),
        ("H", C.c_int32),
        ("H_kv", C.c_int32),
        ("Tq", C.c_int32),
        ("Tkv", C.c_int32),
        ("D", C.c_int32),
        ("q", FaTensor),
        ("k", FaTensor),
        ("v", FaTensor),
        ("o", FaTensor),
        ("lse", C.c_void_p),
        ("kv_lens", C.c_void_p),
        ("scale", C.c_float),
        ("mask", FaMaskSpec),
        ("score", FaScoreSpec),
        ("num_splits", C.c_int32),
        ("status", C.c_void_p),
    ]


class FaBlockMaskOut(C.Structure):
    _fields_ = [
        ("num_b", C.c_int32),
        ("nq", C.c_int32),
        ("nkv", C.c_int32),
        ("tile_class", C.c_void_p),
        ("kv_num_blocks", C.c_void_p),
        ("kv_indices", C.c_void_p),
        ("full_kv_num_blocks", C.c_void_p),
        ("full_kv_indices", C.c_void_p),
        ("q_num_blocks", C.c_void_p),
        ("q_indices", C.c_void_p),
        ("full_q_num_blocks", C.c_void_p),
        ("full_q_indices", C.c_void_p),
    ]


# name -> (restype, argtypes); the exported surface of include/flexattn.h
EXPORTS = {
    "fa_version": (C.c_char_p, []),
    "fa_last_error": (C.c_char_p, []),
    "fa_fwd": (C.c_int, [C.POINTER(FaFwdParams), C.c_void_p]),
    "fa_bwd_preprocess": (C.c_int, [C.POINTER(FaBwdParams), C.c_void_p, C.c_void_p, C.c_void_p]),
    "fa_bwd_workspace_size": (C.c_int, [C.POINTER(FaBwdParams), C.POINTER(C.c_size_t)]),
    "fa_bwd": (C.c_int, [C.POINTER(FaBwdParams), C.c_void_p, C.c_size_t, C.c_void_p]),
    "fa_bwd_noalloc": (C.c_int, [C.POINTER(FaBwdParams), C.c_void_p]),
    "fa_create_block_mask": (
        C.c_int,
        [C.POINTER(FaMaskSpec), C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
         C.POINTER(FaBlockMaskOut), C.c_void_p],
    ),
    "fa_block_tables_from_lists": (
        C.c_int,
        [C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
         C.POINTER(FaBlockMaskOut), C.c_void_p],
    ),
    "fa_decode_workspace_size": (C.c_int, [C.POINTER(FaDecodeParams), C.POINTER(C.c_size_t)]),
    "fa_decode": (C.c_int, [C.POINTER(FaDecodeParams), C.c_void_p, C.c_size_t, C.c_void_p]),
    "fa_lse_merge": (
        C.c_int,
        [C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p],
    ),
}

LIB_PATH = Path(os.environ.get("FLEXATTN_LIB", Path(__file__).resolve().parent / "libflexattn.so"))


class FlexAttnError(RuntimeError):
    """A libflexattn call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libflexattn error {code}: {msg}")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    """Load libflexattn.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python pallas-flexattn_b200/build.py` "
                "(there is no fallback implementation)"
            )
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in EXPORTS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int) -> None:
    if rc != FA_OK:
        raise FlexAttnError(rc, lib().fa_last_error().decode(errors="replace"))


def version() -> str:
    return lib().fa_version().decode()
