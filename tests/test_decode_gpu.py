"""GPU parity of the split-KV decode kernel (flash_attention_decode -> fa_decode) against
the CPU oracle's decode_reference, at the bf16 / fp32 tolerance of the attention tests
(|err| <= atol + 2^-8 |ref| element-wise and relative-L2 <= rtol; lse within 2e-3).

Cases cover single-token and multi-token decode, grouped-query heads up to the row limits
(128 for bf16 on the tcgen05 kernel, 64 for fp32 on the CUDA-core kernel), head dims 64 / 128 / 256, ragged per-sequence cache lengths (not multiples of the
64-row tile, down to Tq), chunkings with empty chunks, causal and sliding-window masks,
ALiBi and softcap (bf16 only: the softcap's tanh is the hardware approximation, about
2^-11 relative), fp32 inputs, and a cache stored as [B, T, H_kv, D] (strided heads).
"""
import math
import zlib

import numpy as np
import pytest
import torch

import pallas_flexattn as pf
from oracle import flexattn_oracle as O
from pallas_flexattn import _lib as L
from pallas_flexattn.flash_attn import check_device_status
from tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def close(name, got, ref, dtype):
    assert_close(name, got.detach().float().cpu().numpy(), ref, bf16=dtype == torch.bfloat16)


CASES = {
    # name: B, H, Hkv, Tq, Tkv, D, dtype, lens, mask, score, splits
    "mha_t1_d128": (2, 8, 8, 1, 1000, 128, torch.bfloat16, [1000, 517], None, None, 0),
    "gqa8_t1_causal": (3, 32, 4, 1, 2048, 128, torch.bfloat16, [2048, 1, 1300], "causal", None, 0),
    "gqa4_t4_window_alibi_d64": (2, 16, 4, 4, 777, 64, torch.bfloat16, [777, 130], "window", "alibi", 0),
    "mqa_t2_softcap_d256_splits5": (2, 4, 1, 2, 900, 256, torch.bfloat16, [2, 899], "causal", "softcap", 5),
    "rows64_d128": (1, 16, 1, 4, 1536, 128, torch.bfloat16, [1500], "causal", "both", 0),
    "rows128_d64": (2, 32, 1, 4, 1000, 64, torch.bfloat16, [1000, 260], "causal", None, 0),
    "rows96_d256_window": (1, 24, 1, 4, 700, 256, torch.bfloat16, [699], "window", None, 0),
    "fp32_rows64": (1, 32, 2, 4, 300, 64, torch.float32, [300], "causal", None, 0),
    "many_splits_empty_chunks": (2, 2, 2, 1, 4096, 64, torch.bfloat16, [65, 4096], None, None, 40),
    "one_chunk_writes_o_d128": (2, 16, 4, 2, 700, 128, torch.bfloat16, [700, 333], "causal", "alibi", 1),
    "one_chunk_writes_o_d64": (3, 8, 8, 1, 300, 64, torch.bfloat16, [300, 1, 129], None, None, 1),
    "no_lens_d64": (2, 8, 2, 3, 640, 64, torch.bfloat16, None, "causal", None, 0),
    "fp32_d64": (2, 4, 2, 2, 500, 64, torch.float32, [500, 77], "causal", "alibi", 0),
    "fp32_d128": (1, 8, 1, 1, 700, 128, torch.float32, [650], None, "alibi", 0),
    "fp32_d256": (1, 2, 2, 1, 300, 256, torch.float32, [300], "causal", None, 3),
}


def _mods(kind, H):
    if kind is None:
        return None, ()
    if kind == "alibi":
        return pf.alibi_score_mod(H), (O.alibi(O.alibi_slopes(H)),)
    if kind == "softcap":
        return pf.softcap_score_mod(15.0), (O.softcap(15.0),)
    return (pf.compose_score_mods(pf.alibi_score_mod(H), pf.softcap_score_mod(15.0)),
            (O.alibi(O.alibi_slopes(H)), O.softcap(15.0)))


def _masks(kind):
    if kind is None:
        return None, None
    if kind == "causal":
        return pf.causal_mask, O.causal
    return (pf.and_masks(pf.causal_mask, pf.sliding_window_mask(100, 0)),
            O.and_(O.causal, O.sliding_window(100, 0)))


def _inputs(B, H, Hkv, Tq, Tkv, D, dtype, seed, layout="bhtd"):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, Tq, D, generator=g).to(DEV, dtype)
    if layout == "bhtd":
        k, v = (torch.randn(B, Hkv, Tkv, D, generator=g).to(DEV, dtype) for _ in range(2))
    else:  # [B, T, H_kv, D] storage viewed as [B, H_kv, T, D]
        k, v = (torch.randn(B, Tkv, Hkv, D, generator=g).to(DEV, dtype).transpose(1, 2) for _ in range(2))
    return q, k, v


def _check(q, k, v, lens, mask, omask, score, omods, splits):
    o, lse = pf.flash_attention_decode(q, k, v, lens, mask, score_mod=score, num_splits=splits)
    torch.cuda.synchronize()
    check_device_status(DEV)
    qn, kn, vn = (t.float().cpu().numpy().astype(np.float64) for t in (q, k, v))
    ro, rl = O.decode_reference(qn, kn, vn, lens, omask, omods)
    close("o", o, ro, q.dtype)
    got_lse = lse.cpu().numpy()
    fin = np.isfinite(rl)
    assert np.array_equal(fin, np.isfinite(got_lse))
    assert float(np.abs(got_lse[fin] - rl[fin]).max()) <= 2e-3
    assert o.dtype == q.dtype and o.shape == q.shape


@pytest.mark.parametrize("name", list(CASES))
def test_decode_matches_oracle(name):
    B, H, Hkv, Tq, Tkv, D, dtype, lens, mk, sk, splits = CASES[name]
    q, k, v = _inputs(B, H, Hkv, Tq, Tkv, D, dtype, seed=zlib.crc32(name.encode()) % 1000)
    mask, omask = _masks(mk)
    score, omods = _mods(sk, H)
    _check(q, k, v, lens, mask, omask, score, omods, splits)


def test_decode_strided_cache_layout():
    q, k, v = _inputs(2, 8, 2, 1, 1200, 128, torch.bfloat16, seed=3, layout="bthd")
    assert not k.is_contiguous()
    _check(q, k, v, [1200, 333], pf.causal_mask, O.causal, None, (), 0)


def test_decode_split_count_does_not_change_the_result():
    q, k, v = _inputs(1, 8, 2, 2, 3000, 128, torch.bfloat16, seed=9)
    outs = [pf.flash_attention_decode(q, k, v, [2900], pf.causal_mask, num_splits=s) for s in (1, 2, 7, 0)]
    ref_o, ref_l = outs[0]
    for o, lse in outs[1:]:
        assert float((o.float() - ref_o.float()).abs().max()) <= 1.6e-2  # one bf16 ulp near |o| ~ 1
        assert float((lse - ref_l).abs().max()) <= 1e-4


def test_decode_rejects_unsupported_requests():
    q, k, v = _inputs(1, 4, 4, 1, 128, 96, torch.bfloat16, seed=0)
    with pytest.raises(L.FlexAttnError):
        pf.flash_attention_decode(q, k, v)  # head dim 96
    q, k, v = _inputs(1, 64, 1, 3, 128, 64, torch.bfloat16, seed=0)
    with pytest.raises(L.FlexAttnError):
        pf.flash_attention_decode(q, k, v)  # 192 query rows per K/V head
    q, k, v = _inputs(1, 32, 1, 3, 128, 64, torch.float32, seed=0)
    with pytest.raises(L.FlexAttnError):
        pf.flash_attention_decode(q, k, v)  # 96 query rows: fp32 allows 64
    q, k, v = _inputs(1, 4, 4, 1, 128, 64, torch.bfloat16, seed=0)
    with pytest.raises(NotImplementedError):
        pf.flash_attention_decode(q, k, v, None, pf.document_mask([64, 64]))
