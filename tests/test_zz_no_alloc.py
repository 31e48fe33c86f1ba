"""fa_bwd_noalloc (backward on the library's static device scratch) against fa_bwd.

Some hosts of this library hand it device pointers but own no device allocator (a
cgo/JNI/ctypes binding inside another runtime's memory pool); fa_bwd_noalloc lets them
run the backward without supplying a workspace.  Both entry points are called through the
C ABI on the same inputs; two no-alloc calls in a row must each agree with fa_bwd within
the parity tolerance of the GPU suite.  The second call must leave torch's allocator
untouched (exact) and the device's free memory unchanged (best effort: another process
on the GPU can move it).  The file sorts last so it also runs after every other GPU test;
it passes alone in a fresh process too (the first call in a context resolves the scratch).
"""
import ctypes as C

import pytest
import torch

import pallas_flexattn as pf
from pallas_flexattn import _lib as L
from pallas_flexattn import flash_attn as FA
from tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


def close(name, got, ref, dtype):
    """The parity tolerance of the GPU suite (tests/tolerance.py)."""
    assert_close(name, got.float().cpu().numpy(), ref.float().cpu().numpy(), bf16=dtype == torch.bfloat16)


# name: (B, H, H_kv, T, D), dtype, mask, score
CASES = {
    "causal_bf16_d128": ((2, 4, 4, 1024, 128), torch.bfloat16, pf.causal_mask, None),
    "window_softcap_bf16_d64_ragged": ((1, 4, 4, 1000, 64), torch.bfloat16, pf.sliding_window_mask(256, 0),
                                       pf.softcap_score_mod(20.0)),
    "gqa_h8_kv2_bf16_d128": ((1, 8, 2, 768, 128), torch.bfloat16, pf.causal_mask, None),
    "causal_fp32_d64_generic": ((1, 2, 2, 300, 64), torch.float32, pf.causal_mask, None),
    # workspace 66,027,520 bytes: just under the 64 MiB scratch, so the dQ accumulator's last
    # rows sit near the end of the array
    "near_limit_bf16_d128": ((1, 31, 31, 4096, 128), torch.bfloat16, pf.causal_mask, None),
}


def _tensors(shape, dtype, seed=7):
    B, H, Hkv, T, D = shape
    g = torch.Generator(device=DEV).manual_seed(seed)
    mk = lambda h: torch.randn((B, h, T, D), generator=g, device=DEV).to(dtype)  # noqa: E731
    return mk(H), mk(Hkv), mk(Hkv), mk(H)


def _bwd_params(plan, q, k, v, o, lse, do, dq, dk, dv):
    p = L.FaBwdParams()
    plan._fill(p)
    p.q, p.k, p.v, p.o, p.dout = (FA._fa_tensor(t) for t in (q, k, v, o, do))
    p.dq, p.dk, p.dv = FA._fa_tensor(dq), FA._fa_tensor(dk), FA._fa_tensor(dv)
    p.lse = lse.data_ptr()
    return p


@pytest.mark.parametrize("case", list(CASES))
def test_noalloc_matches_fa_bwd_twice(case):
    shape, dtype, mask, score = CASES[case]
    q, k, v, do = _tensors(shape, dtype)
    o, lse = pf.flash_attention_fwd(q, k, v, mask, score_mod=score)
    plan = FA._Plan(q, k, v, mask, score, None, 64, 64, 3, None, True)
    lib = L.lib()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    outs = [tuple(torch.empty_like(t) for t in (q, k, v)) for _ in range(3)]
    params = [_bwd_params(plan, q, k, v, o, lse, do, *g3) for g3 in outs]

    nbytes = C.c_size_t(0)
    L.check(lib.fa_bwd_workspace_size(C.byref(params[0]), C.byref(nbytes)))
    assert nbytes.value <= L.FA_NOALLOC_SCRATCH_BYTES
    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=DEV)
    L.check(lib.fa_bwd(C.byref(params[0]), ws.data_ptr(), ws.numel(), stream))
    del ws

    L.check(lib.fa_bwd_noalloc(C.byref(params[1]), stream))
    torch.cuda.synchronize(DEV)
    torch_before = torch.cuda.memory_allocated(DEV)
    free_before = torch.cuda.mem_get_info(DEV)[0]
    L.check(lib.fa_bwd_noalloc(C.byref(params[2]), stream))
    torch.cuda.synchronize(DEV)
    free_after = torch.cuda.mem_get_info(DEV)[0]
    assert torch.cuda.memory_allocated(DEV) == torch_before, "fa_bwd_noalloc allocated through torch"
    assert free_after == free_before, "fa_bwd_noalloc changed the device's free memory"
    FA.check_device_status(DEV)

    for call in (1, 2):
        for name, got, ref in zip(("dq", "dk", "dv"), outs[call], outs[0]):
            close(f"call {call} {name}", got, ref, dtype)


def test_noalloc_rejects_shapes_beyond_the_scratch():
    """A well-formed call whose workspace exceeds the scratch is refused before any work."""
    shape = (1, 16, 16, 8192, 128)
    q, k, v, do = _tensors(shape, torch.bfloat16, seed=1)
    o, lse = torch.empty_like(q), torch.zeros(q.shape[:3], dtype=torch.float32, device=DEV)
    plan = FA._Plan(q, k, v, pf.causal_mask, None, None, 64, 64, 3, None, True)
    p = _bwd_params(plan, q, k, v, o, lse, do, *(torch.empty_like(t) for t in (q, k, v)))
    nbytes = C.c_size_t(0)
    L.check(L.lib().fa_bwd_workspace_size(C.byref(p), C.byref(nbytes)))
    assert nbytes.value > L.FA_NOALLOC_SCRATCH_BYTES
    rc = L.lib().fa_bwd_noalloc(C.byref(p), torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == L.FA_ERR_UNSUPPORTED
    assert "static scratch" in L.lib().fa_last_error().decode()
