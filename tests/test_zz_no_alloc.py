"""fa_bwd_noalloc (backward on the library's static device scratch) against fa_bwd.

Both are called through the C ABI on the same inputs; two no-alloc calls in a row must
each agree with fa_bwd within the bf16/fp32 parity tolerance, and the second call must not
change the device's free memory.  The file sorts last so it also runs after every other
GPU test; it passes alone in a fresh process too (the first call does the per-device setup).
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

import pallas_flexattn as pf
from pallas_flexattn import _lib as L
from pallas_flexattn import flash_attn as FA

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None
# (max-abs, rel-L2, per-element relative term): the parity tolerance of the GPU suite
TOL = {torch.bfloat16: (2e-2, 5e-3, 2.0 ** -8), torch.float32: (2e-4, 1e-5, 0.0)}


def close(name, got, ref, dtype):
    got, ref = got.float().cpu().numpy(), ref.float().cpu().numpy()
    atol, rtol, elem_rel = TOL[dtype]
    diff = np.abs(got - ref)
    excess = float((diff - (atol + elem_rel * np.abs(ref))).max())
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), atol * math.sqrt(ref.size)))
    assert excess <= 0 and rel <= rtol, f"{name}: max-abs {diff.max():.3e}, rel-L2 {rel:.3e}"


CASES = {
    "causal_bf16_d128": dict(shape=(2, 4, 1024, 128), dtype=torch.bfloat16, mask=pf.causal_mask, score=None),
    "window_softcap_bf16_d64_ragged": dict(shape=(1, 4, 1000, 64), dtype=torch.bfloat16,
                                           mask=pf.sliding_window_mask(256, 0), score=pf.softcap_score_mod(20.0)),
    "causal_fp32_d64_generic": dict(shape=(1, 2, 300, 64), dtype=torch.float32, mask=pf.causal_mask, score=None),
}


def _bwd_params(plan, q, k, v, o, lse, do, dq, dk, dv):
    p = L.FaBwdParams()
    plan._fill(p)
    p.q, p.k, p.v, p.o, p.dout = (FA._fa_tensor(t) for t in (q, k, v, o, do))
    p.dq, p.dk, p.dv = FA._fa_tensor(dq), FA._fa_tensor(dk), FA._fa_tensor(dv)
    p.lse = lse.data_ptr()
    return p


@pytest.mark.parametrize("case", list(CASES))
def test_noalloc_matches_fa_bwd_twice(case):
    c = CASES[case]
    g = torch.Generator(device=DEV).manual_seed(7)
    q, k, v, do = (torch.randn(c["shape"], generator=g, device=DEV).to(c["dtype"]) for _ in range(4))
    o, lse = pf.flash_attention_fwd(q, k, v, c["mask"], score_mod=c["score"])
    plan = FA._Plan(q, k, v, c["mask"], c["score"], None, 64, 64, 3, None, True)
    lib = L.lib()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    outs = [tuple(torch.empty_like(t) for t in (q, k, v)) for _ in range(3)]
    params = [_bwd_params(plan, q, k, v, o, lse, do, *g3) for g3 in outs]

    nbytes = C.c_size_t(0)
    L.check(lib.fa_bwd_workspace_size(C.byref(params[0]), C.byref(nbytes)))
    assert nbytes.value <= L.FA_NOALLOC_SCRATCH_BYTES
    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=DEV)
    L.check(lib.fa_bwd(C.byref(params[0]), ws.data_ptr(), ws.numel(), stream))

    L.check(lib.fa_bwd_noalloc(C.byref(params[1]), stream))
    torch.cuda.synchronize(DEV)
    free_before = torch.cuda.mem_get_info(DEV)[0]
    L.check(lib.fa_bwd_noalloc(C.byref(params[2]), stream))
    torch.cuda.synchronize(DEV)
    assert torch.cuda.mem_get_info(DEV)[0] == free_before, "fa_bwd_noalloc changed the device's free memory"
    FA.check_device_status(DEV)

    for call in (1, 2):
        for name, got, ref in zip(("dq", "dk", "dv"), outs[call], outs[0]):
            close(f"call {call} {name}", got, ref, c["dtype"])


def test_noalloc_rejects_shapes_beyond_the_scratch():
    p = L.FaBwdParams()
    p.dtype = L.FA_DTYPE_BF16
    p.B, p.H, p.H_kv, p.Tq, p.Tkv, p.D = 1, 16, 16, 8192, 8192, 128
    nbytes = C.c_size_t(0)
    L.check(L.lib().fa_bwd_workspace_size(C.byref(p), C.byref(nbytes)))
    assert nbytes.value > L.FA_NOALLOC_SCRATCH_BYTES
    rc = L.lib().fa_bwd_noalloc(C.byref(p), None)
    assert rc == L.FA_ERR_UNSUPPORTED
    assert "static scratch" in L.lib().fa_last_error().decode()
