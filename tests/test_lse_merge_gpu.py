"""fa_lse_merge (the log-sum-exp combine of two partial attention results over disjoint keys,
used by the context-parallel ring) against the same combine written in torch: the vector
kernel (bf16 parts, D 64 or 128, 16-byte aligned rows) and the row-per-warp kernel (fp32
parts, other strides), with rows empty on either side or both, on ragged row counts."""
import math

import pytest
import torch

from pallas_flexattn import ring

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0) if torch.cuda.is_available() else None


@pytest.mark.parametrize("D,dtype,pad,rows", [(64, torch.bfloat16, 0, 1000), (128, torch.bfloat16, 0, 517),
                                             (64, torch.float32, 0, 300), (128, torch.bfloat16, 4, 333)])
def test_gpu_merge_matches_torch(D, dtype, pad, rows):
    g = torch.Generator(device=DEV).manual_seed(D + rows)
    o_acc = torch.randn(rows, D, device=DEV, generator=g)
    lse_acc = torch.randn(rows, device=DEV, generator=g) * 3
    part = torch.randn(rows, D + pad, device=DEV, generator=g).to(dtype)
    o_part = part[:, :D]  # pad > 0: a row stride the vector kernel does not take
    lse_part = torch.randn(rows, device=DEV, generator=g) * 3
    lse_acc[::7] = -math.inf          # accumulator empty: takes the part
    lse_part[::5] = -math.inf         # part empty: accumulator unchanged
    lse_acc[::35] = -math.inf         # both empty (multiples of 35): stays empty
    o_acc[::35] = 0.0
    ref_o, ref_l = o_acc.clone(), lse_acc.clone()
    ring.torch_merge(ref_o, ref_l, o_part, lse_part)
    ring.gpu_merge(o_acc, lse_acc, o_part, lse_part)
    torch.cuda.synchronize()
    torch.testing.assert_close(lse_acc, ref_l, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(o_acc, ref_o, rtol=1e-5, atol=1e-5)
    assert torch.all(torch.isneginf(lse_acc[::35])) and torch.all(o_acc[::35] == 0)
