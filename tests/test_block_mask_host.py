"""Host-side block-mask logic: the reference's block-mask tests (tests/test_block_mask.py)
on the engine's BlockMask, the host builders against the golden vectors, and the
mask_mod registry against the oracle predicates.  No GPU needed."""
from pathlib import Path

import numpy as np
import pytest
import torch

import pallas_flexattn as pf
from oracle import flexattn_oracle as O
from pallas_flexattn import _lib as L
from pallas_flexattn import workloads as W
from pallas_flexattn.mask_mod import spec_of

BM = np.load(Path(__file__).resolve().parent / "golden" / "block_masks.npz")


class TestBlockMaskCreation:
    def test_create_causal_block_mask(self):
        bm = pf.create_causal_block_mask(256, 64)
        assert bm.block_size == 64 and bm.q_len == 256 and bm.kv_len == 256
        assert bm.num_q_blocks == 4
        assert [int(x) for x in bm.num_blocks_in_row] == [1, 2, 3, 4]

    def test_create_sliding_window_block_mask(self):
        bm = pf.create_sliding_window_block_mask(256, 64, 64)
        assert bm.block_size == 64 and bm.q_len == 256
        assert int(bm.num_blocks_in_row[1]) == 3 and int(bm.num_blocks_in_row[2]) == 3

    def test_block_mask_sparsity_causal(self):
        bm = pf.create_causal_block_mask(1024, 128)
        n = 1024 // 128
        assert abs(bm.sparsity - (1.0 - (n * (n + 1) / 2) / (n * n))) < 0.01


class TestBlockMaskStructure:
    def test_col_indices_shape(self):
        bm = pf.create_causal_block_mask(256, 64)
        assert tuple(bm.col_indices.shape) == (4, 4)

    def test_col_indices_values_causal(self):
        c = pf.create_causal_block_mask(256, 64).col_indices
        assert int(c[0, 0]) == 0 and int(c[0, 1]) == -1
        assert [int(x) for x in c[2]] == [0, 1, 2, -1]

    def test_num_blocks_in_row_dtype(self):
        bm = pf.create_causal_block_mask(128, 64)
        assert bm.num_blocks_in_row.dtype == torch.int32 and bm.col_indices.dtype == torch.int32


class TestBlockMaskEdgeCases:
    def test_non_power_of_two_seq_len(self):
        assert pf.create_causal_block_mask(300, 64).num_q_blocks == 5

    def test_very_small_block_size(self):
        assert pf.create_causal_block_mask(64, 16).num_q_blocks == 4

    def test_single_block(self):
        bm = pf.create_causal_block_mask(64, 128)
        assert bm.num_q_blocks == 1 and int(bm.num_blocks_in_row[0]) == 1


@pytest.mark.parametrize("T,bs", [(256, 64), (300, 64), (64, 16), (64, 128), (1024, 128), (128, 64)])
def test_causal_builder_golden(T, bs):
    bm = pf.create_causal_block_mask(T, bs)
    np.testing.assert_array_equal(bm.num_blocks_in_row.numpy(), BM[f"causalbuilder_T{T}_b{bs}/num"])
    np.testing.assert_array_equal(bm.col_indices.numpy(), BM[f"causalbuilder_T{T}_b{bs}/cols"])


@pytest.mark.parametrize("T,w,bs", [(256, 64, 64), (1000, 100, 128), (512, 200, 64)])
def test_window_builder_golden(T, w, bs):
    bm = pf.create_sliding_window_block_mask(T, w, bs)
    np.testing.assert_array_equal(bm.num_blocks_in_row.numpy(), BM[f"windowbuilder_T{T}_w{w}_b{bs}/num"])
    np.testing.assert_array_equal(bm.col_indices.numpy(), BM[f"windowbuilder_T{T}_w{w}_b{bs}/cols"])


def test_oracle_reference_rule_on_window_golden():
    num, cols = O.block_mask_ref9(O.sliding_window(16, 16), 300, 300, 64)
    np.testing.assert_array_equal(num, BM["window16_16_T300_b64/num"])
    np.testing.assert_array_equal(cols, BM["window16_16_T300_b64/cols"])


@pytest.mark.parametrize("mm,om", [
    (pf.causal_mask, O.causal),
    (pf.bidirectional_mask, O.bidirectional),
    (pf.sliding_window_mask(5, 3), O.sliding_window(5, 3)),
    (pf.sliding_window_mask(-1, 4), O.sliding_window(-1, 4)),
])
def test_mask_mods_agree_with_oracle_numpy_and_torch(mm, om):
    qi, ki = np.arange(40)[:, None], np.arange(50)[None, :]
    ref = np.broadcast_to(om(qi, ki), (40, 50))
    np.testing.assert_array_equal(np.broadcast_to(mm(qi, ki), (40, 50)), ref)
    got = torch.broadcast_to(mm(torch.as_tensor(qi), torch.as_tensor(ki)), (40, 50)).numpy()
    np.testing.assert_array_equal(got, ref)


def test_and_masks_spec_composition():
    lens = [5, 7, 4]
    m = pf.and_masks(pf.document_mask(lens), pf.causal_mask, pf.sliding_window_mask(6, 0),
                     pf.sliding_window_mask(4, -1))
    s = spec_of(m)
    assert s.flags == L.FA_MASK_DOCUMENT | L.FA_MASK_CAUSAL | L.FA_MASK_WINDOW
    assert (s.window_left, s.window_right) == (4, 0)
    doc = np.repeat(np.arange(3), lens)
    qi, ki = np.arange(16)[:, None], np.arange(16)[None, :]
    ref = O.and_(O.document(doc), O.causal, O.sliding_window(4, 0))(qi, ki)
    np.testing.assert_array_equal(m(torch.as_tensor(qi), torch.as_tensor(ki)).numpy(), ref)


def test_unregistered_callables_have_no_spec():
    assert spec_of(lambda q, kv: q > kv) is None
    assert spec_of(pf.and_masks(pf.causal_mask, lambda q, kv: q > kv)) is None


def test_flash_attention_refuses_cpu_tensors_and_unknown_mods():
    q = torch.zeros(1, 1, 8, 64)
    with pytest.raises(ValueError):
        pf.flash_attention_fwd(q, q, q)


def test_workload_generators():
    assert W.document_lengths(16384, 0) == [3523, 2702, 2219, 1292, 1438, 413, 544, 319, 929, 3005]
    t = W.random_tile_table(256, 0.25, 0)
    assert int(np.tril(t, -1).sum()) == 8164 and np.all(np.diag(t) == 1)
    assert W.count_pairs(W.get(2).mask_mod, 4096, 4096) == 8390656
    assert W.count_pairs(W.get(3).mask_mod, 8192, 8192) == 7872000
