"""GPU create_block_mask: bit-exact against the reference's outputs (golden vectors)
and, for the engine's exact tables, against the oracle's tile classification."""
from pathlib import Path

import numpy as np
import pytest
import torch

import pallas_flexattn as pf
from oracle import flexattn_oracle as O
from pallas_flexattn import workloads as W

pytestmark = pytest.mark.gpu
BM = np.load(Path(__file__).resolve().parent / "golden" / "block_masks.npz")
LENS = [int(x) for x in BM["meta/doc_lengths"]]
TABLE = W.random_tile_table(256, 0.25, seed=0)

CASES = {
    "causal_T256_b64": (pf.causal_mask, O.causal),
    "bidir_T256_b64": (pf.bidirectional_mask, O.bidirectional),
    "window32_32_T256_b64": (pf.sliding_window_mask(32, 32), O.sliding_window(32, 32)),
    "window64_64_T256_b64": (pf.sliding_window_mask(64, 64), O.sliding_window(64, 64)),
    "causal_T300_b64": (pf.causal_mask, O.causal),
    "window16_16_T300_b64": (pf.sliding_window_mask(16, 16), O.sliding_window(16, 16)),
    "causal_Q256_KV384_b64": (pf.causal_mask, O.causal),
    "causal_T64_b16": (pf.causal_mask, O.causal),
    "causal_T64_b128": (pf.causal_mask, O.causal),
    "cfg1_causal_T512_b128": (pf.causal_mask, O.causal),
    "cfg2_causal_T4096_b128": (pf.causal_mask, O.causal),
    "cfg3_window1024_0_T8192_b128": (pf.sliding_window_mask(1024, 0), O.sliding_window(1024, 0)),
    "cfg4_doc_causal_T16384_b128": (pf.and_masks(pf.document_mask(LENS), pf.causal_mask),
                                    O.and_(O.document(np.repeat(np.arange(len(LENS)), LENS)), O.causal)),
    "cfg5_causal_tiles_T32768_b128": (pf.and_masks(pf.causal_mask, pf.tile_mask(TABLE, 128)),
                                      O.and_(O.causal, O.tile_table(TABLE, 128))),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_gpu_create_block_mask_is_bit_exact_with_reference(name):
    ql, kl, bs = (int(x) for x in BM[f"{name}/geom"])
    bm = pf.create_block_mask(CASES[name][0], 1, 1, ql, kl, bs)
    num = bm.num_blocks_in_row.cpu().numpy()
    cols = bm.col_indices.cpu().numpy()
    np.testing.assert_array_equal(num, BM[f"{name}/num"])
    np.testing.assert_array_equal(cols, BM[f"{name}/cols"].reshape(cols.shape))
    assert bm.num_blocks_in_row.dtype == torch.int32 and bm.col_indices.dtype == torch.int32
    assert abs(bm.sparsity - (1 - num.sum() / (bm.num_q_blocks * bm.num_kv_blocks))) < 1e-12


@pytest.mark.parametrize("name", ["causal_T300_b64", "window16_16_T300_b64", "causal_Q256_KV384_b64",
                                  "cfg1_causal_T512_b128", "cfg2_causal_T4096_b128", "bidir_T256_b64"])
def test_gpu_exact_tables_match_oracle(name):
    ql, kl, bs = (int(x) for x in BM[f"{name}/geom"])
    bm = pf.create_block_mask(CASES[name][0], 1, 1, ql, kl, bs)
    cls = O.block_mask_exact(CASES[name][1], ql, kl, bs, bs)
    np.testing.assert_array_equal(bm.tables.tile_class[0].cpu().numpy(), cls)
    ref = O.tables_from_classes(cls)
    for key in ("kv_num_blocks", "kv_indices", "full_kv_num_blocks", "full_kv_indices",
                "q_num_blocks", "q_indices", "full_q_num_blocks", "full_q_indices"):
        np.testing.assert_array_equal(getattr(bm.tables, key)[0].cpu().numpy(), ref[key], err_msg=key)


@pytest.mark.parametrize("name,full,partial", [
    ("cfg2_causal_T4096_b128", 496, 32), ("cfg3_window1024_0_T8192_b128", 420, 120),
    ("cfg4_doc_causal_T16384_b128", 1024, 324), ("cfg5_causal_tiles_T32768_b128", 8164, 256)])
def test_gpu_exact_tile_counts_on_benchmark_masks(name, full, partial):
    ql, kl, bs = (int(x) for x in BM[f"{name}/geom"])
    bm = pf.create_block_mask(CASES[name][0], 1, 1, ql, kl, bs)
    p, f = bm.tables.unmasked_tiles()
    assert (f, p) == (full, partial)


def test_band_mask_exact_finds_tiles_sampling_misses():
    band = pf.and_masks(pf.sliding_window_mask(110, -1), pf.causal_mask)
    bm = pf.create_block_mask(band, 1, 1, 1024, 1024, 128)
    cls = O.block_mask_exact(O.and_(O.sliding_window(110, -1), O.causal), 1024, 1024, 128, 128)
    np.testing.assert_array_equal(bm.tables.tile_class[0].cpu().numpy(), cls)


def test_tables_from_reference_lists_roundtrip():
    bm = pf.create_block_mask(pf.sliding_window_mask(200, 50), 1, 1, 1000, 1000, 128)
    from pallas_flexattn.block_mask import build_tables_from_lists

    t = build_tables_from_lists(bm.tables.kv_num_blocks, bm.tables.kv_indices, 128, 128, bm.tables.nkv,
                                bm.tables.full_kv_num_blocks, bm.tables.full_kv_indices, device=torch.device("cuda"))
    for key in ("tile_class", "q_num_blocks", "q_indices", "full_q_num_blocks", "full_q_indices"):
        assert torch.equal(getattr(t, key), getattr(bm.tables, key)), key


def test_per_batch_document_tables():
    d = torch.tensor([[0] * 150 + [1] * 106, [0] * 40 + [1] * 216], dtype=torch.int32)
    mm = pf.and_masks(pf.document_ids_mask(d), pf.causal_mask)
    bm = pf.create_block_mask(mm, 2, 1, 256, 256, 128)
    assert bm.tables.num_b == 2
    for b in range(2):
        cls = O.block_mask_exact(O.and_(O.document(d[b].numpy()), O.causal), 256, 256, 128, 128)
        np.testing.assert_array_equal(bm.tables.tile_class[b].cpu().numpy(), cls)


def test_create_block_mask_from_a_lambda_is_bit_exact():
    """An arbitrary callable (no registry entry) is evaluated on the GPU into per-tile bitmasks;
    the reference fields still follow the 3x3 rule bit for bit and the tables are exact."""
    band = lambda q, kv: ((q - kv) >= 100) & ((q - kv) <= 110)  # noqa: E731
    bm = pf.create_block_mask(band, 1, 1, 1024, 1024, 128)
    np.testing.assert_array_equal(bm.num_blocks_in_row.cpu().numpy(), BM["band100_110_T1024_b128/num"])
    np.testing.assert_array_equal(bm.col_indices.cpu().numpy(), BM["band100_110_T1024_b128/cols"])
    cls = O.block_mask_exact(lambda q, kv: ((q - kv) >= 100) & ((q - kv) <= 110), 1024, 1024, 128, 128)
    np.testing.assert_array_equal(bm.tables.tile_class[0].cpu().numpy(), cls)


@pytest.mark.parametrize("T,bs", [(1000, 128), (300, 64), (777, 96)])
def test_lambda_tables_match_oracle_exact(T, bs):
    mm = lambda q, kv: ((q * 7 + kv * 3) % 11 < 4) | (q == kv)  # noqa: E731 (scattered pattern)
    bm = pf.create_block_mask(mm, 1, 1, T, T, bs)
    cls = O.block_mask_exact(mm, T, T, bs, bs)
    np.testing.assert_array_equal(bm.tables.tile_class[0].cpu().numpy(), cls)
    num, cols = O.block_mask_ref9(mm, T, T, bs)
    np.testing.assert_array_equal(bm.num_blocks_in_row.cpu().numpy(), num)
