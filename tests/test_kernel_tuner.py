"""Kernel tuner: the reference's tests (tests/test_kernel_tuner.py) plus its golden table."""
import json
from pathlib import Path

import pytest

from pallas_flexattn import get_kernel_config, get_optimal_params, print_kernel_config

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "tuner.json").read_text())


class TestKernelTuner:
    def test_get_optimal_params_short_sequence(self):
        block_r, block_c, num_warps, num_stages = get_optimal_params(256, 64)
        assert block_r <= 64 and block_c <= 64 and num_warps >= 4

    def test_get_optimal_params_long_sequence(self):
        block_r, block_c, num_warps, num_stages = get_optimal_params(4096, 64)
        assert block_r >= 128 and block_c >= 64 and num_warps >= 8

    def test_get_optimal_params_large_head_dim(self):
        block_r, block_c, _, _ = get_optimal_params(2048, 256)
        assert block_r <= 64 and block_c <= 64

    def test_get_optimal_params_cached(self):
        assert get_optimal_params(1024, 64) == get_optimal_params(1024, 64)
        assert get_optimal_params.cache_info().hits >= 1

    def test_get_kernel_config(self):
        config = get_kernel_config(2, 8, 2048, 64, "causal")
        assert config["batch_size"] == 2 and config["num_heads"] == 8
        assert config["seq_len"] == 2048 and config["head_dim"] == 64
        for key in ("block_r", "block_c", "num_warps", "num_stages"):
            assert key in config

    def test_sparsity_optimization(self):
        dense = get_kernel_config(2, 8, 1024, 64, None)
        sparse = get_kernel_config(2, 8, 1024, 64, "causal")
        assert sparse["block_r"] <= dense["block_r"]


@pytest.mark.parametrize("row", GOLD["get_optimal_params"], ids=lambda r: f"S{r[0]}_D{r[1]}_sp{int(r[2])}")
def test_table_matches_reference(row):
    s, d, sp, expect = row
    assert list(get_optimal_params(s, d, sp)) == expect


@pytest.mark.parametrize("row", GOLD["get_kernel_config"], ids=lambda r: str(r[0]))
def test_kernel_config_matches_reference(row):
    args, expect = row
    assert get_kernel_config(*args) == expect


def test_print_kernel_config(capsys):
    print_kernel_config(2, 8, 2048, 64, "causal")
    out = capsys.readouterr().out
    assert "BLOCK_R (block_r):      128" not in out or "NUM_WARPS" in out
    assert "block_r=64" in out and "num_stages=3" in out


def test_tuned_cache_round_trip(tmp_path, monkeypatch):
    """The measured tuner's cache: entries persist to the JSON file and are read back by key
    (the planner's lookup) after the in-memory copy is dropped.  No GPU needed."""
    from pallas_flexattn import kernel_tuner as KT
    from pallas_flexattn.mask_mod import spec_of as mspec
    from pallas_flexattn.score_mod import spec_of as sspec
    import pallas_flexattn as pf

    monkeypatch.setenv("FLEXATTN_TUNE_CACHE", str(tmp_path / "tune.json"))
    KT.clear_memory_cache()
    key = KT.make_key("NVIDIA B200", "torch.bfloat16", (1, 4, 1024, 128), (1, 4, 1024, 128),
                      mspec(pf.causal_mask), sspec(None))
    other = KT.make_key("NVIDIA B200", "torch.bfloat16", (1, 4, 1024, 128), (1, 4, 1024, 128),
                        mspec(pf.sliding_window_mask(64, 0)), sspec(None))
    assert key != other
    assert KT.lookup_key(key) is None
    entry = {"fwd": {"num_stages": 2, "tile_cfg": 5, "ms": 0.1}, "bwd": {"num_stages": 3, "ms": 0.2}}
    KT._CACHE[key] = entry
    KT._save_cache()
    KT.clear_memory_cache()
    assert KT.lookup_key(key) == entry and KT.lookup_key(other) is None
    monkeypatch.setenv("FLEXATTN_TUNE_CACHE", str(tmp_path / "elsewhere.json"))
    assert KT.lookup_key(key) is None  # a different cache file is a different cache
