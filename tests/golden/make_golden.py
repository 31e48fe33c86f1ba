"""Generate golden vectors by running the reference's own source.

    python tests/golden/make_golden.py --reference-src PATH

Imports novastar53/pallas-flexattn from its source tree (PATH is the project's ``src``
directory, or the FLEXATTN_REFERENCE_SRC environment variable; it is only read) under the
numpy stand-in for jax in jax_numpy_standin.py, and records:

* block_masks.npz   create_block_mask (block_mask.py:54-129) on the reference's
                    mask_mods and on document / tile / band predicates, at the
                    test and benchmark geometries; the analytic builders
                    (:132-218);
* tuner.json        get_optimal_params / get_kernel_config (kernel_tuner.py);
* attention.npz     seeded fp32 inputs and the reference kernels' outputs run in
                    Pallas-interpret emulation: flash_attention_fwd (o, lse),
                    flash_attention_bwd (dq, dk, dv), and mha_reference.

Only this script reads the reference tree; the tests read the fixtures.
"""
from __future__ import annotations

import argparse
import os
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def block_mask_cases(ref_mm, np_doc, np_table):
    c, b, sw = ref_mm.causal_mask, ref_mm.bidirectional_mask, ref_mm.sliding_window_mask
    cases = [
        ("causal_T256_b64", c, 256, 256, 64),
        ("bidir_T256_b64", b, 256, 256, 64),
        ("window32_32_T256_b64", sw(32, 32), 256, 256, 64),
        ("window64_64_T256_b64", sw(64, 64), 256, 256, 64),
        ("causal_T300_b64", c, 300, 300, 64),
        ("window16_16_T300_b64", sw(16, 16), 300, 300, 64),
        ("causal_Q256_KV384_b64", c, 256, 384, 64),
        ("causal_T64_b16", c, 64, 64, 16),
        ("causal_T64_b128", c, 64, 64, 128),
        ("cfg1_causal_T512_b128", c, 512, 512, 128),
        ("cfg2_causal_T4096_b128", c, 4096, 4096, 128),
        ("cfg3_window1024_0_T8192_b128", sw(1024, 0), 8192, 8192, 128),
        ("cfg4_doc_causal_T16384_b128", lambda q, kv: (np_doc[q] == np_doc[kv]) & (q >= kv), 16384, 16384, 128),
        ("cfg5_causal_tiles_T32768_b128", lambda q, kv: (q >= kv) & (np_table[q // 128, kv // 128] != 0),
         32768, 32768, 128),
        ("band100_110_T1024_b128", lambda q, kv: ((q - kv) >= 100) & ((q - kv) <= 110), 1024, 1024, 128),
    ]
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("FLEXATTN_REFERENCE_SRC"),
                    help="the reference project's src directory (read-only)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("give --reference-src or set FLEXATTN_REFERENCE_SRC")

    sys.path.insert(0, str(HERE))
    import jax_numpy_standin

    jax_numpy_standin.install()
    sys.path.insert(0, args.reference_src)
    from pallas_flexattn import block_mask as ref_bm  # the reference package
    from pallas_flexattn import flash_attn as ref_fa
    from pallas_flexattn import kernel_tuner as ref_kt
    from pallas_flexattn import mask_mod as ref_mm

    # benchmark mask parameters (same generators as the engine's workloads module)
    rng = np.random.default_rng(0)
    lens, tot = [], 0
    while tot < 16384:
        n = min(int(rng.integers(256, 4097)), 16384 - tot)
        lens.append(n)
        tot += n
    np_doc = np.repeat(np.arange(len(lens)), lens)
    rng = np.random.default_rng(0)
    keep = rng.random((256, 256)) < 0.25
    np.fill_diagonal(keep, True)
    np_table = keep.astype(np.uint8)

    bm = {}
    for name, mm, ql, kl, bs in block_mask_cases(ref_mm, np_doc, np_table):
        m = ref_bm.create_block_mask(mm, 1, 1, ql, kl, bs)
        bm[f"{name}/num"] = np.asarray(m.num_blocks_in_row, np.int32)
        bm[f"{name}/cols"] = np.asarray(m.col_indices, np.int32).reshape(len(bm[f"{name}/num"]), -1)
        bm[f"{name}/geom"] = np.array([ql, kl, bs], np.int64)
        print(f"block mask {name}: {int(bm[f'{name}/num'].sum())} tiles", flush=True)
    for T, bs in ((256, 64), (300, 64), (64, 16), (64, 128), (1024, 128), (128, 64)):
        m = ref_bm.create_causal_block_mask(T, bs)
        bm[f"causalbuilder_T{T}_b{bs}/num"] = np.asarray(m.num_blocks_in_row, np.int32)
        bm[f"causalbuilder_T{T}_b{bs}/cols"] = np.asarray(m.col_indices, np.int32)
    for T, w, bs in ((256, 64, 64), (1000, 100, 128), (512, 200, 64)):
        m = ref_bm.create_sliding_window_block_mask(T, w, bs)
        bm[f"windowbuilder_T{T}_w{w}_b{bs}/num"] = np.asarray(m.num_blocks_in_row, np.int32)
        bm[f"windowbuilder_T{T}_w{w}_b{bs}/cols"] = np.asarray(m.col_indices, np.int32)
    bm["meta/doc_lengths"] = np.array(lens, np.int64)
    np.savez_compressed(HERE / "block_masks.npz", **bm)

    tuner = {"get_optimal_params": [], "get_kernel_config": []}
    for s in (64, 128, 256, 257, 512, 513, 1024, 2048, 2049, 4096, 4097, 8192, 32768):
        for d in (16, 32, 64, 128, 256):
            for sp in (False, True):
                tuner["get_optimal_params"].append([s, d, sp, list(ref_kt.get_optimal_params(s, d, sp))])
    for cfg in ((2, 8, 2048, 64, "causal"), (2, 8, 1024, 64, None), (4, 16, 4096, 128, "sliding_window"),
                (1, 4, 512, 64, "bidirectional")):
        tuner["get_kernel_config"].append([list(cfg), ref_kt.get_kernel_config(*cfg)])
    (HERE / "tuner.json").write_text(json.dumps(tuner, indent=0))

    att = {}
    cases = [("causal_B1H2T128D32", ref_mm.causal_mask, 32), ("bidir_B1H2T128D32", ref_mm.bidirectional_mask, 32),
             ("window32_B1H2T128D32", ref_mm.sliding_window_mask(32, 32), 32),
             ("causal_B1H2T128D64", ref_mm.causal_mask, 64)]
    for i, (name, mm, D) in enumerate(cases):
        g = np.random.default_rng(100 + i)
        q, k, v, do = (g.standard_normal((1, 2, 128, D)).astype(np.float32) for _ in range(4))
        o, lse = ref_fa.flash_attention_fwd(q, k, v, mm, 64, 64, 4, 3, True)
        dq, dk, dv = ref_fa.flash_attention_bwd(q, k, v, o, lse, do, mm, 64, 64, 4, 3, True)
        o_ref = ref_fa.mha_reference(q, k, v, mm)
        for key, val in dict(q=q, k=k, v=v, do=do, o=o, lse=lse, dq=dq, dk=dk, dv=dv, o_ref=o_ref).items():
            att[f"{name}/{key}"] = np.asarray(val, np.float32)
        print(f"attention {name}: |o-o_ref|max {np.abs(o - o_ref).max():.2e}", flush=True)
    np.savez_compressed(HERE / "attention.npz", **att)


if __name__ == "__main__":
    main()
