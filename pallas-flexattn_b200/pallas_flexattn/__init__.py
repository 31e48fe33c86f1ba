"""FlexAttention for NVIDIA B200 — drop-in for the pallas_flexattn API.

Same public names as the reference package (src/pallas_flexattn/__init__.py);
the compute runs in libflexattn.so (hand-written sm_100a CUDA).  Extensions:
score_mod functors, composable mask_mods, GPU-built block tables and measured
autotuning.
"""
from .flash_attn import (
    check_device_status,
    flash_attention,
    flash_attention_bwd,
    flash_attention_fwd,
    mha_reference,
)
from .decode import flash_attention_decode
from .mask_mod import (
    MaskMod,
    and_masks,
    bidirectional_mask,
    causal_mask,
    document_ids_mask,
    document_mask,
    sliding_window_mask,
    tile_mask,
)
from .score_mod import (
    alibi_score_mod,
    alibi_slopes,
    compose_score_mods,
    relative_bias_score_mod,
    softcap_score_mod,
)
from .block_mask import (
    BlockMask,
    create_block_mask,
    create_causal_block_mask,
    create_sliding_window_block_mask,
)
from .kernel_tuner import (
    autotune,
    get_kernel_config,
    get_optimal_params,
    print_kernel_config,
)

__all__ = [
    "flash_attention",
    "flash_attention_fwd",
    "flash_attention_bwd",
    "flash_attention_decode",
    "mha_reference",
    "MaskMod",
    "causal_mask",
    "bidirectional_mask",
    "sliding_window_mask",
    "BlockMask",
    "create_block_mask",
    "create_causal_block_mask",
    "create_sliding_window_block_mask",
    "get_optimal_params",
    "get_kernel_config",
    "print_kernel_config",
    # additions
    "document_mask",
    "document_ids_mask",
    "tile_mask",
    "and_masks",
    "alibi_score_mod",
    "alibi_slopes",
    "softcap_score_mod",
    "relative_bias_score_mod",
    "compose_score_mods",
    "autotune",
    "check_device_status",
]
