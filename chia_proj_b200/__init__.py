"""chia_proj_b200 -- B200-native (sm_100a) attention-variant library.

Drop-in replacements for the ten attention operators of
JoshiP-commits/CHIA_proj ("GraphSynth"): same eager call signatures
``op(q, k, v, **params) -> out`` (reference ``extra_bench.py:32-62``), one
hand-written tcgen05/TMA kernel behind a C ABI (``include/chia_attn.h``).
"""

from .ops import (  # noqa: F401
    CAUSAL,
    FULL,
    OPS,
    Mask,
    alibi_slopes_geometric,
    attention,
    attention_backward,
    bias_alibi,
    bias_block_diagonal,
    bias_dilated,
    bias_local,
    bias_prefix_lm,
    bias_sliding_window,
    check_device_status,
    mask_aware_flops,
    op_config,
    reference_alibi_slopes,
    reference_temps,
    relu_attn,
    sigmoid_attn,
    softcap_gemma2,
    temp_perhead,
    tile_plan,
    visible_pairs,
)
from ._native import ChiaError  # noqa: F401
from . import flex  # noqa: F401,E402
