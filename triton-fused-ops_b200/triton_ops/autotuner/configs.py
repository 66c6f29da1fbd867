"""Configuration spaces (kept for API compatibility with the reference's autotuner).

The launch path does not search these: tiles come from
:mod:`triton_ops.autotuner.tile_table`. The spaces list the tile options the
native kernels are built with, so a user-driven search stays meaningful.
"""

from itertools import product
from typing import Any, Dict, List

# RMSNorm+RoPE: warp per row (vectors_per_lane 4 / 8 / 16, 12 or 16 warps per
# CTA, two row buffers per warp) or CTA per row (threads x vectors_per_thread).
RMSNORM_ROPE_CONFIGS = {"threads": [32, 64, 128, 256], "vectors_per_thread": [1, 2, 4, 8],
                        "warps_per_cta": [12, 16], "vectors_per_lane": [4, 8, 16]}
# Gated MLP: BLOCK_M 256 = a two-CTA (cta_group::2) tile, 6 stages of 32 KB per
# CTA; BLOCK_M 128 = one CTA, 4 stages of 48 KB. BLOCK_N columns of gate and of
# up per tile (one N = 256 MMA over both).
GATED_MLP_CONFIGS = {"BLOCK_M": [128, 256], "BLOCK_N": [128], "BLOCK_K_BYTES": [128], "STAGES": [4, 6],
                     "GROUP_M": [16]}
# FP8 GEMM: two-CTA 256 x 256 tiles (6 stages) for M > 128; one-CTA 128 x 128
# (7 stages; 11 with 32-row A stages for M <= 32) or 128 x 256 (4 stages) for
# M <= 128, with K split into 2-8 slices when the tiles cover under half the GPU.
FP8_GEMM_CONFIGS = {"BLOCK_M": [128, 256], "BLOCK_N": [128, 256], "BLOCK_K_BYTES": [128], "STAGES": [4, 6, 7, 11],
                    "GROUP_M": [16], "K_SPLITS": [1, 2, 4, 8]}


def generate_configs(config_space: Dict[str, List[Any]]) -> List[Dict[str, Any]]:
    """Cartesian product of a configuration space."""
    keys = list(config_space)
    return [dict(zip(keys, values)) for values in product(*(config_space[k] for k in keys))]


def filter_valid_configs(configs: List[Dict[str, Any]], problem_size=None, max_shared_memory: int = 232448,
                         dtype_size: int = 2) -> List[Dict[str, Any]]:
    """Drops configurations whose per-CTA operand ring would not fit in shared memory
    (a 256-row tile is shared by two CTAs, each staging 128 rows of A and half of B)."""
    out = []
    for c in configs:
        bm, bn, kb, st = c.get("BLOCK_M", 0), c.get("BLOCK_N", 0), c.get("BLOCK_K_BYTES", 0), c.get("STAGES", 1)
        ctas = 2 if bm == 256 else 1
        if bm and bn and kb and (bm // ctas + bn // ctas) * kb * st > max_shared_memory:
            continue
        out.append(c)
    return out


def get_default_config(kernel_type: str) -> Dict[str, Any]:
    defaults = {
        "rmsnorm_rope": {"threads": 256, "vectors_per_thread": 2},
        "gated_mlp": {"BLOCK_M": 256, "BLOCK_N": 128, "BLOCK_K_BYTES": 128, "STAGES": 6, "GROUP_M": 16},
        "fp8_gemm": {"BLOCK_M": 256, "BLOCK_N": 256, "BLOCK_K_BYTES": 128, "STAGES": 6, "GROUP_M": 16,
                     "K_SPLITS": 1},
    }
    if kernel_type not in defaults:
        raise ValueError(f"Unknown kernel type: {kernel_type}")
    return dict(defaults[kernel_type])
