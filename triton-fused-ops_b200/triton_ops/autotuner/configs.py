"""Configuration spaces (kept for API compatibility with the reference's autotuner).

The launch path does not search these: tiles come from
:mod:`triton_ops.autotuner.tile_table`. The spaces list the tile options the
native kernels are built with, so a user-driven search stays meaningful.
"""

from itertools import product
from typing import Any, Dict, List

RMSNORM_ROPE_CONFIGS = {"threads": [32, 64, 128, 256], "vectors_per_thread": [1, 2, 4, 8]}
GATED_MLP_CONFIGS = {"BLOCK_M": [128], "BLOCK_N": [128], "BLOCK_K_BYTES": [128], "STAGES": [4], "GROUP_M": [16]}
FP8_GEMM_CONFIGS = {"BLOCK_M": [128], "BLOCK_N": [128, 256], "BLOCK_K_BYTES": [128], "STAGES": [4], "GROUP_M": [16]}


def generate_configs(config_space: Dict[str, List[Any]]) -> List[Dict[str, Any]]:
    """Cartesian product of a configuration space."""
    keys = list(config_space)
    return [dict(zip(keys, values)) for values in product(*(config_space[k] for k in keys))]


def filter_valid_configs(configs: List[Dict[str, Any]], problem_size=None, max_shared_memory: int = 232448,
                         dtype_size: int = 2) -> List[Dict[str, Any]]:
    """Drops configurations whose operand ring would not fit in shared memory."""
    out = []
    for c in configs:
        bm, bn, kb, st = c.get("BLOCK_M", 0), c.get("BLOCK_N", 0), c.get("BLOCK_K_BYTES", 0), c.get("STAGES", 1)
        if bm and bn and kb and (bm + bn) * kb * st > max_shared_memory:
            continue
        out.append(c)
    return out


def get_default_config(kernel_type: str) -> Dict[str, Any]:
    defaults = {
        "rmsnorm_rope": {"threads": 256, "vectors_per_thread": 2},
        "gated_mlp": generate_configs(GATED_MLP_CONFIGS)[0],
        "fp8_gemm": {"BLOCK_M": 128, "BLOCK_N": 256, "BLOCK_K_BYTES": 128, "STAGES": 4, "GROUP_M": 16},
    }
    if kernel_type not in defaults:
        raise ValueError(f"Unknown kernel type: {kernel_type}")
    return dict(defaults[kernel_type])
