"""Launch-configuration selection: a static shape-keyed tile table, plus the
reference's tuner/cache classes kept for API compatibility."""

from triton_ops.autotuner.cache import ConfigCache
from triton_ops.autotuner.configs import FP8_GEMM_CONFIGS, GATED_MLP_CONFIGS, RMSNORM_ROPE_CONFIGS
from triton_ops.autotuner.tuner import TritonAutoTuner

__all__ = ["TritonAutoTuner", "RMSNORM_ROPE_CONFIGS", "GATED_MLP_CONFIGS", "FP8_GEMM_CONFIGS", "ConfigCache"]
