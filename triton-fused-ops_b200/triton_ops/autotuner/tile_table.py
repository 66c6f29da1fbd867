"""Static, shape-keyed tile table: the replacement for run-time autotuning.

The reference's ops launch fixed block sizes and its TritonAutoTuner is never
consulted on the launch path. Here every op picks its launch configuration
from fixed rules evaluated on the host inside the native library; this module
states the same rules in Python so callers can inspect what a shape will use
(``tests/`` checks both agree through ``tfo_select_tile``).
"""

from __future__ import annotations

from typing import Dict

B200_SMS = 148


def rmsnorm_rope_config(hidden: int, head_dim: int, elem_bytes: int = 2) -> Dict[str, int]:
    """Threads per row and 16-byte vectors per thread of the one-pass kernel."""
    e = 16 // elem_bytes
    dv = head_dim // e if head_dim % (2 * e) == 0 else 0
    vec = hidden % e == 0 and dv >= 2 and dv <= 32 and (dv & (dv - 1)) == 0 and hidden // e <= 2048
    if not vec:
        return {"path": 0, "threads": 256, "vectors_per_thread": 0}
    nvec = hidden // e
    for nv in (1, 2, 4, 8):
        threads = ((nvec + nv - 1) // nv + 31) // 32 * 32
        if threads <= 256:
            return {"path": 1, "threads": threads, "vectors_per_thread": nv}
    return {"path": 0, "threads": 256, "vectors_per_thread": 0}


def fp8_gemm_config(M: int, N: int, K: int, sms: int = B200_SMS) -> Dict[str, int]:
    """UMMA tile of the FP8 GEMM: BLOCK_M x BLOCK_N x 128 bytes of K, 4 stages."""
    mb = (M + 127) // 128
    if N <= 128:
        bn = 128
    elif mb * ((N + 255) // 256) >= sms:
        bn = 256
    else:
        bn = 128
    return {"BLOCK_M": 128, "BLOCK_N": bn, "BLOCK_K_BYTES": 128, "STAGES": 4, "GROUP_M": 16}


def gated_mlp_config(M: int, N: int, K: int, sms: int = B200_SMS) -> Dict[str, int]:
    """UMMA tile of the gated MLP: 128 rows x (128 gate + 128 up) columns, 4 stages."""
    return {"BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K_BYTES": 128, "STAGES": 4, "GROUP_M": 16}


def select(op: str, M: int, N: int, K: int) -> Dict[str, int]:
    if op == "fp8_gemm":
        return fp8_gemm_config(M, N, K)
    if op == "gated_mlp":
        return gated_mlp_config(M, N, K)
    if op == "rmsnorm_rope":
        return rmsnorm_rope_config(N, K)
    raise KeyError(op)
