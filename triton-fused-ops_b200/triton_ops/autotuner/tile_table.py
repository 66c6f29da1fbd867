"""Static, shape-keyed tile table: the replacement for run-time autotuning.

The reference's ops launch fixed block sizes and its TritonAutoTuner is never
consulted on the launch path. Here every op picks its launch configuration
from fixed rules evaluated on the host inside the native library; this module
states the same rules in Python so callers can inspect what a shape will use
(``tests/`` checks that both agree through the library's ``tfo_select_tile``).
"""

from __future__ import annotations

from typing import Dict

B200_SMS = 148
CS_RAW_BYTES = 256  # raw cos/sin slot per row buffer of the warp-per-row RMSNorm+RoPE kernel
WARP_SLOTS = 2  # row buffers per warp of that kernel
WARP_BAR_BYTES = 256  # its mbarrier area


def _warp_rows_config(hidden: int, head_dim: int, elem: int, max_warps: int):
    row_bytes = hidden * elem
    cs_stride = (3 * (head_dim // 2) + 3) // 4 * 4
    fixed = WARP_BAR_BYTES + hidden * 4 + 128
    per_warp = WARP_SLOTS * (row_bytes + CS_RAW_BYTES) + cs_stride * 4
    limit = 227 * 1024
    if fixed + 8 * per_warp > limit:
        return 0, 0
    warps = min(max_warps, (limit - fixed) // per_warp)
    smem = ((WARP_BAR_BYTES + (hidden + warps * cs_stride) * 4 + 127) // 128) * 128 + warps * WARP_SLOTS * (
        row_bytes + CS_RAW_BYTES)
    return warps, smem


def rmsnorm_rope_config(hidden: int, head_dim: int, elem_bytes: int = 2, rows: int = 0,
                        sms: int = B200_SMS) -> Dict[str, int]:
    """Kernel of tfo_rmsnorm_rope for 16-byte-aligned rows of `hidden` elements.

    kernel 2 (warp per row) when a row is 4, 8 or 16 16-byte vectors per lane
    and there are at least two rows per resident warp; kernel 1 (CTA per row,
    `threads` threads with `vectors` vectors each); kernel 0 (generic).
    """
    e = 16 // elem_bytes
    dv = head_dim // e
    out = {"kernel": 0, "threads": 256, "vectors": 0, "full": 0, "smem": 0}
    vec = (hidden % e == 0 and head_dim % (2 * e) == 0 and 2 <= dv <= 32 and (dv & (dv - 1)) == 0
           and hidden // e <= 2048)
    if not vec:
        return out
    nvec = hidden // e
    full = (hidden // head_dim) * head_dim == hidden
    vpl = nvec // 32
    if nvec % 32 == 0 and vpl in (4, 8, 16):
        warps, smem = _warp_rows_config(hidden, head_dim, elem_bytes, 12 if vpl >= 16 else 16)
        if warps > 0 and rows >= 2 * sms * warps:
            return {"kernel": 2, "threads": warps, "vectors": vpl, "full": int(full), "smem": smem}
    for nv in (1, 2, 4, 8):
        threads = ((nvec + nv - 1) // nv + 31) // 32 * 32
        if threads <= 256:
            return {"kernel": 1, "threads": threads, "vectors": nv, "full": int(nv * threads == nvec and full),
                    "smem": 0}
    return out


def fp8_gemm_config(M: int, N: int, K: int, sms: int = B200_SMS, pair: bool = True) -> Dict[str, int]:
    """Tile of tfo_fp8_gemm for aligned operands (K a multiple of 16).

    256-column tiles, as two-CTA 256 x 256 tiles (cta_group::2) when M has more
    than one 128-row block; 128-column tiles for N <= 128 or for M <= 128 when
    the 256-column tiles would not cover the GPU; K split when the tiles fill
    less than half of the GPU.
    """
    bn = 256
    if N <= 128 or (M <= 128 and (N + 255) // 256 < sms):
        bn = 128
    cg = 2 if (bn == 256 and M > 128 and pair) else 1
    tiles = ((M + 128 * cg - 1) // (128 * cg)) * ((N + bn - 1) // bn)
    units = sms // cg
    num_k = (K + 127) // 128
    splits = 1
    if tiles < units // 2:
        splits = max(1, min(num_k // 4, units // tiles))
    # 32 KB stages; 48 KB for 128 x 256 single-CTA tiles; 20 KB (32-row A stages) for M <= 32
    stages = 6 if cg == 2 else (4 if bn == 256 else (11 if M <= 32 else 7))
    return {"BLOCK_M": 128 * cg, "BLOCK_N": bn, "CTAS_PER_MMA": cg, "STAGES": stages,
            "SPLIT_K": splits, "GROUP_M": 16}


def gated_mlp_config(M: int, N: int, K: int, sms: int = B200_SMS, pair: bool = True) -> Dict[str, int]:
    """Tile of tfo_gated_mlp: (128 or 256) rows x (128 gate + 128 up) columns."""
    cg = 2 if (M > 128 and pair) else 1
    return {"BLOCK_M": 128 * cg, "BLOCK_N": 128, "CTAS_PER_MMA": cg, "STAGES": 6 if cg == 2 else 4,
            "SPLIT_K": 1, "GROUP_M": 16}


def select(op: str, M: int, N: int, K: int) -> Dict[str, int]:
    if op == "fp8_gemm":
        return fp8_gemm_config(M, N, K)
    if op == "gated_mlp":
        return gated_mlp_config(M, N, K)
    if op == "rmsnorm_rope":
        return rmsnorm_rope_config(N, K, rows=M)
    raise KeyError(op)
