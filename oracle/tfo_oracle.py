"""CPU oracle for the fused transformer-op hot path (numpy).

TEST INFRASTRUCTURE ONLY. This package restates, operation by operation, the
reference implementation's PyTorch oracles (LessUp/triton-fused-ops) so the
CUDA kernels can be checked against them. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it,
and only as the checker or the timed CPU baseline; the library never calls it.

Parity pins: ``tests/golden/make_golden.py`` ran the reference's own oracle
functions (imported from the reference source tree) on seeded inputs and
stored their outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks this module against every stored case (bit-exact for the 8-bit codes
and scales, within one output ulp for the float ops).

Arrays: every float tensor is held as float32 whose values are representable
in the named dtype ("f16", "bf16", "f32"); ``round_to`` performs the
round-to-nearest-even casts the reference does with ``.to(dtype)``.
"""

from __future__ import annotations

import numpy as np

FP8_MAX = np.float32(448.0)
_F32 = np.float32


# ---------------------------------------------------------------------------
# dtype rounding
# ---------------------------------------------------------------------------
def bf16_round(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16, returned as float32 (NaN kept)."""
    a = np.asarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), out).astype(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to `dtype` (RNE), keeping float32 storage."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return a.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_round(a)
    if dtype == "f32":
        return a
    raise ValueError(dtype)


# ---------------------------------------------------------------------------
# RMSNorm + RoPE  (reference: triton_ops/kernels/rmsnorm_rope.py:305-383)
# ---------------------------------------------------------------------------
def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float, x_dtype: str) -> np.ndarray:
    """x / sqrt(mean(x^2) + eps) * weight in fp32, rounded to x's dtype (rmsnorm_rope.py:305-319)."""
    xf = np.asarray(x, dtype=_F32)
    with np.errstate(over="ignore", invalid="ignore"):
        ms = np.mean(xf * xf, axis=-1, keepdims=True, dtype=_F32)
        rms = np.sqrt(ms + _F32(eps), dtype=_F32)
        y = (xf / rms) * np.asarray(weight, dtype=_F32)
    return round_to(y, x_dtype)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, x_dtype: str) -> np.ndarray:
    """Rotate-half RoPE per head with cos/sin[:seq_len, :head_dim/2] (rmsnorm_rope.py:322-353)."""
    b, s, h = x.shape
    d = cos.shape[-1]
    half = d // 2
    xh = np.asarray(x, dtype=_F32).reshape(b, s, h // d, d)
    x1, x2 = xh[..., :half], xh[..., half:]
    c = np.asarray(cos, dtype=_F32)[:s, :half][None, :, None, :]
    sn = np.asarray(sin, dtype=_F32)[:s, :half][None, :, None, :]
    with np.errstate(over="ignore", invalid="ignore"):
        o1 = x1 * c - x2 * sn
        o2 = x1 * sn + x2 * c
    out = np.concatenate([o1, o2], axis=-1).reshape(b, s, h)
    return round_to(out, x_dtype)


def rmsnorm_rope(x, weight, cos, sin, eps: float, x_dtype: str) -> np.ndarray:
    """RMSNorm then RoPE; 4-D [1, S, 1, D] tables are squeezed first (rmsnorm_rope.py:356-383)."""
    cos = np.asarray(cos)
    sin = np.asarray(sin)
    if cos.ndim == 4:
        cos = cos[0, :, 0, :]
        sin = sin[0, :, 0, :]
    return rope(rmsnorm(x, weight, eps, x_dtype), cos, sin, x_dtype)


# ---------------------------------------------------------------------------
# FP8 codec  (reference: triton_ops/models.py:282-299,
#             triton_ops/kernels/fp8_quantize.py:258-312)
# ---------------------------------------------------------------------------
def compute_scale(x: np.ndarray) -> np.float32:
    """448 / max|x| evaluated in double and rounded to fp32; 1.0 for an all-zero tensor."""
    amax = np.max(np.abs(np.asarray(x, dtype=_F32))) if np.size(x) else _F32(0)
    if amax == 0:
        return _F32(1.0)
    return _F32(448.0 / float(amax))


def quantize_ref(x: np.ndarray, scale) -> np.ndarray:
    """uint8 codes int8(rint(clamp(x*s, +-448) / 448 * 127)) + 128 (fp8_quantize.py:280-287).

    NaN inputs encode as 128 (the value PyTorch's float->int8 cast gives NaN on the CPU).
    """
    s = _F32(scale)
    with np.errstate(over="ignore", invalid="ignore"):
        c = np.asarray(x, dtype=_F32) * s
        c = np.clip(c, -FP8_MAX, FP8_MAX)
        t = (c / FP8_MAX) * _F32(127.0)
        q = np.rint(t)
    q = np.where(np.isnan(q), 0, q).astype(np.int32)
    return ((q + 128) & 0xFF).astype(np.uint8)


def dequantize_ref(u: np.ndarray, scale, out_dtype: str) -> np.ndarray:
    """((u - 128) / 127 * 448) / scale in fp32, rounded to out_dtype (fp8_quantize.py:305-312)."""
    xi = np.asarray(u).astype(np.int32) - 128
    xf = (xi.astype(_F32) / _F32(127.0)) * FP8_MAX
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        return round_to(xf / _F32(scale), out_dtype)


def _e4m3_table() -> np.ndarray:
    codes = np.arange(0x7F)
    e = codes >> 3
    m = codes & 7
    vals = np.where(e == 0, m * 2.0**-9, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))
    return vals.astype(np.float64)


_E4M3 = _e4m3_table()


def e4m3_encode(c: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn bytes, round-to-nearest-even, |c| <= 448 expected, NaN -> 0x7F|sign."""
    c = np.asarray(c, dtype=_F32)
    a = np.abs(c).astype(np.float64)
    idx = np.clip(np.searchsorted(_E4M3, a), 1, len(_E4M3) - 1)
    lo, hi = idx - 1, idx
    d_lo = a - _E4M3[lo]
    d_hi = _E4M3[hi] - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(a >= _E4M3[-1], len(_E4M3) - 1, code)
    code = np.where(np.isnan(c), 0x7F, code)
    sign = np.signbit(c).astype(np.int64) << 7
    return (code | sign).astype(np.uint8)


def e4m3_decode(q: np.ndarray) -> np.ndarray:
    q = np.asarray(q).astype(np.int64)
    mag = q & 0x7F
    vals = np.where(mag == 0x7F, np.nan, _E4M3[np.minimum(mag, 0x7E)])
    vals = np.where(q & 0x80, -vals, vals)
    return vals.astype(_F32)


def quantize_e4m3(x: np.ndarray, scale) -> np.ndarray:
    """e4m3fn bytes of clamp(x * s, +-448) (the float8 option of quantize_fp8)."""
    with np.errstate(over="ignore", invalid="ignore"):
        c = np.clip(np.asarray(x, dtype=_F32) * _F32(scale), -FP8_MAX, FP8_MAX)
    return e4m3_encode(c)


def dequantize_e4m3(q: np.ndarray, scale, out_dtype: str) -> np.ndarray:
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        return round_to(e4m3_decode(q) / _F32(scale), out_dtype)


# ---------------------------------------------------------------------------
# FP8 GEMM  (reference: triton_ops/kernels/fp8_gemm.py:190-225)
# ---------------------------------------------------------------------------
def fp8_decode_operand(codes: np.ndarray, scale) -> np.ndarray:
    """uint8 code -> (u - 128) / 127 * 448 / scale, elementwise fp32 (fp8_gemm.py:210-218)."""
    xi = np.asarray(codes).astype(np.int32) - 128
    return ((xi.astype(_F32) / _F32(127.0)) * FP8_MAX) / _F32(scale)


def fp8_gemm(a_codes, b_codes, a_scale, b_scale, out_dtype: str = "f16") -> np.ndarray:
    """dec(a) @ dec(b) with the decoded fp32 operands; products summed in float64 (an exact-er
    stand-in for the reference's fp32 matmul), then rounded to fp32 and to out_dtype."""
    a = fp8_decode_operand(a_codes, a_scale).astype(np.float64)
    b = fp8_decode_operand(b_codes, b_scale).astype(np.float64)
    return round_to((a @ b).astype(_F32), out_dtype)


def fp8_gemm_e4m3(a_codes, b_codes, a_scale, b_scale, out_dtype: str = "f16") -> np.ndarray:
    a = (e4m3_decode(a_codes) / _F32(a_scale)).astype(np.float64)
    b = (e4m3_decode(b_codes) / _F32(b_scale)).astype(np.float64)
    return round_to((a @ b).astype(_F32), out_dtype)


# ---------------------------------------------------------------------------
# Gated MLP  (reference: triton_ops/kernels/gated_mlp.py:221-251)
# ---------------------------------------------------------------------------
def _erf(v: np.ndarray) -> np.ndarray:
    from scipy.special import erf

    return erf(v)


def activation(u: np.ndarray, kind: str) -> np.ndarray:
    u = np.asarray(u, dtype=np.float64)
    with np.errstate(over="ignore"):
        if kind == "silu":
            return u / (1.0 + np.exp(-u))
        if kind == "gelu":
            return 0.5 * u * (1.0 + _erf(u / np.sqrt(2.0)))
        if kind == "gelu_tanh":
            return 0.5 * u * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (u + 0.044715 * u**3)))
    raise ValueError(kind)


def gated_mlp(x, w_gate, w_up, kind: str, x_dtype: str) -> np.ndarray:
    """gate = x W_g^T, up = x W_u^T (float64 sums), out = gate * act(up) rounded to x's dtype.

    The activation is applied to the up projection, as the reference does.
    """
    x2 = np.asarray(x, dtype=np.float64).reshape(-1, np.shape(x)[-1])
    g = x2 @ np.asarray(w_gate, dtype=np.float64).T
    u = x2 @ np.asarray(w_up, dtype=np.float64).T
    out = (g * activation(u, kind)).astype(_F32)
    return round_to(out, x_dtype).reshape(*np.shape(x)[:-1], -1)


def gated_mlp_f32(x, w_gate, w_up, kind: str, x_dtype: str) -> np.ndarray:
    """The reference's arithmetic exactly as it runs on the CPU: fp32 projections
    (F.linear on fp32-cast operands), fp32 activation, fp32 product, cast to x's
    dtype (gated_mlp.py:238-251). Used as the timed CPU baseline."""
    x2 = np.asarray(x, dtype=_F32).reshape(-1, np.shape(x)[-1])
    g = x2 @ np.asarray(w_gate, dtype=_F32).T
    u = x2 @ np.asarray(w_up, dtype=_F32).T
    with np.errstate(over="ignore"):
        if kind == "silu":
            a = u / (_F32(1.0) + np.exp(-u))
        else:
            a = activation(u, kind).astype(_F32)
    return round_to(g * a, x_dtype).reshape(*np.shape(x)[:-1], -1)


# ---------------------------------------------------------------------------
# synthetic inputs shared by the tests, bench and smoke
# ---------------------------------------------------------------------------
def rope_tables(seq_len: int, head_dim: int, base: float = 10000.0) -> tuple[np.ndarray, np.ndarray]:
    """HF-style cos/sin [seq_len, head_dim] = cat(f, f) for f = pos * base^(-2i/head_dim) (fp32)."""
    inv = 1.0 / (base ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))
    f = np.outer(np.arange(seq_len, dtype=np.float64), inv)
    emb = np.concatenate([f, f], axis=-1)
    return np.cos(emb).astype(_F32), np.sin(emb).astype(_F32)


def rel_fro(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))
