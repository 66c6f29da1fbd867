"""The numpy oracle against the reference's own outputs (golden fixtures).

Bit-exact for the 8-bit codes, scales and dequantized values. RMSNorm+RoPE:
>99% of 16-bit outputs bit-identical, the rest within the error one ulp of
the normalised value can cause (the reference's fp32 sum order cannot be
reproduced). GEMMs: relative Frobenius error < 1e-5 in fp32 (the oracle sums
in float64, the reference in fp32), < 1e-3 after rounding to 16 bits.
"""

import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN, load_golden
from oracle import tfo_oracle as O

DT = {"float16": "f16", "bfloat16": "bf16", "float32": "f32"}


def _ulp_diff(a, b, dtype):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if dtype == "f16":
        ai = a.astype(np.float16).view(np.int16).astype(np.int64)
        bi = b.astype(np.float16).view(np.int16).astype(np.int64)
    elif dtype == "bf16":
        ai = (a.view(np.int32) >> 16).astype(np.int64)
        bi = (b.view(np.int32) >> 16).astype(np.int64)
    else:
        ai = a.view(np.int32).astype(np.int64)
        bi = b.view(np.int32).astype(np.int64)
    # map sign-magnitude to a monotonic integer line
    bits = 15 if dtype in ("f16", "bf16") else 31
    ai = np.where(ai < 0, -(ai & ((1 << bits) - 1)), ai)
    bi = np.where(bi < 0, -(bi & ((1 << bits) - 1)), bi)
    both_nan = np.isnan(a) & np.isnan(b)
    return np.where(both_nan, 0, np.abs(ai - bi))


ULP_AT_ONE = {"f16": 2.0**-10, "bf16": 2.0**-7, "f32": 2.0**-23}


def rope_pair_bound(x, w, cos, sin, eps, xd):
    """Per-output error bound for a one-ulp difference in the normalised values.

    The reference's fp32 sum order cannot be reproduced, so mean(x^2) may differ
    in its last bit, which moves some normalised values y by one ulp of x's
    dtype; the rotation then moves each output by at most
    ulp(y1)*|cos| + ulp(y2)*|sin|, plus one rounding ulp of the output.
    """
    y = O.rmsnorm(x, w, eps, xd)
    cos = np.asarray(cos, np.float32)
    sin = np.asarray(sin, np.float32)
    if cos.ndim == 4:
        cos, sin = cos[0, :, 0, :], sin[0, :, 0, :]
    b, s, h = y.shape
    d = cos.shape[-1]
    half = d // 2
    yh = np.abs(y.reshape(b, s, h // d, 2, half))
    mag = yh[..., 0, :] + yh[..., 1, :]
    cs = np.maximum(np.abs(cos[:s, :half]), np.abs(sin[:s, :half]))[None, :, None, :]
    bound = 2 * ULP_AT_ONE[xd] * mag * cs
    return np.concatenate([bound, bound], axis=-1).reshape(b, s, h)


@pytest.mark.parametrize("case", sorted(load_golden("rmsnorm_rope")))
def test_rmsnorm_rope_oracle_matches_reference(case):
    c = load_golden("rmsnorm_rope")[case]
    xd = DT[str(c["x_dtype"])]
    out = O.rmsnorm_rope(c["x"], c["w"], c["cos"], c["sin"], float(c["eps"]), xd)
    ref = np.asarray(c["out"], np.float32)
    exact = (out == ref) | (np.isnan(out) & np.isnan(ref))
    if xd != "f32":  # fp32 outputs expose every last-bit difference of the sum; narrow dtypes hide most
        assert exact.mean() > 0.99, f"{case}: only {exact.mean():.4f} bit-identical"
    k = 1.0 if xd != "f32" else 4.0
    bound = k * rope_pair_bound(c["x"], c["w"], c["cos"], c["sin"], float(c["eps"]), xd)
    err = np.abs(out - ref)
    ok = exact | (err <= bound + k * ULP_AT_ONE[xd] * np.abs(ref))
    assert ok.all(), f"{case}: {np.count_nonzero(~ok)} outputs beyond the one-ulp-of-y bound"


@pytest.mark.parametrize("case", sorted(load_golden("fp8_codec")))
def test_codec_oracle_bit_exact(case):
    c = load_golden("fp8_codec")[case]
    x = c["x"]
    given = float(c["given_scale"])
    scale = O.compute_scale(x) if np.isnan(given) else np.float32(given)
    assert np.float32(scale).view(np.uint32) == np.float32(c["scale"]).view(np.uint32)
    if np.isnan(given):
        assert np.float32(scale).view(np.uint32) == np.float32(c["scale_model"]).view(np.uint32)
    q = O.quantize_ref(x, scale)
    np.testing.assert_array_equal(q, c["q"])
    np.testing.assert_array_equal(O.dequantize_ref(q, scale, "f16"), np.asarray(c["dq_f16"], np.float32))
    np.testing.assert_array_equal(O.dequantize_ref(q, scale, "f32"), c["dq_f32"])


def full_codec_input():
    """The 4096 x 4096 outlier tensor of the golden digest, regenerated from its seed."""
    import torch

    meta = json.loads((GOLDEN / "fp8_codec_full.json").read_text())
    g = torch.Generator().manual_seed(meta["seed"])
    x = torch.randn(*meta["shape"], generator=g)
    n = x.numel()
    k = int(round(n * meta["outlier_fraction"]))
    idx = torch.randperm(n, generator=g)[:k]
    sgn = torch.randint(0, 2, (k,), generator=g).float() * 2 - 1
    x.view(-1)[idx] = meta["outlier_value"] * sgn
    return x.half().numpy(), meta


def test_codec_oracle_full_size_digest():
    x, meta = full_codec_input()
    assert hashlib.sha256(x.tobytes()).hexdigest() == meta["x_sha256"], "input regeneration drifted"
    s = O.compute_scale(x)
    assert int(np.float32(s).view(np.uint32)) == meta["scale_bits"]
    q = O.quantize_ref(x, s)
    assert hashlib.sha256(q.tobytes()).hexdigest() == meta["q_sha256"]
    dq = O.dequantize_ref(q, s, "f16").astype(np.float16)
    assert hashlib.sha256(dq.tobytes()).hexdigest() == meta["dq_f16_sha256"]


@pytest.mark.parametrize("case", sorted(load_golden("fp8_e4m3")))
def test_e4m3_oracle_matches_torch_cast(case):
    c = load_golden("fp8_e4m3")[case]
    q = O.quantize_e4m3(c["x"], c["scale"])
    np.testing.assert_array_equal(q, c["q"])


@pytest.mark.parametrize("case", sorted(load_golden("fp8_gemm")))
def test_fp8_gemm_oracle_matches_reference(case):
    c = load_golden("fp8_gemm")[case]
    out32 = O.fp8_gemm(c["qa"], c["qb"], c["sa"], c["sb"], "f32")
    assert O.rel_fro(out32, c["c32"]) < 1e-5
    out16 = O.fp8_gemm(c["qa"], c["qb"], c["sa"], c["sb"], "f16")
    assert O.rel_fro(out16, c["c16"]) < 1e-3
    assert (out16 == np.asarray(c["c16"], np.float32)).mean() > 0.95


@pytest.mark.parametrize("case", sorted(load_golden("gated_mlp")))
def test_gated_mlp_oracle_matches_reference(case):
    c = load_golden("gated_mlp")[case]
    xd = DT[str(c["x_dtype"])]
    out = O.gated_mlp(c["x"], c["wg"], c["wu"], str(c["act"]), xd)
    assert O.rel_fro(out, c["out"]) < (1e-5 if xd == "f32" else 1e-3)


def test_codec_oracle_ties_round_half_even():
    # (k + 0.5) * 448 / 127 at scale 1 rounds to the even neighbour when it is an exact tie in fp32
    t = np.float32(0.5 * 448.0 / 127.0)
    assert O.quantize_ref(np.array([0.0], np.float32), 1.0)[0] == 128
    assert O.quantize_ref(np.array([448.0, -448.0, 1e9, -1e9], np.float32), 1.0).tolist() == [255, 1, 255, 1]
    assert O.quantize_ref(np.array([np.nan], np.float32), 1.0)[0] == 128
    assert abs(int(O.quantize_ref(np.array([t], np.float32), 1.0)[0]) - 128) <= 1
