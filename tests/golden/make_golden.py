"""Generates the golden fixtures in this directory from the reference itself.

Runs the reference implementation's own PyTorch oracle functions
(LessUp/triton-fused-ops: triton_ops/kernels/rmsnorm_rope.py
``fused_rmsnorm_rope_reference``, triton_ops/kernels/fp8_quantize.py
``fp8_quantize_reference`` / ``fp8_dequantize_reference``,
triton_ops/models.py ``FP8Format.compute_scale``,
triton_ops/kernels/fp8_gemm.py ``fp8_gemm_reference``,
triton_ops/kernels/gated_mlp.py ``gated_mlp_reference``) on the CPU over
seeded inputs and stores inputs and outputs as compressed ``.npz`` files
(small cases) or SHA-256 digests (full-size codec case).

Usage (needs the reference source tree; not run by the tests)::

    python tests/golden/make_golden.py --reference /path/to/reference

The e4m3 cases use PyTorch's own ``torch.float8_e4m3fn`` cast as the golden
(the reference has no e4m3 path).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _np(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.float().numpy()  # bf16 values are exact in fp32
    if t.dtype == torch.float16:
        return t.numpy()  # stored as float16
    return t.numpy()


def rope_tables_torch(seq_len, head_dim, dtype):
    import torch

    inv = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    f = torch.outer(torch.arange(seq_len, dtype=torch.float64), inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().float().to(dtype), emb.sin().float().to(dtype)


def gen_rmsnorm(ref, torch):
    from triton_ops.kernels.rmsnorm_rope import fused_rmsnorm_rope_reference

    cases = {}
    specs = [
        # name, B, S, H, D, x dtype, w dtype, cs dtype, table kind, eps
        ("tiny_f16", 1, 1, 64, 64, torch.float16, torch.float16, torch.float16, "randn", 1e-6),
        ("small_f16_d32", 2, 16, 256, 32, torch.float16, torch.float16, torch.float16, "randn", 1e-6),
        ("small_bf16_d64", 2, 16, 256, 64, torch.bfloat16, torch.bfloat16, torch.bfloat16, "rope", 1e-6),
        ("small_f32_d64", 3, 7, 512, 64, torch.float32, torch.float32, torch.float32, "rope", 1e-5),
        ("module_f16x_f32w", 2, 9, 512, 128, torch.float16, torch.float32, torch.float32, "rope", 1e-6),
        ("cfg1_like_f16", 2, 12, 4096, 64, torch.float16, torch.float16, torch.float16, "rope", 1e-6),
        ("odd_rows_f16", 3, 5, 1024, 64, torch.float16, torch.float16, torch.float16, "randn", 1e-6),
    ]
    for i, (name, B, S, H, D, xd, wd, cd, kind, eps) in enumerate(specs):
        g = torch.Generator().manual_seed(100 + i)
        x = torch.randn(B, S, H, generator=g).to(xd)
        w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(wd)
        if kind == "rope":
            cos, sin = rope_tables_torch(S, D, cd)
        else:
            cos = torch.randn(S, D, generator=g).to(cd)
            sin = torch.randn(S, D, generator=g).to(cd)
        out = fused_rmsnorm_rope_reference(x, w, cos, sin, eps)
        cases[name] = dict(x=_np(x), w=_np(w), cos=_np(cos), sin=_np(sin), out=_np(out), eps=np.float64(eps),
                           x_dtype=str(xd).split(".")[-1], w_dtype=str(wd).split(".")[-1],
                           cs_dtype=str(cd).split(".")[-1])
    # 4-D tables [1, S, 1, D]
    g = torch.Generator().manual_seed(199)
    x = torch.randn(2, 8, 256, generator=g).half()
    w = torch.randn(256, generator=g).half()
    cos, sin = rope_tables_torch(8, 64, torch.float16)
    out = fused_rmsnorm_rope_reference(x, w, cos[None, :, None, :], sin[None, :, None, :])
    cases["table4d_f16"] = dict(x=_np(x), w=_np(w), cos=_np(cos[None, :, None, :]), sin=_np(sin[None, :, None, :]),
                                out=_np(out), eps=np.float64(1e-6), x_dtype="float16", w_dtype="float16",
                                cs_dtype="float16")
    return cases


def outlier_tensor(torch, shape, seed):
    """N(0,1) fp16 with 0.1% of entries set to +-200 (seeded positions and signs)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g)
    n = x.numel()
    k = int(round(n * 0.001))
    idx = torch.randperm(n, generator=g)[:k]
    sgn = torch.randint(0, 2, (k,), generator=g).float() * 2 - 1
    flat = x.view(-1)
    flat[idx] = 200.0 * sgn
    return x.half()


def gen_codec(ref, torch):
    from triton_ops.kernels.fp8_quantize import fp8_dequantize_reference, fp8_quantize_reference
    from triton_ops.models import FP8Format

    cases = {}

    def add(name, x, scale=None):
        q, s = fp8_quantize_reference(x, scale)
        s2 = FP8Format.compute_scale(x) if scale is None else scale
        dq = fp8_dequantize_reference(q, s, torch.float16)
        dq32 = fp8_dequantize_reference(q, s, torch.float32)
        cases[name] = dict(x=_np(x), x_dtype=str(x.dtype).split(".")[-1], q=q.numpy(),
                           scale=np.float32(s.item()), scale_model=np.float32(s2.item()),
                           given_scale=np.float32(scale.item()) if scale is not None else np.float32(np.nan),
                           dq_f16=_np(dq), dq_f32=_np(dq32))

    add("outliers_256x256_f16", outlier_tensor(torch, (256, 256), 7))
    g = torch.Generator().manual_seed(8)
    add("randn10_f16", (torch.randn(300, 77, generator=g) * 10).half())
    add("randn_bf16", torch.randn(64, 129, generator=g).bfloat16())
    add("randn_f32", torch.randn(1000, generator=g) * 3.7)
    add("zeros_f16", torch.zeros(100).half())
    add("small_f16", (torch.randn(100, generator=g) * 1e-4).half())
    # known-answer values at scale 1: rounding ties, clamps, signed zero, non-finite
    kat = []
    for k in range(-127, 128):
        t = (k + 0.5) * 448.0 / 127.0
        kat += [t, math.nextafter(t, -math.inf), math.nextafter(t, math.inf)]
    kat += [0.0, -0.0, 448.0, -448.0, 449.0, -1e30, 1e-30, float("inf"), float("-inf"), float("nan")]
    add("kat_f32_scale1", torch.tensor(kat, dtype=torch.float32), torch.tensor(1.0))
    add("kat_f16_scale1", torch.tensor(kat, dtype=torch.float32).half(), torch.tensor(1.0))
    add("given_scale_f16", (torch.randn(40, 40, generator=g) * 3).half(), torch.tensor(17.25))

    # full-size config-2 tensor: digests only
    x = outlier_tensor(torch, (4096, 4096), 2)
    q, s = fp8_quantize_reference(x)
    dq = fp8_dequantize_reference(q, s, torch.float16)
    full = dict(seed=2, shape=[4096, 4096], outlier_fraction=0.001, outlier_value=200.0,
                x_sha256=hashlib.sha256(x.numpy().tobytes()).hexdigest(),
                q_sha256=hashlib.sha256(q.numpy().tobytes()).hexdigest(),
                dq_f16_sha256=hashlib.sha256(dq.numpy().tobytes()).hexdigest(),
                scale=float(s.item()), scale_bits=int(np.float32(s.item()).view(np.uint32)))
    # e4m3 golden from torch's own cast
    e4 = {}
    g = torch.Generator().manual_seed(9)
    for name, x in (("e4m3_randn_f16", (torch.randn(128, 64, generator=g) * 5).half()),
                    ("e4m3_kat_f32", torch.tensor(kat, dtype=torch.float32))):
        sc = FP8Format.compute_scale(x[torch.isfinite(x)]) if name.endswith("f32") else FP8Format.compute_scale(x)
        c = (x.float() * sc).clamp(-448.0, 448.0)
        q8 = c.to(torch.float8_e4m3fn).view(torch.uint8)
        e4[name] = dict(x=_np(x), x_dtype=str(x.dtype).split(".")[-1], scale=np.float32(sc.item()), q=q8.numpy())
    return cases, full, e4


def gen_gemm(ref, torch):
    from triton_ops.kernels.fp8_gemm import fp8_gemm_reference
    from triton_ops.kernels.fp8_quantize import fp8_quantize_reference

    cases = {}
    for i, (M, N, K) in enumerate([(64, 96, 80), (33, 47, 129), (128, 256, 256), (16, 512, 384)]):
        g = torch.Generator().manual_seed(300 + i)
        a = torch.randn(M, K, generator=g).half()
        b = torch.randn(K, N, generator=g).half()
        qa, sa = fp8_quantize_reference(a)
        qb, sb = fp8_quantize_reference(b)
        c16 = fp8_gemm_reference(qa, qb, sa, sb, torch.float16)
        c32 = fp8_gemm_reference(qa, qb, sa, sb, torch.float32)
        cases[f"gemm_{M}x{N}x{K}"] = dict(qa=qa.numpy(), qb=qb.numpy(), sa=np.float32(sa.item()),
                                          sb=np.float32(sb.item()), c16=_np(c16), c32=_np(c32))
    return cases


def gen_mlp(ref, torch):
    from triton_ops.kernels.gated_mlp import gated_mlp_reference

    cases = {}
    specs = [
        ("silu_f16", 2, 8, 256, 384, "silu", torch.float16, torch.float16, 0.1),
        ("gelu_f16", 1, 24, 256, 256, "gelu", torch.float16, torch.float16, 0.1),
        ("silu_bf16", 2, 16, 256, 256, "silu", torch.bfloat16, torch.bfloat16, 0.05),
        ("silu_f16x_f32w", 2, 5, 256, 320, "silu", torch.float16, torch.float32, 0.02),
        ("gelu_f32", 1, 10, 128, 192, "gelu", torch.float32, torch.float32, 0.1),
    ]
    for i, (name, B, S, H, I, act, xd, wd, sd) in enumerate(specs):
        g = torch.Generator().manual_seed(400 + i)
        x = torch.randn(B, S, H, generator=g).to(xd)
        wg = (torch.randn(I, H, generator=g) * sd).to(wd)
        wu = (torch.randn(I, H, generator=g) * sd).to(wd)
        out = gated_mlp_reference(x, wg, wu, act)
        cases[name] = dict(x=_np(x), wg=_np(wg), wu=_np(wu), out=_np(out), act=act,
                           x_dtype=str(xd).split(".")[-1], w_dtype=str(wd).split(".")[-1])
    return cases


def save(name, cases):
    flat = {}
    for case, d in cases.items():
        for k, v in d.items():
            flat[f"{case}/{k}"] = np.asarray(v)
    np.savez_compressed(HERE / f"{name}.npz", **flat)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, help="root of the reference source tree")
    args = ap.parse_args()
    repo_pkg = str(HERE.parents[1] / "triton-fused-ops_b200")
    sys.path = [p for p in sys.path if Path(p or ".").resolve() != Path(repo_pkg).resolve()]
    sys.path.insert(0, args.reference)
    import torch
    import triton_ops as ref

    assert str(Path(ref.__file__).resolve()).startswith(str(Path(args.reference).resolve())), ref.__file__
    torch.set_num_threads(4)
    save("rmsnorm_rope", gen_rmsnorm(ref, torch))
    codec, full, e4 = gen_codec(ref, torch)
    save("fp8_codec", codec)
    save("fp8_e4m3", e4)
    (HERE / "fp8_codec_full.json").write_text(json.dumps(full, indent=2) + "\n")
    save("fp8_gemm", gen_gemm(ref, torch))
    save("gated_mlp", gen_mlp(ref, torch))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
