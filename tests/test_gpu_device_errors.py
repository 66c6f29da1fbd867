"""Device error word: clean after normal work; a bounded wait that runs out reports instead of hanging."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_timeout_sets_flag_and_context_survives(cuda):
    from triton_ops import _lib, fused_rmsnorm_rope

    _lib.device_error_flags(clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("tfo_selftest_bounded_wait", 200_000, stream)  # ~0.1 ms budget on a barrier nobody arrives on
    flags = _lib.device_error_flags(clear=True)
    assert flags & (1 << 3), f"expected the wait-timeout bit, got {flags:#x}"
    assert _lib.device_error_flags(clear=False) == 0
    # the context is still usable
    x = torch.randn(1, 4, 64, device="cuda", dtype=torch.float16)
    cs = torch.ones(4, 64, device="cuda", dtype=torch.float16)
    y = fused_rmsnorm_rope(x, torch.ones(64, device="cuda", dtype=torch.float16), cs, cs * 0)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()


def test_gemm_pipelines_finish_without_timeouts(cuda):
    from triton_ops import _lib, fp8_gemm, fused_gated_mlp

    _lib.device_error_flags(clear=True)
    a = torch.randn(512, 1024, device="cuda", dtype=torch.float16)
    b = torch.randn(1024, 768, device="cuda", dtype=torch.float16)
    fp8_gemm(a, b)
    fused_gated_mlp(a.view(1, 512, 1024), b.t().contiguous(), b.t().contiguous())
    assert _lib.device_error_flags(clear=True) == 0
