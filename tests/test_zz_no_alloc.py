"""tfo_fp8_quantize_noalloc: dynamic-scale quantize without any device allocation.

Some callers cannot allocate device memory at all (a framework that owns the
whole memory pool, a serving process with a fixed budget, a plugin without an
allocator), so this entry point keeps its scratch in a static device array of
the library instead of asking for a workspace. This test calls it through the
C ABI twice in a row, on different tensors, and requires exactly the codes and
scale of the allocating entry point (the codec is bit-exact, so the tolerance
is zero). It runs last so that a failure here cannot hide another test's.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(call):
    g = torch.Generator(device="cuda").manual_seed(40 + call)
    if call == 0:  # 4096 x 4096 fp16, N(0, 1) with 0.1% +-200 outliers, reference codec
        x = torch.randn(4096, 4096, device="cuda", generator=g).half()
        idx = torch.randperm(x.numel(), device="cuda", generator=g)[: x.numel() // 1000]
        x.view(-1)[idx] = 200.0
        return x, torch.uint8
    # ragged bf16 tensor, e4m3 bytes
    x = (torch.randn(1000, 333, device="cuda", generator=g) * 3).bfloat16()
    return x, torch.float8_e4m3fn


def test_noalloc_quantize_matches_allocating_entry_point(cuda):
    from triton_ops import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x, code_dtype = _inputs(call)
        n = x.numel()
        xc = _lib.dtype_code(x.dtype)
        oc = _lib.dtype_code(code_dtype)

        # existing entry point, caller-provided workspace
        ws_bytes = lib.tfo_fp8_scale_workspace_bytes(n)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        q_ref = torch.empty(x.shape, dtype=code_dtype, device="cuda")
        s_ref = torch.empty((), dtype=torch.float32, device="cuda")
        assert lib.tfo_fp8_quantize(x.data_ptr(), n, xc, None, s_ref.data_ptr(), q_ref.data_ptr(), oc,
                                    ws.data_ptr(), ws_bytes, stream) == _lib.OK

        # no-allocation entry point: outputs from the caller, no workspace
        q = torch.full(x.shape, 7, dtype=torch.uint8, device="cuda").view(code_dtype)
        s = torch.full((), -1.0, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        status = lib.tfo_fp8_quantize_noalloc(x.data_ptr(), n, xc, s.data_ptr(), q.data_ptr(), oc, stream)
        assert status == _lib.OK, lib.tfo_last_error().decode()
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before

        assert np.float32(s.item()).view(np.uint32) == np.float32(s_ref.item()).view(np.uint32)
        assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8)), f"call {call}: codes differ"
    assert _lib.device_error_flags(clear=True) == 0


def _quantize_both(lib, x, code_dtype, stream):
    """Codes and scale from tfo_fp8_quantize (workspace) and from the no-allocation entry point."""
    from triton_ops import _lib

    n = x.numel()
    xc, oc = _lib.dtype_code(x.dtype), _lib.dtype_code(code_dtype)
    ws_bytes = lib.tfo_fp8_scale_workspace_bytes(n)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    q_ref = torch.empty(x.shape, dtype=code_dtype, device="cuda")
    s_ref = torch.empty((), dtype=torch.float32, device="cuda")
    assert lib.tfo_fp8_quantize(x.data_ptr() if n else None, n, xc, None, s_ref.data_ptr(),
                                q_ref.data_ptr() if n else None, oc, ws.data_ptr(), max(ws_bytes, 16), stream) == _lib.OK
    q = torch.full(x.shape, 7, dtype=torch.uint8, device="cuda").view(code_dtype)
    s = torch.full((), -1.0, dtype=torch.float32, device="cuda")
    status = lib.tfo_fp8_quantize_noalloc(x.data_ptr() if n else None, n, xc, s.data_ptr(),
                                          q.data_ptr() if n else None, oc, stream)
    assert status == _lib.OK, lib.tfo_last_error().decode()
    torch.cuda.synchronize()
    return q, s, q_ref, s_ref


def test_noalloc_empty_and_unaligned_inputs(cuda):
    """numel == 0 (scale 1.0, amax-partials kernel then the scale finalisation)
    and a view starting 2 bytes past a 16-byte boundary (the kernels' scalar,
    non-vector path), each bit for bit against the allocating entry point."""
    from triton_ops import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    q, s, q_ref, s_ref = _quantize_both(lib, torch.empty(0, device="cuda", dtype=torch.float16), torch.uint8, stream)
    assert s.item() == 1.0 and s_ref.item() == 1.0
    g = torch.Generator(device="cuda").manual_seed(44)
    base = torch.randn(300001, device="cuda", generator=g).half()
    for x, code_dtype in ((base[1:], torch.uint8), (base[1:100001], torch.float8_e4m3fn)):
        assert x.data_ptr() % 16 == 2
        q, s, q_ref, s_ref = _quantize_both(lib, x, code_dtype, stream)
        assert np.float32(s.item()).view(np.uint32) == np.float32(s_ref.item()).view(np.uint32)
        assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    assert _lib.device_error_flags(clear=True) == 0


def test_noalloc_rejects_bad_arguments(cuda):
    from triton_ops import _lib

    lib = _lib.load()
    x = torch.zeros(16, device="cuda", dtype=torch.float16)
    out = torch.empty(16, dtype=torch.uint8, device="cuda")
    assert lib.tfo_fp8_quantize_noalloc(x.data_ptr(), 16, 7, None, out.data_ptr(), 3, None) == _lib.ERR_DTYPE
    assert lib.tfo_fp8_quantize_noalloc(x.data_ptr(), 16, 0, None, out.data_ptr(), 3, None) == _lib.ERR_INVALID
    assert b"NULL" in lib.tfo_last_error()
