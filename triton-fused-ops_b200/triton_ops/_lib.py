"""ctypes binding of the sm_100a library (``_lib/libtfo_b200.so``).

The library exports the C ABI declared in ``include/tfo_b200.h``. This module
loads it on first use, declares every entry point's argument types, maps
torch dtypes to the ABI's dtype codes, and turns non-zero status codes into
this package's exceptions. There is no fallback: if the library is missing or
cannot be loaded, every op raises :class:`~triton_ops.exceptions.TritonKernelError`.
"""

from __future__ import annotations

import ctypes
import os
import threading
from collections import OrderedDict
from pathlib import Path

import torch

from triton_ops.exceptions import TritonKernelError, UnsupportedDtypeError

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtfo_b200.so"

# dtype codes (include/tfo_b200.h)
F16, BF16, F32, U8, E4M3 = 0, 1, 2, 3, 4
_DTYPE_CODE = {
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.float32: F32,
    torch.uint8: U8,
}
if hasattr(torch, "float8_e4m3fn"):
    _DTYPE_CODE[torch.float8_e4m3fn] = E4M3

# status codes
OK, ERR_INVALID, ERR_DTYPE, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3, 4

# activations
ACT_CODE = {"silu": 0, "gelu": 1, "gelu_tanh": 2}

# layout of fp8_gemm's B operand
B_KN, B_NK = 0, 1

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_size = ctypes.c_size_t

# name -> (restype, argtypes)
_SIGNATURES = {
    "tfo_version": (ctypes.c_char_p, []),
    "tfo_last_error": (ctypes.c_char_p, []),
    "tfo_kernel_launches": (ctypes.c_ulonglong, []),
    "tfo_device_error_flags": (_c_int, [ctypes.POINTER(ctypes.c_uint32), _c_int]),
    "tfo_selftest_bounded_wait": (_c_int, [_c_i64, _c_vp]),
    "tfo_select_tile": (_c_int, [_c_int, _c_i64, _c_i64, _c_i64, _c_int, ctypes.POINTER(ctypes.c_int32), _c_int]),
    "tfo_rmsnorm_rope": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         ctypes.c_double, _c_int, _c_int, _c_int, _c_int, _c_vp],
    ),
    "tfo_rmsnorm_rope_quantize_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64, _c_int]),
    "tfo_rmsnorm_rope_quantize": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         ctypes.c_double, _c_int, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_int, _c_vp, _c_size, _c_vp],
    ),
    "tfo_fp8_scale_workspace_bytes": (_c_size, [_c_i64]),
    "tfo_fp8_compute_scale": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_size, _c_vp]),
    "tfo_fp8_quantize": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_size, _c_vp]),
    "tfo_fp8_quantize_noalloc": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_vp]),
    "tfo_fp8_dequantize": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_vp]),
    "tfo_fp8_compute_scale_rows": (_c_int, [_c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_vp]),
    "tfo_fp8_quantize_rows": (_c_int, [_c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_vp]),
    "tfo_fp8_quantize_per_token": (_c_int, [_c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_vp]),
    "tfo_fp8_dequantize_rows": (_c_int, [_c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_vp]),
    "tfo_fp8_gemm_scaled_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64, _c_int, _c_int]),
    "tfo_fp8_gemm_scaled": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_vp,
         _c_size, _c_vp],
    ),
    "tfo_fp8_gemm_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64, _c_int, _c_int]),
    "tfo_fp8_gemm": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_vp, _c_size, _c_vp],
    ),
    "tfo_fp8_linear": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_vp,
         _c_size, _c_vp],
    ),
    "tfo_fp8_prepare_weight": (_c_int, [_c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_vp]),
    "tfo_fp8_linear_prepared": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_vp,
         _c_size, _c_vp],
    ),
    "tfo_gated_mlp_quantize_workspace_bytes": (_c_size, [_c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int,
                                                          _c_int]),
    "tfo_gated_mlp_quantize": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_int, _c_vp,
         _c_size, _c_vp],
    ),
    "tfo_gated_mlp_workspace_bytes": (_c_size, [_c_i64, _c_i64, _c_i64, _c_int, _c_int]),
    "tfo_gated_mlp": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_vp, _c_size, _c_vp],
    ),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Loads the library once and declares its entry points."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("TFO_B200_LIB", LIB_PATH))
        if not path.exists():
            raise TritonKernelError(
                f"native library {path} is missing; build it with "
                "`python triton-fused-ops_b200/build.py` (there is no fallback path)"
            )
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as e:  # pragma: no cover - depends on the machine
            raise TritonKernelError(f"cannot load native library {path}: {e}") from e
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


_ext = None
_ext_tried = False


def ext():
    """The PyTorch extension over the C ABI (``_lib/_tfo_ext*.so``), or None.

    It serves the launch-latency-bound calls (dynamic quantize, FP8Linear's
    forward) in one C++ call; without it those calls take the ctypes path,
    which runs the same kernels. Not used when ``TFO_B200_LIB`` points the
    ctypes binding at another library, so that both always use one library.
    """
    global _ext, _ext_tried
    if _ext_tried:
        return _ext
    load()  # the extension links this library: load it first (outside _lock, which load() takes)
    with _lock:
        if _ext_tried:
            return _ext
        override = os.environ.get("TFO_B200_LIB")
        paths = sorted(LIB_PATH.parent.glob("_tfo_ext*.so"))
        if paths and (override is None or Path(override).resolve() == LIB_PATH.resolve()):
            import importlib.util

            spec = importlib.util.spec_from_file_location("triton_ops._tfo_ext", paths[0])
            mod = importlib.util.module_from_spec(spec)
            try:
                spec.loader.exec_module(mod)
                _ext = mod
            except ImportError:  # pragma: no cover - a stale build for another torch
                _ext = None
        _ext_tried = True
        return _ext


def raise_ext_error(exc: RuntimeError):
    """Re-raises an extension error ("tfo status <n>: ...") as the package's exception for that status."""
    msg = str(exc)
    if msg.startswith("tfo status "):
        status = int(msg.split()[2].rstrip(":"))
        text = msg.split(": ", 1)[1] if ": " in msg else msg
        if status == ERR_DTYPE:
            raise UnsupportedDtypeError(text) from exc
        raise TritonKernelError(f"{text} (status {status})") from exc
    raise exc


def declared_symbols() -> list[str]:
    return list(_SIGNATURES)


def dtype_code(dtype: torch.dtype, what: str = "tensor") -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise UnsupportedDtypeError(
            f"{what} has unsupported dtype {dtype}",
            dtype=dtype,
            supported_dtypes=list(_DTYPE_CODE),
            tensor_name=what,
        ) from None


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    """Raw handle of torch's current stream on t's device (no Stream object is built)."""
    if _raw_stream is not None:
        return _raw_stream(t.get_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def check(status: int, what: str) -> None:
    """Raises the package exception that matches a non-zero status code."""
    if status == OK:
        return
    msg = (load().tfo_last_error() or b"").decode(errors="replace")
    if status == ERR_DTYPE:
        raise UnsupportedDtypeError(f"{what}: {msg}")
    raise TritonKernelError(f"{what} failed (status {status}): {msg}")


def call(name: str, *args) -> None:
    """Calls entry point `name` and raises on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def device_error_flags(clear: bool = True) -> int:
    """Synchronises and returns (optionally clearing) the device error word."""
    flags = ctypes.c_uint32(0)
    check(load().tfo_device_error_flags(ctypes.byref(flags), int(clear)), "tfo_device_error_flags")
    return int(flags.value)


OP_FP8_GEMM, OP_GATED_MLP, OP_RMSNORM_ROPE = 0, 1, 2


def select_tile(op: int, M: int, N: int, K: int, aux: int) -> list:
    """The library's launch configuration for a shape (six integers, see tfo_select_tile)."""
    out = (ctypes.c_int32 * 6)()
    check(load().tfo_select_tile(op, M, N, K, aux, out, 6), "tfo_select_tile")
    return list(out)


def kernel_launches() -> int:
    """Kernels launched by the library so far in this process."""
    return int(load().tfo_kernel_launches())


def version() -> str:
    return load().tfo_version().decode()


# One grow-only scratch buffer per (device, stream): calls on one stream run in
# order, so each may reuse the buffer of the one before. (A fresh tensor from
# torch's caching allocator costs ~2 us of host time per call.) At most
# _WS_MAX_ENTRIES (device, stream) buffers are kept, least recently used first
# out, so a process that makes a stream per request does not keep one buffer
# per stream it ever used; clear_workspaces() drops them all (for example after
# destroying streams, since a new stream may receive a destroyed one's handle).
# Dropping a buffer is safe while kernels that use it are in flight: the
# caching allocator reuses its memory only in that stream's order.
# While a CUDA graph is being captured a fresh tensor is taken instead, so that
# no buffer is shared between a graph's private pool and eager calls.
_WS_MAX_ENTRIES = 8
_ws_cache: OrderedDict = OrderedDict()
_ws_lock = threading.Lock()
_is_capturing = getattr(torch.cuda, "is_current_stream_capturing", lambda: False)


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A scratch buffer of at least `nbytes` (and 16) bytes on `device` for the current stream."""
    n = max(int(nbytes), 16)
    if _is_capturing():
        return torch.empty(n, dtype=torch.uint8, device=device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, _raw_stream(idx) if _raw_stream is not None else torch.cuda.current_stream(idx).cuda_stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < n:
            buf = torch.empty(max(n, 2 * buf.numel() if buf is not None else n), dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
        _ws_cache.move_to_end(key)
        while len(_ws_cache) > _WS_MAX_ENTRIES:
            _ws_cache.popitem(last=False)
    return buf


def clear_workspaces() -> None:
    """Releases every cached scratch buffer (they return to torch's caching allocator)."""
    with _ws_lock:
        _ws_cache.clear()
    if _ext is not None:
        _ext.clear_workspaces()
