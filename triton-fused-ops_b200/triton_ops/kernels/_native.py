"""Handles that stand in for the reference's per-op Triton kernel objects.

The reference exports its ``@triton.jit`` functions (``fused_rmsnorm_rope_kernel``,
``fp8_gemm_kernel`` ...) from ``triton_ops.kernels``. Here each name is bound to
a :class:`NativeKernel` that records which C-ABI entry point (and CUDA kernel
family) implements it, so imports keep working; the ops themselves are the
supported way to launch the kernels.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class NativeKernel:
    name: str
    entry_point: str
    description: str

    def __getitem__(self, grid):
        raise TypeError(
            f"{self.name} is a native sm_100a kernel launched through {self.entry_point}(); "
            "call the corresponding op instead of indexing it with a grid"
        )

    def __repr__(self) -> str:
        return f"<native kernel {self.name} via {self.entry_point}>"
