"""Output comparison helpers (API of the reference's CorrectnessVerifier)."""

from typing import Any, Dict, Tuple

import torch


class CorrectnessVerifier:
    """Element-wise check: |a - e| <= atol or |a - e| / |e| <= rtol."""

    def __init__(self, rtol: float = 1e-3, atol: float = 1e-5):
        self.rtol = rtol
        self.atol = atol

    def verify(self, actual: torch.Tensor, expected: torch.Tensor) -> Tuple[bool, Dict[str, Any]]:
        if actual.shape != expected.shape:
            return False, {"error": f"shape mismatch: {tuple(actual.shape)} vs {tuple(expected.shape)}"}
        a, e = actual.float(), expected.float()
        abs_diff = (a - e).abs()
        rel_diff = abs_diff / e.abs().clamp_min(1e-12)
        ok = (abs_diff <= self.atol) | (rel_diff <= self.rtol) | (torch.isnan(a) & torch.isnan(e))
        details = {
            "max_abs_diff": abs_diff.nan_to_num(0).max().item() if abs_diff.numel() else 0.0,
            "max_rel_diff": rel_diff.nan_to_num(0).max().item() if rel_diff.numel() else 0.0,
            "mean_abs_diff": abs_diff.nan_to_num(0).mean().item() if abs_diff.numel() else 0.0,
            "num_violations": int((~ok).sum().item()),
            "total_elements": a.numel(),
            "rtol": self.rtol,
            "atol": self.atol,
        }
        return bool(ok.all().item()), details

    def verify_allclose(self, actual: torch.Tensor, expected: torch.Tensor) -> bool:
        return torch.allclose(actual.float(), expected.float(), rtol=self.rtol, atol=self.atol)

    def compute_relative_error(self, actual: torch.Tensor, expected: torch.Tensor) -> float:
        """Relative Frobenius error ||a - e|| / ||e||."""
        a, e = actual.float(), expected.float()
        den = e.norm().item()
        return (a - e).norm().item() / den if den > 0 else (a - e).norm().item()


def verify_fp8_accuracy(fp8_output: torch.Tensor, fp16_output: torch.Tensor, max_relative_error: float = 0.01):
    """Mean element-wise relative error of an FP8 result against a higher-precision one."""
    rel = (fp8_output.float() - fp16_output.float()).abs() / (fp16_output.float().abs() + 1e-6)
    mean_rel = rel.mean().item()
    return mean_rel <= max_relative_error, {"mean_relative_error": mean_rel, "max_relative_error": rel.max().item()}


def verify_nan_inf_propagation(input_tensor: torch.Tensor, output_tensor: torch.Tensor) -> Tuple[bool, Dict]:
    """True when non-finite inputs leave non-finite outputs."""
    has_bad_in = bool((~torch.isfinite(input_tensor)).any().item())
    has_bad_out = bool((~torch.isfinite(output_tensor)).any().item())
    return (not has_bad_in) or has_bad_out, {"input_nonfinite": has_bad_in, "output_nonfinite": has_bad_out}
