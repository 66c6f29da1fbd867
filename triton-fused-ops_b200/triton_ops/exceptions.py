"""Exception hierarchy of the library.

Same classes, constructor arguments and attributes as the reference
(triton_ops/exceptions.py:6-139), so code that catches them keeps working.
:class:`DeviceError` is also exported from the package root here.
"""

from __future__ import annotations

from typing import Any, List, Optional, Tuple


class TritonKernelError(Exception):
    """Base class of every error raised by this library."""


class ShapeMismatchError(TritonKernelError):
    """Input tensors have incompatible shapes.

    Attributes:
        expected: expected shape (or a description of it)
        actual: shape that was received
        tensor_name: which argument was wrong
    """

    def __init__(
        self,
        message: str,
        expected: Optional[Tuple[Any, ...]] = None,
        actual: Optional[Tuple[Any, ...]] = None,
        tensor_name: Optional[str] = None,
    ):
        super().__init__(message)
        self.expected = expected
        self.actual = actual
        self.tensor_name = tensor_name


class UnsupportedDtypeError(TritonKernelError):
    """An input has a dtype the op does not accept.

    Attributes:
        dtype: the rejected dtype
        supported_dtypes: dtypes the op accepts
        tensor_name: which argument was wrong
    """

    def __init__(
        self,
        message: str,
        dtype: Any = None,
        supported_dtypes: Optional[List[Any]] = None,
        tensor_name: Optional[str] = None,
    ):
        super().__init__(message)
        self.dtype = dtype
        self.supported_dtypes = supported_dtypes
        self.tensor_name = tensor_name


class NumericalOverflowError(TritonKernelError):
    """FP8 quantization could not avoid overflow by shrinking the scale.

    Attributes:
        max_value: largest magnitude in the input
        scale: last scale that was tried
        attempts: number of scale reductions performed
    """

    def __init__(
        self,
        message: str,
        max_value: Optional[float] = None,
        scale: Optional[float] = None,
        attempts: Optional[int] = None,
    ):
        super().__init__(message)
        self.max_value = max_value
        self.scale = scale
        self.attempts = attempts


class TuningFailedError(TritonKernelError):
    """No usable kernel configuration exists for a problem size.

    Attributes:
        problem_size: the problem that could not be configured
        configs_tried: number of configurations examined
        last_error: the last exception seen, if any
    """

    def __init__(
        self,
        message: str,
        problem_size: Optional[Tuple[Any, ...]] = None,
        configs_tried: Optional[int] = None,
        last_error: Optional[Exception] = None,
    ):
        super().__init__(message)
        self.problem_size = problem_size
        self.configs_tried = configs_tried
        self.last_error = last_error


class DeviceError(TritonKernelError):
    """A tensor is not on the CUDA device the op runs on.

    Attributes:
        expected_device: where the tensor had to be
        actual_device: where it was
        tensor_name: which argument was wrong
    """

    def __init__(
        self,
        message: str,
        expected_device: Optional[str] = None,
        actual_device: Optional[str] = None,
        tensor_name: Optional[str] = None,
    ):
        super().__init__(message)
        self.expected_device = expected_device
        self.actual_device = actual_device
        self.tensor_name = tensor_name
