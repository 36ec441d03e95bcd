"""Exceptions raised for non-OK statuses of the C ABI.

The classes line up with the reference's C++ exceptions so callers can keep their
handling: std::invalid_argument -> InvalidArgument (a ValueError), std::length_error ->
LengthError, cuvit::CudaError -> CudaError, std::runtime_error from weight loading ->
WeightError.
"""

from __future__ import annotations

from . import _lib


class CuvitError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class InvalidArgument(CuvitError, ValueError):
    pass


class LengthError(CuvitError, ValueError):
    pass


class CudaError(CuvitError):
    pass


class DeviceTimeout(CuvitError):
    pass


class Unsupported(CuvitError):
    pass


class WeightError(CuvitError):
    pass


class OutOfMemory(CuvitError, MemoryError):
    pass


_BY_STATUS = {
    _lib.INVALID_ARGUMENT: InvalidArgument,
    _lib.LENGTH_ERROR: LengthError,
    _lib.CUDA_ERROR: CudaError,
    _lib.DEVICE_TIMEOUT: DeviceTimeout,
    _lib.UNSUPPORTED: Unsupported,
    _lib.RUNTIME_ERROR: WeightError,
    _lib.OUT_OF_MEMORY: OutOfMemory,
}


def check(status: int) -> None:
    """Raises the exception matching a non-OK status, with the library's detail text."""
    if status == _lib.OK:
        return
    lib = _lib.library()
    name = lib.cuvit_status_string(status).decode()
    detail = _lib.last_error()
    raise _BY_STATUS.get(status, CuvitError)(status, f"{name}: {detail}" if detail else name)
