"""Exceptions raised by the Python layer.

The reference reports misuse with ``assert!`` panics whose messages its tests
match (``#[should_panic(expected = ...)]``); here the same messages arrive as
exceptions carrying the C ABI status, so ``pytest.raises(..., match=...)``
reads like the reference's tests.
"""

from __future__ import annotations

from . import _lib


class CubeAwqError(RuntimeError):
    """A call into libcube_awq.so failed."""

    def __init__(self, message: str, status: int = _lib.CAWQ_ERR_INVALID_ARGUMENT):
        super().__init__(message)
        self.status = status


class ShapeError(CubeAwqError, ValueError):
    """A shape rule of the reference failed (CAWQ_ERR_INVALID_SHAPE)."""


class DTypeError(CubeAwqError, TypeError):
    """Unsupported dtype or packed element size (CAWQ_ERR_DTYPE)."""


class UnsupportedDeviceError(CubeAwqError):
    """No sm_100 device for a GPU entry point (CAWQ_ERR_UNSUPPORTED)."""


class DeviceTimeoutError(CubeAwqError):
    """A bounded device-side wait gave up (CAWQ_ERR_TIMEOUT)."""


_BY_STATUS = {
    _lib.CAWQ_ERR_INVALID_SHAPE: ShapeError,
    _lib.CAWQ_ERR_DTYPE: DTypeError,
    _lib.CAWQ_ERR_UNSUPPORTED: UnsupportedDeviceError,
    _lib.CAWQ_ERR_TIMEOUT: DeviceTimeoutError,
}


def check(status: int) -> None:
    """Raise the exception for a non-zero cawq_status."""
    if status != _lib.CAWQ_OK:
        cls = _BY_STATUS.get(status, CubeAwqError)
        raise cls(_lib.last_error(), status)
