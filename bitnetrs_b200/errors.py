"""BitNetError variants returned across the C ABI.

Mirrors ``bitnet_core::error::BitNetError`` (crates/bitnet-core/src/error.rs:12-60):
each C entry point returns one of the ``BITNET_ERR_*`` codes of
``include/bitnet_cuda.h`` and this module turns it into the matching
exception, carrying the message from ``bitnet_cuda_last_error()``.
"""
from __future__ import annotations

OK = 0
ERR_INVALID_SHAPE = 1
ERR_QUANTIZATION = 2
ERR_BACKEND = 3
ERR_INVALID_CONFIG = 4


class BitNetError(Exception):
    """Base of every error raised by the backend."""

    code = -1


class InvalidShape(BitNetError):
    """BitNetError::InvalidShape { expected, got }; both fields are kept."""

    code = ERR_INVALID_SHAPE

    def __init__(self, message: str = "", expected: str = "", got: str = ""):
        super().__init__(message)
        self.expected = expected
        self.got = got


class QuantizationError(BitNetError):
    """BitNetError::QuantizationError(msg)."""

    code = ERR_QUANTIZATION


class BackendError(BitNetError):
    """BitNetError::BackendError { backend: "CUDA", message }."""

    code = ERR_BACKEND


class InvalidConfig(BitNetError):
    """BitNetError::InvalidConfig(msg)."""

    code = ERR_INVALID_CONFIG


_BY_CODE = {c.code: c for c in (InvalidShape, QuantizationError, BackendError, InvalidConfig)}


def raise_for(code: int, message: str, expected: str = "", got: str = "") -> None:
    """Raise the exception for a non-zero C return code (with the
    InvalidShape fields when the library reported them)."""
    if code == OK:
        return
    if code == ERR_INVALID_SHAPE:
        raise InvalidShape(message, expected, got)
    raise _BY_CODE.get(code, BackendError)(message)
