"""Exceptions raised for llmc_status codes.

They mirror the exception types the reference throws for the same conditions (the C#
type is named on each), while remaining catchable as the closest Python builtin.
"""

from __future__ import annotations


class LlmcError(RuntimeError):
    """Base class; ``status`` holds the llmc_status code."""

    status = 8

    def __init__(self, message: str, status: int | None = None):
        super().__init__(message)
        if status is not None:
            self.status = status


class ArgumentError(LlmcError, ValueError):
    """ArgumentNullException / ArgumentException (null input, "last dim", "square")."""

    status = 1


class ShapeError(ArgumentError):
    status = 2


class NotSupportedError(LlmcError, NotImplementedError):
    """NotSupportedException (ActOrder, unsupported strategy)."""

    status = 3


class NotPositiveDefiniteError(LlmcError):
    """A Hessian factorised with deferred errors had no Cholesky factor (factoring it again
    synchronously takes HessianInverseSolver's pinv fallback), or the eigensolver inside that
    fallback did not converge."""

    status = 4


class CudaError(LlmcError):
    status = 5


class TimeoutError_(LlmcError):
    status = 7


class InvalidOperationError(LlmcError):
    """InvalidOperationException (no calibration samples, missing NamedModules, ...)."""

    status = 9


class ArgumentOutOfRangeError(ArgumentError):
    """ArgumentOutOfRangeException (numBits outside [2, 16], inFeatures <= 0)."""

    status = 10


_BY_STATUS = {
    1: ArgumentError,
    2: ShapeError,
    3: NotSupportedError,
    4: NotPositiveDefiniteError,
    5: CudaError,
    6: LlmcError,
    7: TimeoutError_,
    8: LlmcError,
    9: InvalidOperationError,
    10: ArgumentOutOfRangeError,
}


def raise_for_status(status: int, message: str) -> None:
    cls = _BY_STATUS.get(int(status), LlmcError)
    raise cls(message, int(status))
