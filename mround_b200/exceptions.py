"""Error types raised deliberately by mround_b200.

The hierarchy is the one MRound's callers already catch (reference
``mround/exceptions.py:24-78``): every deliberate refusal is an
:class:`MRoundError`, malformed schemes are also :class:`ValueError`, and the
export and calibration refusals keep their names.  Two classes are new and
belong to the device boundary: :class:`DeviceError` (a CUDA status returned by
the native library) and :class:`NativeLibraryError` (the library is missing or
does not export what ``include/mround_b200.h`` declares).
"""

from __future__ import annotations

__all__ = [
    "ArchitectureError",
    "CalibrationError",
    "DeviceError",
    "ExportError",
    "MRoundError",
    "MemoryBudgetError",
    "NativeLibraryError",
    "PlatformError",
    "ResumeError",
    "SchemeError",
    "UnsupportedSchemeError",
]


class MRoundError(Exception):
    """Root of every error this package raises on purpose."""


class PlatformError(MRoundError):
    """The host cannot run the requested operation (here: no usable CUDA device)."""


class SchemeError(MRoundError, ValueError):
    """A scheme is malformed, or does not apply to the weight it was given.

    Subclasses :class:`ValueError` as well, so callers validating one field
    with ``except ValueError`` keep working.
    """


class UnsupportedSchemeError(SchemeError):
    """A target format cannot hold the requested scheme without approximation."""


class CalibrationError(MRoundError):
    """Calibration inputs are missing, malformed or inconsistent with the model."""


class ArchitectureError(MRoundError):
    """The model's block structure could not be interpreted."""


class ExportError(MRoundError):
    """A checkpoint could not be written, or its tensors are inconsistent."""


class MemoryBudgetError(MRoundError):
    """A run would need more device memory than it is allowed to use."""


class DeviceError(MRoundError):
    """The native CUDA library reported a failure (a CUDA error or a timeout)."""


class ResumeError(MRoundError):
    """A resume directory belongs to another run, or one of its block files is unreadable."""


class NativeLibraryError(MRoundError):
    """The compiled CUDA library is absent, stale, or missing a declared symbol.

    There is no CPU fallback: the package refuses to run rather than compute
    the hot path anywhere but the sm_100a kernels.
    """
