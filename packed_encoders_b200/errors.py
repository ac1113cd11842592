"""Exceptions, mirroring packed_encoders/errors.py:11-20 (same class names, same meaning):
a refusal is an exception, never a silent downgrade to another kernel."""

from __future__ import annotations

try:  # inside a process that already imported the reference, share its hierarchy
    from packed_encoders.errors import PackedEncodersError, UnsupportedTargetError, ValidationError
except ImportError:  # standalone
    class PackedEncodersError(Exception):
        """Base class for every error this package raises."""

    class UnsupportedTargetError(PackedEncodersError):
        """The inputs are outside what the B200 kernels implement."""

    class ValidationError(PackedEncodersError):
        """A parity / validation gate failed."""

__all__ = ["PackedEncodersError", "UnsupportedTargetError", "ValidationError"]
