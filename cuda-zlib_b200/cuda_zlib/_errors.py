"""Errors distinguish malformed input from unavailable/unsupported backends.

Same taxonomy as the reference (src/cuda_zlib/_errors.py:6-15).
"""


class CodecError(ValueError):
    """Malformed stream, checksum/extent mismatch, or codec workspace limit."""


class BackendUnavailable(NotImplementedError):
    """The requested CUDA device or the native codec library is unavailable."""


class UnsupportedStream(NotImplementedError):
    """Valid wrapper features outside this bounded implementation's subset."""
