"""Keyword-device convenience wrappers (the reference's cuda_zlib.jax module,
src/cuda_zlib/jax.py:17-34).  Here `device` is a CUDA torch.device."""

from . import _codec
from ._errors import BackendUnavailable


def _admit(device):
    _codec._validate_device(device)
    if type(device) is int:
        raise BackendUnavailable("CUDA torch device required")
    return device


def decompress_zlib(payload, expected_bytes, *, device):
    return _codec.decompress_zlib(payload, expected_bytes, _admit(device))


def compress_zlib(data, *, device, chunk_bytes=32768):
    return _codec.compress_zlib(data, _admit(device), chunk_bytes=chunk_bytes)


def compress_zlib_padded(data, *, device, chunk_bytes=32768):
    return _codec.compress_zlib_padded(data, _admit(device), chunk_bytes=chunk_bytes)


def decompress_zlib_checked(payload, expected_bytes, *, device):
    return _codec.decompress_zlib_checked(payload, expected_bytes, _admit(device))
