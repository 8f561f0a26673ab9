"""gzip (RFC 1952) and raw Deflate (RFC 1951) wrappers on the same body codec.

The reference supports RFC 1950 zlib only and rejects gzip members with
status 16 (src/cuda_zlib/_codec.py:105-111); these calls are this codec's
own.  Each mirrors its zlib counterpart in _codec.py: the same chunked
encoder (so a raw or gzip body is byte-identical to the zlib stream's body
at the same chunk size), the same decode routes and bounds, the same
metadata layouts and errors.

  raw Deflate  the bare body; decoding requires the final block to end in
               the payload's last byte (as the zlib route requires of the
               body) and checks no checksum.
  gzip         one member: header (MTIME 0, XFL 0, OS 255 when encoding;
               FEXTRA, FNAME, FCOMMENT and FHCRC accepted when decoding),
               body, CRC-32 and ISIZE.  CRC-32 is computed on the GPU
               (segmented and combined); status 25 is a CRC-32 mismatch,
               26 an ISIZE mismatch, 24 an invalid header.  Multi-member
               files are not decoded: the member must end at the payload's
               end.

Padded capacities: size + 5 * S + W, with S the stored-block count of the
zlib formula and W = 0 (raw) or 18 (gzip) instead of zlib's 6.  Every
encoder call takes level 1 (the reference's parse) or 2 (hash chains with
lazy evaluation, as compress_zlib_padded's level 2).
"""
import ctypes

import numpy as np

from . import _codec, _native
from ._errors import CodecError

FORMAT_ZLIB, FORMAT_RAW, FORMAT_GZIP = 0, 1, 2
_WRAPPER = {FORMAT_ZLIB: 6, FORMAT_RAW: 0, FORMAT_GZIP: 18}
_GZIP_PROBE = 65536  # header bytes read first from a device-resident member


def _capacity(size, chunk_bytes, fmt):
    capacity, chunks, blocks = _codec._layout(size, chunk_bytes)
    return capacity - 6 + _WRAPPER[fmt], blocks


def gzip_header_size(member):
    """Length of a gzip member's header, from host bytes of the member.

    Raises CodecError when the bytes do not start with a valid, complete
    header (cuda_zlib_gzip_header)."""
    view = np.frombuffer(memoryview(member).cast("B"), dtype=np.uint8)
    size = ctypes.c_uint64(0)
    status = _native.library().cuda_zlib_gzip_header(
        view.ctypes.data if view.size else None, view.size, ctypes.byref(size))
    if status:
        raise CodecError("invalid gzip header (Deflate status %d)" % status)
    return int(size.value)


def _member_header(payload, size):
    if isinstance(payload, (bytes, bytearray, memoryview)):
        return gzip_header_size(payload)
    if isinstance(payload, np.ndarray):
        return gzip_header_size(np.ascontiguousarray(payload))
    # A tensor: read its first bytes, and all of it if the header runs past them.
    head = payload[:min(size, _GZIP_PROBE)].cpu().numpy()
    try:
        return gzip_header_size(head)
    except CodecError:
        if size <= _GZIP_PROBE:
            raise
        return gzip_header_size(payload.cpu().numpy())


def _compress_padded(data, device, chunk_bytes, fmt, level=1):
    _codec._check_level(level)
    _codec._check_chunk(chunk_bytes)
    size = _codec._input_size(data, limit=_codec._MAX_STREAM)
    capacity, blocks = _capacity(size, chunk_bytes, fmt)
    if blocks > _codec._MAX_BLOCKS:
        raise ValueError("chunk count exceeds decoder block limit")
    selected = _codec._select_device(device)
    torch = _codec._torch()
    lib = _native.library()
    raw = _codec._device_input(data, selected)
    with torch.cuda.device(selected):
        output = torch.empty(max(capacity, 1), dtype=torch.uint8, device=selected)[:capacity]
        metadata = torch.empty(2, dtype=torch.uint32, device=selected)
        _native.check(lib.cuda_zlib_compress_format(
            _codec._ptr(raw), size, chunk_bytes, fmt, level, output.data_ptr(), capacity,
            metadata.data_ptr(), _codec._stream(selected)), "CUDA compression")
    return output, metadata


def _decompress_checked(payload, expected_bytes, device, fmt, max_candidates, max_blocks):
    _codec._validate_size(expected_bytes)
    size = _codec._input_size(payload, "compressed payload",
                              _codec._MAX_STREAM_PAYLOAD)
    if size > _codec._MAX_STREAM_PAYLOAD - 6 + _WRAPPER[fmt]:
        raise ValueError("compressed payload exceeds 2**29 - 2**16 bytes of Deflate body")
    header = _member_header(payload, size) if fmt == FORMAT_GZIP else 0
    selected = _codec._select_device(device)
    torch = _codec._torch()
    lib = _native.library()
    raw = _codec._device_input(payload, selected)
    with torch.cuda.device(selected):
        output = torch.empty(expected_bytes, dtype=torch.uint8, device=selected)
        metadata = torch.empty(2, dtype=torch.uint32, device=selected)
        _native.check(lib.cuda_zlib_decompress_format(
            _codec._ptr(raw), size, fmt, header, int(max_candidates), int(max_blocks),
            _codec._ptr(output), expected_bytes, metadata.data_ptr(), _codec._stream(selected)),
            "CUDA decompression")
    return output, metadata


def _finished(output, metadata, operation):
    length, status = (int(v) for v in metadata.cpu().numpy())
    _codec._check_value(status, operation)
    return output[:length]


# ---------------------------------------------------------------- raw Deflate
def compress_deflate_padded(data, device=0, *, chunk_bytes=32768, level=1):
    """Return ``(buffer, [encoded_length, status])``: a raw Deflate stream
    (the zlib stream's body) and zero padding, without a host sync."""
    return _compress_padded(data, device, chunk_bytes, FORMAT_RAW, level)


def compress_deflate(data, device=0, *, chunk_bytes=32768, level=1):
    """Encode to a completed, exact-length raw Deflate CUDA tensor."""
    output, metadata = compress_deflate_padded(data, device, chunk_bytes=chunk_bytes, level=level)
    return _finished(output, metadata, "CUDA compression")


def decompress_deflate_checked(payload, expected_bytes, device=0, *,
                               max_candidates=_codec._MAX_CANDIDATES,
                               max_blocks=_codec._MAX_BLOCKS):
    """Return ``(output, [status, 0])`` for a raw Deflate stream, no host sync."""
    return _decompress_checked(payload, expected_bytes, device, FORMAT_RAW, max_candidates,
                               max_blocks)


def decompress_deflate(payload, expected_bytes, device=0):
    """Decode a raw Deflate stream to a completed CUDA tensor."""
    output, metadata = decompress_deflate_checked(payload, expected_bytes, device)
    _codec._check_value(int(metadata.cpu().numpy()[0]), "CUDA decompression")
    return output


# ---------------------------------------------------------------- gzip
def compress_gzip_padded(data, device=0, *, chunk_bytes=32768, level=1):
    """Return ``(buffer, [encoded_length, status])``: one gzip member and zero
    padding, without a host sync."""
    return _compress_padded(data, device, chunk_bytes, FORMAT_GZIP, level)


def compress_gzip(data, device=0, *, chunk_bytes=32768, level=1):
    """Encode to a completed, exact-length gzip member (CUDA tensor)."""
    output, metadata = compress_gzip_padded(data, device, chunk_bytes=chunk_bytes, level=level)
    return _finished(output, metadata, "CUDA compression")


def compress_gzip_host(data, device=0, *, chunk_bytes=32768, level=1) -> np.ndarray:
    """compress_gzip, then one transfer into pinned host memory."""
    return _codec._to_pinned_host(compress_gzip(data, device, chunk_bytes=chunk_bytes,
                                                level=level))


def decompress_gzip_checked(payload, expected_bytes, device=0, *,
                            max_candidates=_codec._MAX_CANDIDATES,
                            max_blocks=_codec._MAX_BLOCKS):
    """Return ``(output, [status, 0])`` for one gzip member.

    The header is parsed on the host (from the first bytes of a device
    tensor); the body, CRC-32 and ISIZE are checked on the GPU.  A failed
    output is all zero."""
    return _decompress_checked(payload, expected_bytes, device, FORMAT_GZIP, max_candidates,
                               max_blocks)


def decompress_gzip(payload, expected_bytes, device=0):
    """Decode one gzip member to a completed CUDA tensor."""
    output, metadata = decompress_gzip_checked(payload, expected_bytes, device)
    _codec._check_value(int(metadata.cpu().numpy()[0]), "CUDA decompression")
    return output


def decompress_gzip_host(payload, expected_bytes, device=0) -> np.ndarray:
    """decompress_gzip, then one transfer into pinned host memory."""
    return _codec._to_pinned_host(decompress_gzip(payload, expected_bytes, device))
