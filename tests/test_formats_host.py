"""Host-side checks of the gzip / raw Deflate wrappers (no GPU).

* The segmented CRC-32 restatement (oracle.crc32_segmented: the method the
  GPU kernels use, crc32.cu) equals the stdlib's zlib.crc32.
* cuda_zlib_gzip_header, called through the library, accepts exactly the
  headers the stdlib's zlib inflate (wbits 31) accepts, FHCRC included, and
  returns their length.
* The padded capacities and the argument checks that precede any device call.
"""
import struct
import zlib

import numpy as np
import pytest

from oracle import oracle


@pytest.mark.parametrize("size", [0, 1, 15, 16, 255, 4096, 65535, 65536, 65537, 1 << 20])
@pytest.mark.parametrize("segment", [16, 4096, 65536])
def test_segmented_crc32_equals_zlib(size, segment):
    data = np.random.default_rng(size + segment).integers(0, 256, size, dtype=np.uint8)
    assert oracle.crc32_segmented(data, segment) == zlib.crc32(data)


def test_gf2_shift_is_zero_bytes():
    # Shifting a register by n bytes is the same as running n zero bytes.
    for reg in (1, 0xDEADBEEF, 0x80000000):
        for n in (0, 1, 7, 1000):
            register = reg
            for _ in range(n):
                for _ in range(8):
                    register = (register >> 1) ^ (oracle.CRC_POLY if register & 1 else 0)
            assert oracle.gf2_mul(reg, oracle.gf2_shift_bytes(n)) == register


def _member(flags=0, extra=b"", name=b"", comment=b"", body=None, hcrc=None):
    header = bytes([0x1F, 0x8B, 8, flags]) + struct.pack("<I", 0) + bytes([0, 255])
    if flags & 4:
        header += struct.pack("<H", len(extra)) + extra
    if flags & 8:
        header += name + b"\0"
    if flags & 16:
        header += comment + b"\0"
    if flags & 2:
        crc = zlib.crc32(header) & 0xFFFF if hcrc is None else hcrc
        header += struct.pack("<H", crc)
    data = b"gzip header test " * 10
    if body is None:
        c = zlib.compressobj(6, zlib.DEFLATED, -15)
        body = c.compress(data) + c.flush()
    return header, header + body + struct.pack("<II", zlib.crc32(data), len(data)), data


def _stdlib_accepts(member, data):
    try:
        return zlib.decompress(member, 31) == data
    except zlib.error:
        return False


def _header(member):
    from cuda_zlib import formats
    return formats.gzip_header_size(member)


CASES = [
    dict(),
    dict(flags=1),
    dict(flags=4, extra=b"AB\x02\x00xy"),
    dict(flags=8, name=b"file.txt"),
    dict(flags=16, comment=b"a comment"),
    dict(flags=2),
    dict(flags=2 | 4 | 8 | 16, extra=b"Z" * 300, name=b"n", comment=b"c"),
    dict(flags=4, extra=b"E" * 65535),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_valid_headers_match_stdlib(case):
    header, member, data = _member(**CASES[case])
    assert _stdlib_accepts(member, data)
    assert _header(member) == len(header)


@pytest.mark.parametrize("mutate", ["magic", "method", "reserved", "hcrc", "truncated_name",
                                    "truncated_extra", "short"])
def test_invalid_headers_match_stdlib(mutate):
    from cuda_zlib import CodecError
    if mutate == "hcrc":
        _, member, data = _member(flags=2, hcrc=0x1234)
    elif mutate == "truncated_name":
        header, _, data = _member(flags=8, name=b"abc")
        member = header[:12]
    elif mutate == "truncated_extra":
        header, _, data = _member(flags=4, extra=b"x" * 50)
        member = header[:30]
    else:
        header, member, data = _member()
        member = bytearray(member)
        if mutate == "magic":
            member[1] = 0x8C
        elif mutate == "method":
            member[2] = 7
        elif mutate == "reserved":
            member[3] = 0x20
        elif mutate == "short":
            member = member[:9]
        member = bytes(member)
    assert not _stdlib_accepts(member, data)
    with pytest.raises(CodecError, match="status 24"):
        _header(member)


def test_capacities():
    from cuda_zlib import formats
    for size, chunk in ((0, 32768), (1, 256), (100000, 32768), (300000, 262144)):
        zlib_capacity = oracle.capacity(size, chunk)
        assert formats._capacity(size, chunk, formats.FORMAT_RAW)[0] == zlib_capacity - 6
        assert formats._capacity(size, chunk, formats.FORMAT_GZIP)[0] == zlib_capacity + 12


def test_argument_checks_before_device():
    import cuda_zlib
    with pytest.raises(ValueError, match="chunk_bytes"):
        cuda_zlib.compress_gzip_padded(b"abc", 0, chunk_bytes=100)
    with pytest.raises(ValueError, match="chunk_bytes"):
        cuda_zlib.compress_deflate_padded(b"abc", 0, chunk_bytes=262145)
    with pytest.raises(ValueError, match="expected_bytes"):
        cuda_zlib.decompress_gzip_checked(b"\x1f\x8b", -1, 0)
    with pytest.raises(cuda_zlib.CodecError, match="gzip header"):
        cuda_zlib.decompress_gzip_checked(b"\x1f\x8b\x08", 10, 0)


def test_oracle_members_decode_with_stdlib():
    data = bytes(range(256)) * 300
    assert zlib.decompress(oracle.raw_deflate(data, 4096), -15) == data
    assert zlib.decompress(oracle.gzip_member(data, 4096), 31) == data


def test_level_argument_checks():
    import cuda_zlib
    for bad in (0, 3, "2", 2.0):
        with pytest.raises(ValueError, match="level"):
            cuda_zlib.compress_zlib_padded(b"abc", 0, level=bad)
        with pytest.raises(ValueError, match="level"):
            cuda_zlib.compress_gzip_padded(b"abc", 0, level=bad)


@pytest.mark.parametrize("chunk", [256, 32768, 262144])
def test_oracle_level2_streams_decode_and_shrink_text(chunk):
    import workloads
    text = workloads.corpus()[:1 << 20].tobytes()
    one, two = oracle.compress(text, chunk), oracle.compress(text, chunk, 2)
    assert zlib.decompress(two) == text
    assert len(two) < len(one)
