"""GPU parity of the gzip (RFC 1952) and raw Deflate (RFC 1951) wrappers.

Encoding: the raw stream and the gzip member are byte-identical to the
oracle's (the zlib stream's body, and that body between the fixed gzip header
and the stdlib's CRC-32 / ISIZE), and the stdlib decodes them.  Decoding:
streams made by the stdlib's zlib (wbits -15 and 31, levels 0-9, with header
fields) decode to their source on both routes (small: output <= 64 KiB;
general: the block-parallel path); corrupt members report 24/25/26 with an
all-zero output.  Integer/byte work: every comparison is exact.
"""
import gzip
import struct
import zlib

import numpy as np
import pytest

import workloads
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def codec():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cuda_zlib
    cuda_zlib.compile_kernels(0)
    return cuda_zlib


def _data(size, seed=0):
    text = workloads.corpus()
    rng = np.random.default_rng(seed)
    if size <= text.size:
        start = int(rng.integers(0, text.size - size + 1))
        return text[start:start + size].tobytes()
    return np.resize(text, size).tobytes()


def _raw(data, level=6, strategy=zlib.Z_DEFAULT_STRATEGY):
    c = zlib.compressobj(level, zlib.DEFLATED, -15, 8, strategy)
    return c.compress(data) + c.flush()


SIZES = [0, 1, 300, 65536, 70000, 1 << 20, 8 << 20]


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("chunk", [4096, 32768, 262144])
def test_encode_matches_oracle(codec, size, chunk):
    data = _data(size, size)
    raw = codec.compress_deflate(data, 0, chunk_bytes=chunk).cpu().numpy().tobytes()
    assert raw == oracle.raw_deflate(data, chunk)
    assert zlib.decompress(raw, -15) == data
    member = codec.compress_gzip(data, 0, chunk_bytes=chunk).cpu().numpy().tobytes()
    assert member == oracle.gzip_member(data, chunk)
    assert gzip.decompress(member) == data


def test_padded_metadata_and_host_call(codec):
    data = _data(100000, 3)
    out, meta = codec.compress_gzip_padded(data, 0)
    length, status = (int(v) for v in meta.cpu())
    assert status == 0 and out.numel() == oracle.capacity(len(data), 32768) + 12
    assert out[length:].sum().item() == 0
    host = codec.compress_gzip_host(data, 0)
    assert not host.flags.writeable and host.tobytes() == out[:length].cpu().numpy().tobytes()


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("level", [0, 1, 6, 9])
def test_raw_decode_of_stdlib_streams(codec, size, level):
    data = _data(size, size + level)
    out, meta = codec.decompress_deflate_checked(_raw(data, level), len(data), 0)
    assert [int(v) for v in meta.cpu()] == [0, 0]
    assert out.cpu().numpy().tobytes() == data


@pytest.mark.parametrize("size", [300, 70000, 4 << 20])
def test_raw_decode_fixed_huffman(codec, size):
    data = _data(size, 9)
    payload = _raw(data, 1, zlib.Z_FIXED)
    assert codec.decompress_deflate(payload, len(data), 0).cpu().numpy().tobytes() == data


@pytest.mark.parametrize("size", SIZES)
@pytest.mark.parametrize("level", [1, 6, 9])
def test_gzip_decode_of_stdlib_members(codec, size, level):
    data = _data(size, 2 * size + level)
    member = gzip.compress(data, level, mtime=0)
    out, meta = codec.decompress_gzip_checked(member, len(data), 0)
    assert [int(v) for v in meta.cpu()] == [0, 0]
    assert out.cpu().numpy().tobytes() == data


def _header_member(data, flags, extra=b"", name=b"", comment=b""):
    header = bytes([0x1F, 0x8B, 8, flags]) + struct.pack("<I", 1234567) + bytes([2, 3])
    if flags & 4:
        header += struct.pack("<H", len(extra)) + extra
    if flags & 8:
        header += name + b"\0"
    if flags & 16:
        header += comment + b"\0"
    if flags & 2:
        header += struct.pack("<H", zlib.crc32(header) & 0xFFFF)
    return header + _raw(data) + struct.pack("<II", zlib.crc32(data), len(data) & 0xFFFFFFFF)


@pytest.mark.parametrize("flags", [1, 2, 4, 8, 16, 31])
@pytest.mark.parametrize("size", [5000, 200000])
def test_gzip_header_fields_host_and_device_payloads(codec, flags, size):
    import torch
    data = _data(size, flags)
    member = _header_member(data, flags, extra=b"X" * 65535, name=b"name.bin",
                            comment=b"c" * 100)
    assert zlib.decompress(member, 31) == data
    assert codec.decompress_gzip(member, len(data), 0).cpu().numpy().tobytes() == data
    # A device-resident member: the header is read from its first bytes
    # (all of them when FEXTRA runs past the first 64 KiB).
    on_device = torch.from_numpy(np.frombuffer(member, dtype=np.uint8).copy()).to("cuda:0")
    out = codec.decompress_gzip(on_device, len(data), 0)
    assert out.cpu().numpy().tobytes() == data
    assert codec.decompress_gzip_host(member, len(data), 0).tobytes() == data


@pytest.mark.parametrize("size", [20000, 300000])
def test_gzip_trailer_mismatches(codec, size):
    data = _data(size, 5)
    member = bytearray(gzip.compress(data, 6, mtime=0))
    bad_crc = bytearray(member)
    bad_crc[-8] ^= 1
    out, meta = codec.decompress_gzip_checked(bytes(bad_crc), len(data), 0)
    assert [int(v) for v in meta.cpu()] == [25, 0] and not out.any()
    bad_size = bytearray(member)
    bad_size[-1] ^= 0x80
    out, meta = codec.decompress_gzip_checked(bytes(bad_size), len(data), 0)
    assert [int(v) for v in meta.cpu()] == [26, 0] and not out.any()
    with pytest.raises(codec.CodecError, match="status 25"):
        codec.decompress_gzip(bytes(bad_crc), len(data), 0)
    # A member whose trailer is cut off: the body cannot end where it must.
    out, meta = codec.decompress_gzip_checked(bytes(member[:-3]), len(data), 0)
    assert int(meta.cpu()[0]) != 0 and not out.any()


def test_format_bounds_through_the_c_abi(codec):
    import torch
    from cuda_zlib import _native, _codec
    lib = _native.library()
    dev = torch.device("cuda", 0)
    meta = torch.full((2,), 99, dtype=torch.int32, device=dev)
    status = lambda: meta.cpu().numpy().tolist()
    out = torch.ones(16, dtype=torch.uint8, device=dev)
    member = np.frombuffer(gzip.compress(b"abc", mtime=0), np.uint8).copy()
    member = torch.from_numpy(member).to(dev)
    stream = _codec._stream(dev)
    # header_bytes past the member's end: 24, output zeroed.
    assert lib.cuda_zlib_decompress_format(member.data_ptr(), member.numel(), 2, 30, 262144,
                                           262144, out.data_ptr(), 3, meta.data_ptr(),
                                           stream) == 0
    assert status() == [24, 0] and not out[:3].any()
    # A one-byte raw stream cannot be complete: 1.
    out.fill_(1)
    assert lib.cuda_zlib_decompress_format(member.data_ptr(), 1, 1, 0, 262144, 262144,
                                           out.data_ptr(), 3, meta.data_ptr(), stream) == 0
    assert status() == [1, 0] and not out[:3].any()
    # Unknown formats are invalid arguments.
    assert lib.cuda_zlib_decompress_format(member.data_ptr(), member.numel(), 3, 0, 262144,
                                           262144, out.data_ptr(), 3, meta.data_ptr(),
                                           stream) == 1
    assert lib.cuda_zlib_compress_format(member.data_ptr(), 3, 32768, 5, 1, out.data_ptr(), 16,
                                         meta.data_ptr(), stream) == 1
    assert lib.cuda_zlib_compress_format(member.data_ptr(), 3, 32768, 0, 3, out.data_ptr(), 16,
                                         meta.data_ptr(), stream) == 1
    # A capacity that is not the format's: [0, 23].
    assert lib.cuda_zlib_compress_format(member.data_ptr(), 3, 32768, 2, 1, out.data_ptr(), 16,
                                         meta.data_ptr(), stream) == 0
    assert status() == [0, 23]


@pytest.mark.parametrize("size", [30000, 200000])
def test_corrupt_raw_streams_match_oracle_status(codec, size):
    """Raw decode reports what the reference route reports for the same body
    framed as zlib with its true Adler-32, except that a body which decodes
    to the right size with other bytes (21 there) succeeds here: raw Deflate
    has no checksum."""
    data = _data(size, 11)
    body = _raw(data, 6)
    rng = np.random.default_rng(size)
    for trial in range(40):
        bad = bytearray(body)
        for _ in range(1 + trial % 3):
            bad[int(rng.integers(0, len(bad)))] ^= 1 << int(rng.integers(0, 8))
        framed = b"\x78\x9c" + bytes(bad) + zlib.adler32(data).to_bytes(4, "big")
        _, want = oracle.decompress(framed, len(data))
        out, meta = codec.decompress_deflate_checked(bytes(bad), len(data), 0)
        got = int(meta.cpu()[0])
        assert got == (0 if want == 21 else want), (trial, want, got)
        if got:
            assert not out.any()


def test_large_members_combine_many_crc_segments(codec):
    """96 MiB + 12345 bytes: 1537 CRC segments, more than the combining
    CTA's 1024 threads, and a partial front segment."""
    data = np.resize(workloads.corpus(), (96 << 20) + 12345)
    member = codec.compress_gzip(data, 0).cpu().numpy().tobytes()
    assert struct.unpack("<II", member[-8:]) == (zlib.crc32(data), data.size)
    assert member == oracle.gzip_member(data, 32768, crc=zlib.crc32(data))
    out = codec.decompress_gzip(member, data.size, 0)
    import torch
    assert torch.equal(out, torch.from_numpy(data).to("cuda:0"))
