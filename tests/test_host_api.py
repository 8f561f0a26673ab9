"""Host-side checks that need no GPU.

* The C-ABI library loads and exports every function include/cuda_zlib_b200.h
  declares (no compute call is made).
* The Python API rejects invalid arguments and bad zlib wrappers on the host,
  before it loads the native library or touches a device, as the reference's
  tests require (tests/test_batch.py:15-32, tests/test_host.py:50-67,
  tests/test_decode.py:460-496 of the reference).
"""
import ctypes
import os
import re
import struct
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cuda_zlib_b200.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"#.*", "", text)
    return sorted(set(re.findall(r"\b([A-Za-z_]\w*)\s*\([^;{]*\)\s*;", text)))


def test_header_declares_the_drop_in_entry_points():
    names = _declared_functions()
    for name in ("cuda_zlib_compress", "cuda_zlib_decompress", "cuda_zlib_compress_batch",
                 "cuda_zlib_decompress_batch", "cuda_zlib_compress_noalloc",
                 "CudaZlibSetWorkspaceRetention", "CudaZlibWorkspacePoolStats",
                 "CudaZlibTrimWorkspacePool"):
        assert name in names


def test_library_loads_and_exports_every_declared_symbol():
    from cuda_zlib import _native
    assert os.path.exists(_native.LIBRARY), "build it with cuda-zlib_b200/build.py"
    handle = ctypes.CDLL(_native.LIBRARY)
    missing = [name for name in _declared_functions() if not hasattr(handle, name)]
    assert not missing
    exported = subprocess.run(["nm", "-D", "--defined-only", _native.LIBRARY],
                              capture_output=True, text=True, check=True).stdout
    for name in _declared_functions():
        assert re.search(r" T %s$" % re.escape(name), exported, re.M), name
    handle.cuda_zlib_b200_version.restype = ctypes.c_char_p
    assert re.fullmatch(rb"\d+\.\d+\.\d+", handle.cuda_zlib_b200_version())


@pytest.fixture
def no_backend(monkeypatch):
    """Fail the test if a call reaches the native library or a device."""
    from cuda_zlib import _codec, _native

    def forbidden(*_args, **_kwargs):
        pytest.fail("invalid input reached the native backend")

    monkeypatch.setattr(_native, "library", forbidden)
    monkeypatch.setattr(_codec, "_select_device", forbidden)
    import cuda_zlib
    return cuda_zlib


@pytest.mark.parametrize("sizes", [(), (-1,), (True,), (1.0,), (2**28 + 1,), (2**28, 1), 1, "1"])
def test_batch_invalid_static_sizes(no_backend, sizes):
    with pytest.raises(ValueError):
        no_backend.compress_zlib_batch_padded(b"", sizes)
    with pytest.raises(ValueError):
        no_backend.decompress_zlib_batch_checked(b"", sizes, (0,))


@pytest.mark.parametrize("sizes, message", [
    ((3, True), "must contain integers"),        # bool after good sizes
    ((np.int64(3),), "must contain integers"),   # NumPy integers are not ints
    ((1, 2, -1), "must contain integers"),
    ((1, 2**28 + 1), "must contain integers"),
    ((2**27, 2**27, 1), "total exceeds 2\\*\\*28"),
    (tuple([1] * 262145), "between 1 and 262144"),
])
def test_batch_static_sizes_messages(no_backend, sizes, message):
    """The size checks run as C-level passes over the whole list; each
    failure keeps the message of its class, wherever the bad size sits."""
    with pytest.raises(ValueError, match=message):
        no_backend.decompress_zlib_batch_checked(b"", list(sizes), list(sizes))


def test_batch_invalid_extents_and_chunks(no_backend):
    codec = no_backend
    with pytest.raises(ValueError, match="packed input"):
        codec.compress_zlib_batch_padded(b"x", (0,))
    with pytest.raises(ValueError, match="matching lengths"):
        codec.decompress_zlib_batch_checked(b"", (0,), (0, 0))
    with pytest.raises(ValueError, match="packed input"):
        codec.decompress_zlib_batch_checked(b"x", (0,), (0,))
    with pytest.raises(ValueError, match="chunk_bytes"):
        codec.compress_zlib_batch_padded(b"", (0,), chunk_bytes=255)
    with pytest.raises(ValueError, match="chunk_bytes"):
        codec.compress_zlib_batch_padded(b"", (0,), chunk_bytes=262145)


# chunk_bytes is a superset of the reference's [256, 65535]: up to 262144.
@pytest.mark.parametrize("chunk", [255, 262145, True, 1.0])
def test_compress_rejects_bad_chunk_bytes(no_backend, chunk):
    with pytest.raises(ValueError, match="chunk_bytes"):
        no_backend.compress_zlib_padded(b"abc", chunk_bytes=chunk)


@pytest.mark.parametrize("data", ["text", 3, [1, 2]])
def test_compress_rejects_non_byte_input(no_backend, data):
    with pytest.raises(TypeError):
        no_backend.compress_zlib_padded(data)


def _header(cmf=0x78, flags=0):
    flg = flags | (31 - (cmf * 256 + flags) % 31) % 31
    return bytes((cmf, flg))


@pytest.mark.parametrize("payload, expected, error", [
    (b"", 0, "CodecError"),
    (b"\x78\x00" + b"\x00" * 8, 0, "CodecError"),
    (b"", -1, ValueError),
    (b"", True, ValueError),
    (b"\x78\x9c" + b"\x00" * 8, 2**31 + 1, ValueError),
])
def test_host_rejects_invalid_input_before_the_backend(no_backend, payload, expected, error):
    if isinstance(error, str):
        error = getattr(no_backend, error)
    for decoder in (no_backend.decompress_zlib_host, no_backend.decompress_zlib,
                    no_backend.decompress_zlib_checked):
        with pytest.raises(error):
            decoder(payload, expected)


@pytest.mark.parametrize("payload", [
    b"", b"x", b"\x78\x9c", b"\x78\x00" + b"\x00" * 8,
    _header(cmf=0x79) + b"\x00" * 8,
    _header(cmf=0x88) + b"\x00" * 8,
    _header(flags=0x20) + b"\x00" * 12,
    b"\x1f\x8b" + b"\x00" * 12,
], ids=["empty", "one-byte", "header-only", "header-check", "method", "window",
        "dictionary", "gzip"])
def test_bad_wrapper_is_rejected_without_cuda(no_backend, payload):
    codec = no_backend
    gzip = payload.startswith(b"\x1f\x8b")
    dictionary = len(payload) >= 2 and payload[1] & 0x20 and payload[0] == 0x78
    expected = codec.UnsupportedStream if (gzip or dictionary) else codec.CodecError
    match = "RFC 1950 zlib" if gzip else ("dictionaries" if dictionary else None)
    with pytest.raises(expected, match=match):
        codec.decompress_zlib(payload, 0, device=0)


def test_status_messages_cover_every_reference_code():
    from cuda_zlib import _codec
    for status in list(range(1, 8)) + list(range(9, 24)):
        assert status in _codec._MESSAGES
    with pytest.raises(_codec.UnsupportedStream):
        _codec._check_value(16, "x")
    with pytest.raises(_codec.CodecError, match="Adler32"):
        _codec._check_value(21, "x")


def test_workspace_retention_environment_is_validated(monkeypatch):
    from cuda_zlib import _native
    for bad in ("-1", "1e3", "x", str(1 << 64), "١"):
        monkeypatch.setenv("CUDA_ZLIB_WORKSPACE_RETENTION_BYTES", bad)
        with pytest.raises(ValueError):
            _native._workspace_retention()
    monkeypatch.setenv("CUDA_ZLIB_WORKSPACE_RETENTION_BYTES", "12345")
    assert _native._workspace_retention() == 12345


def test_golden_payload_framing_matches_host_precheck():
    """Stored-block helper used by the fixtures is valid RFC 1950 framing."""
    import zlib
    from golden_io import _stored_blocks
    data = bytes(range(256)) * 300
    body = _stored_blocks(data, final=True)
    stream = b"\x78\x01" + body + struct.pack(">I", zlib.adler32(data))
    assert zlib.decompress(stream) == data


def test_single_stream_bounds_are_the_documented_superset():
    """One stream holds up to 2**31 uncompressed bytes (the reference stops at
    2**28); chunks above 65535 bytes count one stored block per 65535 bytes in
    the padded capacity, which otherwise keeps the reference's formula."""
    from cuda_zlib import _codec
    assert _codec._MAX_STREAM == 2**31
    assert _codec._MAX_STREAM_PAYLOAD == 2**29 - 2**16
    for size, chunk in [(0, 256), (1, 32768), (100000, 32768), (2**28, 65535)]:
        chunks = max(1, -(-size // chunk))
        assert _codec._capacity(size, chunk) == (size + 5 * chunks + 6, chunks)
    # 2**30 at 262144: 4096 chunks of five stored blocks each.
    assert _codec._capacity(2**30, 262144) == (2**30 + 5 * 4096 * 5 + 6, 4096)
    assert _codec._capacity(262145, 262144) == (262145 + 5 * (5 + 1) + 6, 2)
    with pytest.raises(ValueError, match="2\\*\\*29"):
        _codec._check_framing(b"\x78\x9c" + bytes(2**29), 0)


def test_oracle_capacity_matches_the_api():
    from cuda_zlib import _codec
    from oracle import oracle
    for size in (0, 1, 65535, 65536, 262144, 262145, 10**6, 2**30):
        for chunk in (256, 32768, 65535, 65536, 131072, 262144):
            if size // chunk > 300000:
                continue
            assert oracle.capacity(size, chunk) == _codec._capacity(size, chunk)[0]


def test_host_batch_groups_respect_call_bounds():
    """The pipelined host calls cut a batch into device calls within the
    batch bounds (files/chunks, input and output bytes) and cover it."""
    import numpy as np
    from cuda_zlib import _hostio
    rng = np.random.default_rng(3)
    for n in (1, 2, 7, 5000):
        ins = rng.integers(0, 1 << 22, n)
        outs = rng.integers(0, 1 << 22, n)
        units = rng.integers(1, 9, n)
        limits = (1000, 1 << 28, 1 << 28)
        groups = _hostio.plan_groups(ins, outs, units, limits)
        assert groups[0][0] == 0 and groups[-1][1] == n
        assert all(b > a for a, b in groups)
        assert all(g[1] == h[0] for g, h in zip(groups, groups[1:]))
        for a, b in groups:
            if b - a > 1:
                assert units[a:b].sum() <= limits[0]
                assert ins[a:b].sum() <= limits[1] and outs[a:b].sum() <= limits[2]
    # A large batch of equal files splits into at least four groups.
    groups = _hostio.plan_groups([1000] * 65536, [65536] * 65536, [2] * 65536,
                                 (262144, 1 << 28, 1 << 28))
    assert len(groups) >= 16 and max(b - a for a, b in groups) <= 4096


def test_host_batch_pack_reuses_back_to_back_views():
    import numpy as np
    from cuda_zlib import _hostio
    owner = np.arange(1000, dtype=np.uint8)
    views = [owner[10:20], owner[20:20], owner[20:95], owner[95:96]]
    packed = _hostio.pack(views, None)  # no copy: torch is not needed
    assert packed.base is owner or packed.base is owner.base or np.shares_memory(packed, owner)
    assert np.array_equal(packed, owner[10:96])
