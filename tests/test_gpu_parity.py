"""GPU parity: the CUDA codec against the CPU oracle and the golden vectors.

Every call goes through the product path: cuda_zlib -> libcuda_zlib_b200.so
(C ABI) -> sm_100a kernels.  The oracle (oracle/zlib_oracle.c, pinned to the
reference's golden vectors by test_oracle_golden.py) is only the checker.
Integer/byte work, so every comparison is bit-exact.
"""
import hashlib
import random
import zlib

import numpy as np
import pytest

from golden_io import decode_vectors, encode_vectors
from oracle import oracle

pytestmark = pytest.mark.gpu

ENCODE = encode_vectors()
DECODE = decode_vectors()


@pytest.fixture(scope="module")
def codec():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cuda_zlib
    cuda_zlib.compile_kernels(0)
    return cuda_zlib


def _bytes(tensor):
    return tensor.cpu().numpy().tobytes()


def _meta(tensor):
    return [int(v) for v in tensor.cpu().numpy().reshape(-1)]


# ---------------------------------------------------------------- encoder
@pytest.mark.parametrize("record", ENCODE, ids=[r["name"] for r in ENCODE])
def test_encoder_reproduces_frozen_reference_streams(codec, record):
    raw, chunk = record["input"], record["chunk_bytes"]
    stream = _bytes(codec.compress_zlib(raw, 0, chunk_bytes=chunk))
    if record["size"] is not None:
        assert len(stream) == record["size"]
    assert hashlib.sha256(stream).hexdigest() == record["sha256"]
    assert zlib.decompress(stream) == raw
    # The batch encoder produces the same stream next to ragged siblings
    # (test_encode_match.py:15-23, test_encode_bounds.py:56-60).
    siblings = (b"", raw, raw[:1], raw[:260])
    streams = codec.compress_zlib_batch_host(siblings, 0, chunk_bytes=chunk)
    assert streams[1] == stream
    assert tuple(zlib.decompress(s) for s in streams) == siblings


def _inputs():
    rng = random.Random(2024)
    cases = []
    for size in (0, 1, 2, 3, 255, 256, 257, 4095, 32767, 32768, 32769, 65535, 65536, 131073):
        cases.append(("random", size, rng.randbytes(size)))
        cases.append(("repeat", size, b"a" * size))
        cases.append(("alphabet", size, (bytes(range(256)) * (size // 256 + 1))[:size]))
        cases.append(("skewed", size, bytes(rng.choices(range(16), weights=range(1, 17), k=size))))
    words = [bytes(rng.choices(b"abcdefghijklmnopqrstuvwxyz", k=rng.randint(3, 10)))
             for _ in range(500)]
    text = b" ".join(rng.choices(words, k=40000))[:200000]
    cases.append(("text", len(text), text))
    return cases


INPUTS = _inputs()


@pytest.mark.parametrize("chunk", [256, 1000, 4096, 32768, 65535])
@pytest.mark.parametrize("case", INPUTS, ids=["%s-%d" % (k, n) for k, n, _ in INPUTS])
def test_encoder_matches_oracle_byte_for_byte(codec, case, chunk):
    _, size, raw = case
    if size > 70000 and chunk < 4096:
        pytest.skip("covered by the larger chunk sizes")
    expected_out, expected_meta = oracle.compress_padded(raw, chunk)
    output, metadata = codec.compress_zlib_padded(raw, 0, chunk_bytes=chunk)
    assert _meta(metadata) == [int(v) for v in expected_meta]
    assert _bytes(output) == expected_out.tobytes()
    assert zlib.decompress(_bytes(output)[:int(expected_meta[0])]) == raw


def test_encoder_device_tensor_input(codec):
    import torch
    raw = bytes(range(251)) * 400
    tensor = torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda()
    assert _bytes(codec.compress_zlib(tensor, 0)) == oracle.compress(raw)


# ---------------------------------------------------------------- decoder
def _native_decompress(payload, expected, max_candidates, max_blocks):
    """Direct C-ABI call with device buffers (no host-side pre-checks)."""
    import torch
    from cuda_zlib import _native
    source = torch.frombuffer(bytearray(payload + b"\x00"), dtype=torch.uint8)[:len(payload)].cuda()
    output = torch.empty(expected, dtype=torch.uint8, device="cuda")
    metadata = torch.empty(2, dtype=torch.uint32, device="cuda")
    code = _native.library().cuda_zlib_decompress(
        source.data_ptr() if len(payload) else None, len(payload), max_candidates, max_blocks,
        output.data_ptr() if expected else None, expected, metadata.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert code == 0
    return output, metadata


@pytest.mark.parametrize("record", DECODE, ids=[r["name"] for r in DECODE])
def test_decoder_matches_oracle_and_reference_statuses(codec, record):
    payload, expected = record["payload"], record["expected"]
    want_out, want_status = oracle.decompress(payload, expected, record["max_candidates"],
                                              record["max_blocks"])
    if record["want"] >= 0:
        assert want_status == record["want"]
    # Device-resident payloads reach the device's own framing checks, as the
    # reference tests' JAX arrays do.
    output, metadata = _native_decompress(payload, expected, record["max_candidates"],
                                          record["max_blocks"])
    assert _meta(metadata) == [want_status, 0]
    assert _bytes(output) == want_out
    if want_status == 0:
        assert hashlib.sha256(want_out).hexdigest() == record["sha256"]


def test_bytes_payloads_are_prechecked_on_the_host(codec):
    with pytest.raises(codec.CodecError, match="truncated"):
        codec.decompress_zlib(b"\x78\x9c", 0, 0)
    with pytest.raises(codec.UnsupportedStream, match="RFC 1950"):
        codec.decompress_zlib(b"\x1f\x8b" + bytes(12), 0, 0)
    with pytest.raises(codec.CodecError, match="CMF/FLG"):
        codec.decompress_zlib(b"\x88\x1c" + bytes(8), 0, 0)
    with pytest.raises(codec.UnsupportedStream, match="dictionaries"):
        codec.decompress_zlib(bytes((0x78, 0x20 | (-(0x78 * 256 + 0x20) % 31))) + bytes(12), 0, 0)


def _zlib(raw, level=6, strategy=zlib.Z_DEFAULT_STRATEGY):
    c = zlib.compressobj(level, zlib.DEFLATED, zlib.MAX_WBITS, 8, strategy)
    return c.compress(raw) + c.flush()


@pytest.mark.parametrize("level", [0, 1, 6, 9])
@pytest.mark.parametrize("strategy", [zlib.Z_DEFAULT_STRATEGY, zlib.Z_FIXED, zlib.Z_HUFFMAN_ONLY])
def test_decoder_matches_stdlib_streams(codec, level, strategy):
    rng = random.Random(level * 10 + strategy)
    for size in (0, 1, 1000, 65536, 70000, 300000):
        raw = bytes(rng.choices(range(40), k=size // 2)) + rng.randbytes(size // 4) + bytes(size - size // 2 - size // 4)
        payload = _zlib(raw, level, strategy)
        output, metadata = codec.decompress_zlib_checked(payload, size, 0)
        assert _meta(metadata) == [0, 0]
        assert _bytes(output) == raw


def test_decompress_host_returns_pinned_read_only_array(codec):
    raw = np.arange(100000, dtype=np.float32).tobytes()
    host = codec.decompress_zlib_host(zlib.compress(raw, 6), len(raw), 0)
    assert isinstance(host, np.ndarray) and not host.flags.writeable
    assert host.tobytes() == raw


# ---------------------------------------------------------------- batch
def test_batch_decode_matches_serial_oracle_per_file(codec):
    rng = random.Random(7)
    payloads, sizes = [], []
    for index in range(64):
        size = rng.choice([0, 1, 100, 5000, 65536, 100000])
        raw = bytes(rng.choices(range(8 + index % 200), k=size))
        payload = _zlib(raw, rng.choice([0, 1, 6, 9]))
        if index % 7 == 3:  # corrupt a few: checksum, body, size
            payload = payload[:-1] + bytes((payload[-1] ^ 1,))
        if index % 11 == 5 and len(payload) > 12:
            payload = payload[:7] + b"\xff" + payload[8:]
        if index % 13 == 4:
            size += 1
        payloads.append(payload)
        sizes.append(size)
    output, metadata = codec.decompress_zlib_batch_checked(
        b"".join(payloads), [len(p) for p in payloads], sizes, 0)
    out = _bytes(output)
    meta = metadata.cpu().numpy()
    offset = 0
    for payload, size, row in zip(payloads, sizes, meta):
        want, status = oracle.inflate_serial(payload, size)
        assert [int(row[0]), int(row[1])] == [status, 0]
        assert out[offset:offset + size] == want
        offset += size


def test_batch_decode_of_compression_slots(codec):
    files = (b"", b"abc" * 1000, bytes(range(256)) * 300, random.Random(3).randbytes(5000))
    sizes = [len(f) for f in files]
    slots, enc_meta = codec.compress_zlib_batch_padded(b"".join(files), sizes, 0)
    caps = [n + 5 * max(1, -(-n // 32768)) + 6 for n in sizes]
    output, meta = codec.decompress_zlib_batch_checked(slots, caps, sizes, 0,
                                                       encoded_metadata=enc_meta)
    assert _meta(meta) == [0, 0] * len(files)
    assert _bytes(output) == b"".join(files)


def test_batch_compress_matches_oracle_per_file(codec):
    rng = random.Random(11)
    files = [rng.randbytes(rng.randint(0, 3000)) + b"z" * rng.randint(0, 70000) for _ in range(40)]
    streams = codec.compress_zlib_batch_host(files, 0, chunk_bytes=16384)
    for raw, stream in zip(files, streams):
        assert stream == oracle.compress(raw, 16384)


def test_exact_length_batch_apis(codec):
    files = [b"hello" * n for n in range(6)]
    streams = codec.compress_zlib_batch(files, 0)
    assert tuple(zlib.decompress(_bytes(s)) for s in streams) == tuple(files)
    decoded = codec.decompress_zlib_batch([_bytes(s) for s in streams], [len(f) for f in files], 0)
    assert tuple(_bytes(d) for d in decoded) == tuple(files)
    views = codec.decompress_zlib_batch_host([_bytes(s) for s in streams], [len(f) for f in files], 0)
    assert tuple(v.tobytes() for v in views) == tuple(files)


def test_failed_call_does_not_poison_the_next(codec):
    raw = b"recovery " * 5000
    payload = zlib.compress(raw)
    bad = payload[:-1] + bytes((payload[-1] ^ 1,))
    with pytest.raises(codec.CodecError, match="Adler32"):
        codec.decompress_zlib(bad, len(raw), 0)
    assert _bytes(codec.decompress_zlib(payload, len(raw), 0)) == raw


def test_workspace_pool_stats_and_trim(codec):
    import torch
    raw = bytes(range(256)) * 4097
    codec.decompress_zlib(zlib.compress(raw), len(raw), 0)
    torch.cuda.synchronize()
    before = codec.workspace_pool_stats(0)
    assert before["pool_count"] >= 1 and before["used_bytes"] == 0
    codec.trim_workspace_pool(0)
    after = codec.workspace_pool_stats(0)
    assert after["retention_bytes"] == before["retention_bytes"]
    assert after["reserved_bytes"] <= before["reserved_bytes"] and after["used_bytes"] == 0


# ---------------------------------------------------------------- host I/O
def test_compress_host_returns_pinned_exact_stream(codec):
    import torch
    raw = bytes(range(256)) * 5000 + random.Random(5).randbytes(70000)
    host = codec.compress_zlib_host(raw, 0, chunk_bytes=16384)
    assert isinstance(host, np.ndarray) and not host.flags.writeable
    assert torch.from_numpy(host.copy()).numel() == host.size
    assert host.tobytes() == oracle.compress(raw, 16384)


def test_pinned_inputs_skip_staging_and_match(codec):
    import torch
    raw = random.Random(6).randbytes(300000) + b"q" * 200000
    payload = zlib.compress(raw, 6)
    pinned = torch.frombuffer(bytearray(payload), dtype=torch.uint8).pin_memory()
    assert codec.decompress_zlib_host(pinned, len(raw), 0).tobytes() == raw
    # A *_host result is page-locked memory and is accepted as input directly.
    stream = codec.compress_zlib_host(raw, 0)
    assert codec.decompress_zlib_host(stream, len(raw), 0).tobytes() == raw


def test_large_bytes_input_uses_threaded_staging(codec):
    rng = random.Random(8)
    raw = bytes(rng.choices(range(12), k=12 << 20))   # above two staging pieces
    payload = zlib.compress(raw, 1)
    assert codec.decompress_zlib_host(payload, len(raw), 0).tobytes() == raw
    assert codec.compress_zlib_host(raw, 0).tobytes() == oracle.compress(raw)


@pytest.mark.parametrize("size, chunk, piece", [
    (200000, 256, 4096),            # many pieces, ragged last chunk and piece
    (3 * 65536, 32768, 65536),      # whole pieces only
    (1000003, 65535, 300000),       # piece rounded down to whole 65535-byte chunks
    (130000, 16384, 1 << 20),       # one piece
])
def test_pipelined_host_compress_matches_one_call(codec, monkeypatch, size, chunk, piece):
    import torch
    from cuda_zlib import _codec
    monkeypatch.setattr(_codec, "_PIPE_MIN", 1)
    monkeypatch.setattr(_codec, "_PIPE_PIECE", piece)
    rng = random.Random(size)
    raw = bytes(rng.choices(range(40), k=size // 2)) + rng.randbytes(size // 4) + \
        b"\0" * (size - size // 2 - size // 4)
    expected = oracle.compress(raw, chunk)
    pinned = torch.frombuffer(bytearray(raw), dtype=torch.uint8).pin_memory()
    # Pageable inputs take the pieces; a pinned tensor takes the one-call path.
    for data in (raw, bytearray(raw), np.frombuffer(raw, dtype=np.uint8),
                 torch.frombuffer(bytearray(raw), dtype=torch.uint8), pinned):
        host = codec.compress_zlib_host(data, 0, chunk_bytes=chunk)
        assert isinstance(host, np.ndarray) and not host.flags.writeable
        assert host.tobytes() == expected
    # A *_host result lives in pinned memory and goes in without staging.
    again = codec.compress_zlib_host(codec.decompress_zlib_host(expected, size, 0), 0,
                                     chunk_bytes=chunk)
    assert again.tobytes() == expected


def test_pipelined_host_compress_at_default_threshold(codec):
    from cuda_zlib import _codec
    rng = np.random.default_rng(11)
    raw = np.cumsum(rng.integers(-2, 3, _codec._PIPE_MIN + 12345)).astype(np.uint8)
    host = codec.compress_zlib_host(raw, 0)
    device, meta = codec.compress_zlib_padded(raw, 0)
    length = int(meta.cpu()[0])
    assert host.tobytes() == device[:length].cpu().numpy().tobytes()
    assert zlib.decompress(host.tobytes()) == raw.tobytes()


# ---------------------------------------------------------------- token arena
def _flushed_stream(raw, every, level=6):
    """A stream cut into many blocks by full flushes (a block + an empty stored block each)."""
    c = zlib.compressobj(level)
    parts = []
    for i in range(0, len(raw), every):
        parts.append(c.compress(raw[i:i + every]))
        parts.append(c.flush(zlib.Z_FULL_FLUSH))
    parts.append(c.flush())
    return b"".join(parts)


def test_token_arena_overflow_falls_back_to_exact_layout(codec, monkeypatch):
    """Many small blocks leave a partial arena page each; with no slack the
    arena runs out and the second decoding pass must give the same bytes."""
    import ctypes
    from cuda_zlib import _native
    lib = _native.library()
    lib.cuda_zlib_b200_profile.argtypes = [ctypes.c_int]
    lib.cuda_zlib_b200_profile_read.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                                                ctypes.POINTER(ctypes.c_uint64)]
    rng = random.Random(21)
    raw = bytes(rng.choices(range(64), k=4 << 20))
    payload = _flushed_stream(raw, 1500)
    times = {}
    for slack in (None, "0"):
        if slack is None:
            monkeypatch.delenv("CUDA_ZLIB_TOKEN_ARENA_SLACK", raising=False)
        else:
            monkeypatch.setenv("CUDA_ZLIB_TOKEN_ARENA_SLACK", slack)
        lib.cuda_zlib_b200_profile(1)
        out, meta = codec.decompress_zlib_checked(payload, len(raw), 0)
        assert _meta(meta) == [0, 0]
        assert _bytes(out) == raw
        total, launches = ctypes.c_double(), ctypes.c_uint64()
        lib.cuda_zlib_b200_profile_read(b"symbols_kernel", ctypes.byref(total),
                                        ctypes.byref(launches))
        lib.cuda_zlib_b200_profile(0)
        assert launches.value == 1
        times[slack] = total.value
    # Without slack the second pass decodes every node; with it, it returns at once.
    assert times["0"] > 5 * times[None]
