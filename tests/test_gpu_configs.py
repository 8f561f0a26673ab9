"""GPU parity on the five BASELINE configurations at their stated sizes.

Inputs come from workloads.py (the generators bench.py times).  Decoded bytes
are compared with the source bytes, which are what the host's zlib and the
oracle decode these valid streams to; encoded streams are compared byte for
byte with the oracle's restatement of the reference encoder (oracle/), and
decoded again on the GPU.  Integer/byte work: every comparison is exact.

Configs 3 (1 GiB, and chunk_bytes=262144) and 4b (compressed random and
period streams above 2**28 bytes) exceed the reference's single-call bounds;
they run through this codec's documented larger single-stream bounds.
"""
import zlib

import numpy as np
import pytest

import workloads
from oracle import oracle

pytestmark = pytest.mark.gpu

MIB = 1 << 20


@pytest.fixture(scope="module")
def codec():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cuda_zlib
    cuda_zlib.compile_kernels(0)
    return cuda_zlib


def _device(array):
    import torch
    return torch.from_numpy(np.ascontiguousarray(array)).to("cuda:0")


def _decode_equal(codec, payload, raw):
    """Single-stream decode on the GPU; compares on the device (exact)."""
    import torch
    out, meta = codec.decompress_zlib_checked(payload, int(raw.size), 0)
    assert [int(v) for v in meta.cpu()] == [0, 0]
    assert torch.equal(out, _device(raw))


def _encode_equal(codec, raw, chunk):
    """One-call compression equals the oracle's stream; returns it."""
    out, meta = codec.compress_zlib_padded(_device(raw), 0, chunk_bytes=chunk)
    length, status = (int(v) for v in meta.cpu())
    assert status == 0
    stream = out[:length].cpu().numpy().tobytes()
    assert stream == oracle.compress_parallel(raw, chunk)
    return stream


# ---------------------------------------------------------------- config 0
@pytest.fixture(scope="module")
def text():
    return np.frombuffer(workloads.zipf_text(16 * MIB, 0), dtype=np.uint8)


def test_config0_text_level6_decode(codec, text):
    payload = workloads.zlib_stream(text.tobytes(), 6)
    host = codec.decompress_zlib_host(payload, text.size, 0)
    assert np.array_equal(host, text)
    assert codec.decompress_zlib(payload, text.size, 0).cpu().numpy().tobytes() == \
        zlib.decompress(payload)


def test_config0_text_compress_chunk32768(codec, text):
    stream = _encode_equal(codec, text, 32768)
    assert zlib.decompress(stream) == text.tobytes()
    _decode_equal(codec, stream, text)


# ---------------------------------------------------------------- config 1
@pytest.fixture(scope="module")
def samples():
    return np.frombuffer(workloads.config1_float32(), dtype=np.uint8)


@pytest.mark.parametrize("level", [1, 6])
def test_config1_float32_decode_to_pinned_host(codec, samples, level):
    import torch
    payload = workloads.zlib_stream(samples.tobytes(), level)
    host = codec.decompress_zlib_host(payload, samples.size, 0)
    assert not host.flags.writeable and torch.from_numpy(host.copy()).numel() == host.size
    assert np.array_equal(host.view("<f4"), samples.view("<f4"))


def test_config1_checksum_mismatch_reports_21_without_replay(codec, samples):
    """A 64 MiB stream whose only fault is its Adler-32: status 21 (the
    reference route's status once chain and history pass) and a zeroed
    output, reported by the block-parallel path without a serial replay of
    the stream (which takes seconds at this size)."""
    import time
    import torch
    payload = bytearray(workloads.zlib_stream(samples.tobytes(), 6))
    payload[-1] ^= 0x40
    dev = torch.device("cuda", 0)
    z = _device(np.frombuffer(bytes(payload), dtype=np.uint8))
    codec.decompress_zlib_checked(z, int(samples.size), dev)  # warm the workspace
    torch.cuda.synchronize()
    begin = time.perf_counter()
    out, meta = codec.decompress_zlib_checked(z, int(samples.size), dev)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - begin
    assert [int(v) for v in meta.cpu()] == [21, 0]
    assert not out.any()
    assert elapsed < 0.5, elapsed
    with pytest.raises(codec.CodecError, match="status 21"):
        codec.decompress_zlib_host(bytes(payload), int(samples.size), 0)


def test_config1_float32_compress_matches_oracle(codec, samples):
    stream = _encode_equal(codec, samples, 32768)
    _decode_equal(codec, stream, samples)


# ---------------------------------------------------------------- config 2
@pytest.fixture(scope="module")
def files():
    return workloads.config2_files()


def test_config2_batch_decode_zlib_level6(codec, files):
    streams = workloads.parallel_map(lambda f: workloads.zlib_stream(f, 6), files)
    outs = codec.decompress_zlib_batch_host(streams, [len(f) for f in files], 0)
    assert all(o.tobytes() == f for o, f in zip(outs, files))
    # Per-file statuses through the device-metadata call: the oracle's (0).
    out, meta = codec.decompress_zlib_batch_checked(
        b"".join(streams), [len(s) for s in streams], [len(f) for f in files], 0)
    statuses = meta.cpu().numpy()[:, 0].tolist()
    assert statuses == [oracle.inflate_serial(s, len(f))[1] for s, f in zip(streams, files)]


def test_config2_batch_compress_and_decode_codec_streams(codec, files):
    streams = codec.compress_zlib_batch_host(files, 0, chunk_bytes=32768)
    expected = workloads.parallel_map(lambda f: oracle.compress(f, 32768), files)
    assert list(streams) == expected
    outs = codec.decompress_zlib_batch_host(list(streams), [len(f) for f in files], 0)
    assert all(o.tobytes() == f for o, f in zip(outs, files))


# ---------------------------------------------------------------- config 3
@pytest.fixture(scope="module")
def records():
    return workloads.config3_records()


@pytest.fixture(scope="module")
def record_streams(records):
    raw = records.tobytes()
    jobs = {"l9": lambda: workloads.zlib_stream(raw, 9),
            "fixed": lambda: workloads.zlib_stream(raw, 1, zlib.Z_FIXED)}
    keys = list(jobs)
    return dict(zip(keys, workloads.parallel_map(lambda k: jobs[k](), keys, 2)))


@pytest.mark.parametrize("kind", ["l9", "fixed"])
def test_config3_records_decode(codec, records, record_streams, kind):
    payload = record_streams[kind]
    assert len(payload) > 2**28 // 4  # a 1 GiB stream: beyond the reference's bound
    _decode_equal(codec, payload, records)


@pytest.mark.parametrize("chunk", [32768, 262144])
def test_config3_records_compress(codec, records, chunk):
    stream = _encode_equal(codec, records, chunk)
    _decode_equal(codec, stream, records)
    # The same stream from chunk ranges spliced on the host (the sharded path,
    # here with one device taking several ranges).
    from cuda_zlib import sharding
    import cuda_zlib._codec as _codec
    saved = _codec._MAX_STREAM
    try:
        _codec._MAX_STREAM = 300 * MIB  # force several ranges
        spliced = sharding.compress_zlib_host_sharded(records, [0], chunk_bytes=chunk)
    finally:
        _codec._MAX_STREAM = saved
    assert spliced.tobytes() == stream


# ---------------------------------------------------------------- config 4a
@pytest.fixture(scope="module")
def batch4a():
    packed, kinds = workloads.config4a_files()
    streams = workloads.zlib_files(packed, 65536, 6)
    return packed, kinds, streams


def test_config4a_batch_checked_decode(codec, batch4a):
    import torch
    packed, _, streams = batch4a
    count = len(streams)
    per_call = (1 << 28) // 65536  # outputs of one call stay within 2**28 bytes
    for first in range(0, count, per_call):
        group = streams[first:first + per_call]
        out, meta = codec.decompress_zlib_batch_checked(
            b"".join(group), [len(s) for s in group], [65536] * len(group), 0)
        assert not meta.cpu().numpy().any()
        assert torch.equal(out, _device(packed[first * 65536:(first + len(group)) * 65536]))


def test_config4a_batch_padded_compress(codec, batch4a):
    packed, _, _ = batch4a
    count = packed.size // 65536
    capacity = 65536 + 5 * 2 + 6
    per_call = (1 << 28) // capacity  # slots of one call stay within 2**28 bytes
    expected = workloads.parallel_map(
        lambda k: oracle.compress(packed[k * 65536:(k + 1) * 65536], 32768), range(count))
    for first in range(0, count, per_call):
        n = min(per_call, count - first)
        slots, meta = codec.compress_zlib_batch_padded(
            _device(packed[first * 65536:(first + n) * 65536]), [65536] * n, 0,
            chunk_bytes=32768)
        meta = meta.cpu().numpy()
        assert not meta[:, 1].any()
        host = slots.cpu().numpy()
        for k in range(n):
            length = int(meta[k, 0])
            assert host[k * capacity:k * capacity + length].tobytes() == expected[first + k]


# ---------------------------------------------------------------- config 4b
@pytest.fixture(scope="module")
def streams4b():
    return workloads.config4b_streams()


@pytest.mark.parametrize("name", ["zeros", "random", "period"])
def test_config4b_decode_zlib_level6(codec, streams4b, name):
    raw = streams4b[name]
    payload = workloads.zlib_stream(raw.tobytes(), 6)
    if name != "zeros":
        assert len(payload) > 2**28  # beyond the reference's decode bound
    _decode_equal(codec, payload, raw)


@pytest.mark.parametrize("name", ["zeros", "random", "period"])
def test_config4b_compress_chunk65535(codec, streams4b, name):
    raw = streams4b[name]
    stream = _encode_equal(codec, raw, 65535)
    _decode_equal(codec, stream, raw)
    if name == "period":
        # The data is random with period 32768, so a ratio near one half can
        # only come from matches at distance 32768 (maximal-distance
        # matches; CPU zlib never emits them and stores this input).
        assert len(stream) < 0.6 * raw.size
