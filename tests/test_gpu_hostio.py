"""GPU checks of the pipelined host-buffer batch calls.

decompress_zlib_batch_checked_host / compress_zlib_batch_padded_host must
return exactly what the device calls return (packed outputs, padded slots,
metadata), whether the batch is one group or many, whether the packed input
is pageable or pinned, and beyond one device call's 2**28-byte totals.  The
per-file host calls built on them return the reference's types and raise for
the first failing file.
"""
import zlib

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def codec():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cuda_zlib
    cuda_zlib.compile_kernels(0)
    return cuda_zlib


def _files(count, seed, size=None):
    rng = np.random.default_rng(seed)
    out = []
    for k in range(count):
        n = size if size is not None else int(rng.integers(0, 70000))
        kind = k % 3
        if kind == 0:
            data = rng.integers(0, 256, n, dtype=np.uint8)
        elif kind == 1:
            data = np.repeat(rng.integers(0, 16, n // 50 + 1, dtype=np.uint8), 50)[:n]
        else:
            data = (np.arange(n) % 251).astype(np.uint8) ^ rng.integers(0, 4, n, dtype=np.uint8)
        out.append(data.tobytes())
    return out


@pytest.mark.parametrize("pinned", [False, True])
def test_checked_host_matches_device_call(codec, monkeypatch, pinned):
    import torch
    from cuda_zlib import _hostio
    monkeypatch.setattr(_hostio, "_GROUP_MIN", 1 << 20)  # many groups
    files = _files(300, 1)
    streams = [zlib.compress(f, 6) for f in files]
    sizes, expected = [len(s) for s in streams], [len(f) for f in files]
    packed = np.frombuffer(b"".join(streams), dtype=np.uint8)
    if pinned:
        packed = torch.from_numpy(packed.copy()).pin_memory().numpy()
    out, meta = codec.decompress_zlib_batch_checked_host(packed, sizes, expected, 0)
    assert not out.flags.writeable and meta.dtype == np.uint32 and meta.shape == (300, 2)
    dev_out, dev_meta = codec.decompress_zlib_batch_checked(b"".join(streams), sizes, expected, 0)
    assert np.array_equal(meta, dev_meta.cpu().numpy())
    assert out.tobytes() == dev_out.cpu().numpy().tobytes() == b"".join(files)


@pytest.mark.parametrize("chunk", [4096, 32768, 262144])
def test_padded_host_matches_device_call(codec, monkeypatch, chunk):
    from cuda_zlib import _hostio
    monkeypatch.setattr(_hostio, "_GROUP_MIN", 1 << 20)
    files = _files(200, 2)
    sizes = [len(f) for f in files]
    slots, meta = codec.compress_zlib_batch_padded_host(b"".join(files), sizes, 0,
                                                        chunk_bytes=chunk)
    dev_slots, dev_meta = codec.compress_zlib_batch_padded(b"".join(files), sizes, 0,
                                                           chunk_bytes=chunk)
    assert np.array_equal(meta, dev_meta.cpu().numpy())
    assert slots.tobytes() == dev_slots.cpu().numpy().tobytes()
    streams = codec.compress_zlib_batch_host(files, 0, chunk_bytes=chunk)
    assert list(streams) == [oracle.compress(f, chunk) for f in files]


def test_host_batches_beyond_one_call(codec):
    """300 MiB of files: more than one device call's 2**28 bytes."""
    files = _files(4800, 3, size=65536)
    streams = codec.compress_zlib_batch_host(files, 0)
    assert sum(len(f) for f in files) > 2**28
    outs = codec.decompress_zlib_batch_host(list(streams), [len(f) for f in files], 0)
    assert all(o.tobytes() == f for o, f in zip(outs, files))
    assert all(zlib.decompress(s) == f for s, f in zip(streams[::97], files[::97]))


def test_host_batch_statuses(codec):
    files = _files(12, 4)
    streams = [zlib.compress(f, 6) for f in files]
    bad = bytearray(streams[5])
    bad[-1] ^= 1  # Adler-32 mismatch
    streams[5] = bytes(bad)
    sizes, expected = [len(s) for s in streams], [len(f) for f in files]
    out, meta = codec.decompress_zlib_batch_checked_host(b"".join(streams), sizes, expected, 0)
    want = [oracle.inflate_serial(s, n)[1] for s, n in zip(streams, expected)]
    assert meta[:, 0].tolist() == want and want[5] == 21
    with pytest.raises(codec.CodecError, match="file 5"):
        codec.decompress_zlib_batch_host(streams, expected, 0)


@pytest.mark.parametrize("chunk", [4096, 32768])
def test_packed_batch_compression(codec, monkeypatch, chunk):
    """compress_zlib_batch_packed: the padded call's streams back to back,
    zeros after; the host variant copies only those bytes, group by group
    (many groups here), and compress_zlib_batch_host builds on it."""
    from cuda_zlib import _hostio
    monkeypatch.setattr(_hostio, "_GROUP_MIN", 1 << 20)
    files = _files(500, 5)
    sizes = [len(f) for f in files]
    joined = b"".join(files)
    padded, pmeta = codec.compress_zlib_batch_padded(joined, sizes, 0, chunk_bytes=chunk)
    packed, meta = codec.compress_zlib_batch_packed(joined, sizes, 0, chunk_bytes=chunk)
    pmeta, meta = pmeta.cpu().numpy(), meta.cpu().numpy()
    assert np.array_equal(meta, pmeta) and not meta[:, 1].any()
    capacities = [oracle.capacity(n, chunk) for n in sizes]
    starts = np.concatenate(([0], np.cumsum(capacities)))
    slots = padded.cpu().numpy()
    want = b"".join(slots[starts[k]:starts[k] + meta[k, 0]].tobytes() for k in range(len(files)))
    host_packed = packed.cpu().numpy()
    total = int(meta[:, 0].sum())
    assert host_packed[:total].tobytes() == want and not host_packed[total:].any()
    streams, hmeta = codec.compress_zlib_batch_packed_host(joined, sizes, 0, chunk_bytes=chunk)
    assert not streams.flags.writeable and np.array_equal(hmeta, meta)
    assert streams.tobytes() == want
    expected = [oracle.compress(f, chunk) for f in files[:50]]
    per_file = codec.compress_zlib_batch_host(files, 0, chunk_bytes=chunk)
    assert list(per_file[:50]) == expected
    assert b"".join(per_file) == want
