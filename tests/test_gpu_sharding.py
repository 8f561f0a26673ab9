"""GPU checks of the sharded paths: byte-identical to the one-device calls.

With one visible GPU the device list repeats device 0, which still runs every
range and file group as its own call; with more GPUs every device is used.
"""
import random
import zlib

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import cuda_zlib
    from cuda_zlib import sharding
    count = torch.cuda.device_count()
    devices = list(range(count)) if count > 1 else [0, 0, 0]
    return cuda_zlib, sharding, devices


def _data(size, seed):
    rng = random.Random(seed)
    return bytes(rng.choices(range(30), k=size // 2)) + rng.randbytes(size // 4) + \
        b"z" * (size - size // 2 - size // 4)


@pytest.mark.parametrize("size, chunk", [(0, 32768), (1, 256), (100000, 256),
                                         (1 << 20, 32768), (5_000_001, 65535)])
def test_sharded_stream_equals_one_device_stream(env, size, chunk):
    codec, sharding, devices = env
    raw = _data(size, size)
    single = codec.compress_zlib_host(raw, 0, chunk_bytes=chunk).tobytes()
    sharded = sharding.compress_zlib_host_sharded(raw, devices, chunk_bytes=chunk)
    assert isinstance(sharded, np.ndarray) and not sharded.flags.writeable
    assert sharded.tobytes() == single
    if size <= 1 << 20:
        assert single == oracle.compress(raw, chunk)
    assert zlib.decompress(single) == raw


def test_range_entry_bodies_splice(env):
    import torch
    codec, sharding, _ = env
    from cuda_zlib import _native
    lib = _native.library()
    raw = _data(300000, 3)
    chunk = 16384
    cuts = [0, 5 * chunk, 6 * chunk, len(raw)]
    bodies, adlers = [], []
    for k, (a, b) in enumerate(zip(cuts, cuts[1:])):
        part = torch.frombuffer(bytearray(raw[a:b]), dtype=torch.uint8).cuda()
        chunks = max(1, -(-(b - a) // chunk))
        out = torch.empty(b - a + 5 * chunks + 6, dtype=torch.uint8, device="cuda")
        meta = torch.zeros(3, dtype=torch.uint32, device="cuda")
        code = lib.cuda_zlib_compress_range(part.data_ptr(), b - a, chunk, int(k == 2),
                                            out.data_ptr(), out.numel(), meta.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
        assert code == 0
        length, status, adler = (int(v) for v in meta.cpu())
        assert status == 0 and adler == zlib.adler32(raw[a:b])
        bodies.append(out[:length].cpu().numpy().tobytes())
        adlers.append(adler)
    stream = sharding.splice_header() + b"".join(bodies) + sharding.splice_trailer(
        sharding.combine_adlers(adlers, [b - a for a, b in zip(cuts, cuts[1:])]))
    assert stream == oracle.compress(raw, chunk)
    # A range that is not last must hold whole chunks.
    part = torch.zeros(1000, dtype=torch.uint8, device="cuda")
    out = torch.empty(1000 + 5 + 6, dtype=torch.uint8, device="cuda")
    meta = torch.zeros(3, dtype=torch.uint32, device="cuda")
    assert lib.cuda_zlib_compress_range(part.data_ptr(), 1000, 4096, 0, out.data_ptr(),
                                        out.numel(), meta.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream) == 1


def test_sharded_stream_beyond_the_single_call_bound(env):
    codec, sharding, _ = env
    size = (1 << 28) + (3 << 20) + 12345
    raw = np.frombuffer(_data(1 << 20, 9), dtype=np.uint8)
    raw = np.tile(raw, size // raw.size + 1)[:size]
    stream = sharding.compress_zlib_host_sharded(raw, [0], chunk_bytes=32768)
    out = zlib.decompressobj()
    assert out.decompress(stream.tobytes()) == raw.tobytes()
    assert out.eof and not out.unused_data


def test_sharded_batch_decode_and_encode(env):
    codec, sharding, devices = env
    rng = random.Random(12)
    files = [_data(rng.choice([0, 1, 300, 5000, 70000, 262144]), i) for i in range(200)]
    streams = [zlib.compress(f, rng.choice([1, 6, 9])) for f in files]
    views = sharding.decompress_zlib_batch_host_sharded(streams, [len(f) for f in files],
                                                        devices)
    assert tuple(v.tobytes() for v in views) == tuple(files)
    ours = sharding.compress_zlib_batch_host_sharded(files, devices, chunk_bytes=16384)
    assert ours == codec.compress_zlib_batch_host(files, 0, chunk_bytes=16384)
    bad = list(streams)
    bad[17] = bad[17][:-1] + bytes((bad[17][-1] ^ 1,))
    with pytest.raises(codec.CodecError, match="file 17"):
        sharding.decompress_zlib_batch_host_sharded(bad, [len(f) for f in files], devices)
