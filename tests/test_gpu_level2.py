"""GPU parity of the opt-in level-2 encoder (no reference counterpart).

Level 2 changes only the parse: each position's best match is the longest
of its first 32 hash-chain candidates within the window (length-3 matches
farther than 4096 bytes dropped), with one-step lazy evaluation.  Its
streams must equal oracle/zlib_oracle.c's restatement of that parse byte for
byte (chunking, block choice and trees are level 1's), decode with the
stdlib's zlib and with this codec, and come out smaller than level 1 on text.
"""
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


def _kind(name, size, seed):
    rng = np.random.default_rng(seed)
    if name == "text":
        text = workloads.corpus()
        start = int(rng.integers(0, text.size - size + 1))
        return text[start:start + size].tobytes()
    if name == "random":
        return rng.integers(0, 256, size, dtype=np.uint8).tobytes()
    if name == "runs":
        return np.repeat(rng.integers(0, 4, size // 20 + 1, dtype=np.uint8), 20)[:size].tobytes()
    if name == "records":
        return workloads.config3_records(size=max(64, size // 64 * 64), seed=seed).tobytes()[:size]
    return np.frombuffer(workloads.config1_float32(size // 4 + 1, seed), np.uint8)[:size].tobytes()


@pytest.mark.parametrize("kind", ["text", "random", "runs", "records", "float"])
@pytest.mark.parametrize("size", [0, 5, 1000, 40000, 300000])
@pytest.mark.parametrize("chunk", [256, 32768, 65535, 262144])
def test_level2_matches_oracle(codec, kind, size, chunk):
    data = _kind(kind, size, size + chunk)
    stream = codec.compress_zlib(data, 0, chunk_bytes=chunk, level=2).cpu().numpy().tobytes()
    assert stream == oracle.compress(data, chunk, 2)
    assert zlib.decompress(stream) == data


@pytest.mark.parametrize("chunk", [32768, 262144])
def test_level2_config0_text(codec, chunk):
    import torch
    text = workloads.corpus()
    out, meta = codec.compress_zlib_padded(torch.from_numpy(text).to("cuda:0"), 0,
                                           chunk_bytes=chunk, level=2)
    length, status = (int(v) for v in meta.cpu())
    assert status == 0
    stream = out[:length].cpu().numpy().tobytes()
    assert stream == oracle.compress_parallel(text, chunk, level=2)
    assert length < 0.92 * len(oracle.compress_parallel(text, chunk))
    decoded = codec.decompress_zlib(stream, text.size, 0)
    assert torch.equal(decoded, torch.from_numpy(text).to("cuda:0"))


def test_level2_wrappers_and_host_call(codec):
    data = _kind("text", 200000, 1)
    raw = codec.compress_deflate(data, 0, level=2).cpu().numpy().tobytes()
    assert raw == oracle.raw_deflate(data, 32768, level=2)
    member = codec.compress_gzip(data, 0, level=2).cpu().numpy().tobytes()
    assert member == oracle.gzip_member(data, 32768, level=2)
    host = codec.compress_zlib_host(data, 0, level=2)
    assert host.tobytes() == oracle.compress(data, 32768, 2)
