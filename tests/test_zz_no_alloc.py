"""GPU check of cuda_zlib_compress_noalloc, the allocation-free compressor.

Collected last (file name) so it also runs after every other GPU test has
used the pooled entry points in the same process.  Calls go straight to the
C ABI; each stream and metadata pair must equal cuda_zlib_compress's on the
same input, on two calls in a row that reuse the same static scratch.
"""
import ctypes
import random
import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_INPUT = 1 << 20   # CUDA_ZLIB_NOALLOC_MAX_INPUT
MAX_CHUNK = 32768     # CUDA_ZLIB_NOALLOC_MAX_CHUNK
INVALID_VALUE = 1     # cudaErrorInvalidValue


@pytest.fixture(scope="module")
def native():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from cuda_zlib import _native
    lib = _native.library()
    entry = lib.cuda_zlib_compress_noalloc
    entry.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_void_p,
                      ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    entry.restype = ctypes.c_int
    return lib


def _capacity(size, chunk):
    return size + 5 * max(1, -(-size // chunk)) + 6


def _run(entry, raw, chunk, stream):
    """Call one compress entry point; return (code, output bytes, metadata)."""
    import torch
    source = torch.frombuffer(bytearray(raw + b"\x00"), dtype=torch.uint8)[:len(raw)].cuda()
    capacity = _capacity(len(raw), chunk)
    output = torch.full((capacity,), 0xA5, dtype=torch.uint8, device="cuda")
    metadata = torch.from_numpy(np.full(2, 0xDEADBEEF, dtype=np.uint32)).cuda()
    torch.cuda.synchronize()
    code = entry(source.data_ptr() if raw else None, len(raw), chunk, output.data_ptr(), capacity,
                 metadata.data_ptr(), stream.cuda_stream)
    stream.synchronize()
    return code, output.cpu().numpy().tobytes(), [int(v) for v in metadata.cpu().numpy()]


def _inputs():
    rng = random.Random(99)
    words = [bytes(rng.choices(b"etaoinshrdlu", k=rng.randint(2, 9))) for _ in range(300)]
    text = b" ".join(rng.choices(words, k=200000))[:MAX_INPUT]
    mixed = rng.randbytes(200000) + b"\x00" * 100000 + bytes(range(256)) * 400
    return [("text-1MiB", text, 32768), ("mixed", mixed, 16384), ("small", b"abc" * 100, 256),
            ("empty", b"", 4096)]


@pytest.mark.parametrize("chunk_override", [None, 1000])
def test_noalloc_matches_pooled_entry_on_consecutive_calls(native, chunk_override):
    import torch
    stream = torch.cuda.Stream()
    cases = _inputs()
    assert len(cases[0][1]) == MAX_INPUT
    for name, raw, chunk in cases + cases[:2]:  # two full passes over the first two inputs
        chunk = chunk_override or chunk
        code, out, meta = _run(native.cuda_zlib_compress_noalloc, raw, chunk, stream)
        want_code, want_out, want_meta = _run(native.cuda_zlib_compress, raw, chunk, stream)
        assert code == 0 and want_code == 0, name
        assert meta == want_meta, name
        assert meta[1] == 0, name
        assert out == want_out, name
        assert zlib.decompress(out[:meta[0]]) == raw, name


def test_noalloc_rejects_calls_beyond_its_limits(native):
    import torch
    stream = torch.cuda.current_stream()
    big = bytes(MAX_INPUT + 1)
    for raw, chunk in ((big, 32768), (b"x" * 1000, MAX_CHUNK + 1), (b"x" * 1000, 255)):
        code, out, meta = _run(native.cuda_zlib_compress_noalloc, raw, chunk, stream)
        assert code == INVALID_VALUE
        assert meta == [0xDEADBEEF, 0xDEADBEEF]
        assert out == b"\xa5" * len(out)
    # A capacity other than size + 5 * chunks + 6 is rejected the same way.
    source = torch.zeros(100, dtype=torch.uint8, device="cuda")
    output = torch.zeros(200, dtype=torch.uint8, device="cuda")
    metadata = torch.zeros(2, dtype=torch.int32, device="cuda")
    code = native.cuda_zlib_compress_noalloc(source.data_ptr(), 100, 256, output.data_ptr(), 200,
                                             metadata.data_ptr(), stream.cuda_stream)
    assert code == INVALID_VALUE
    # The scratch is intact afterwards: a valid call still matches.
    raw = b"after rejection " * 500
    code, out, meta = _run(native.cuda_zlib_compress_noalloc, raw, 4096, stream)
    want = _run(native.cuda_zlib_compress, raw, 4096, stream)
    assert (code, out, meta) == want


_FRESH_PROCESS = r"""
import ctypes, json, sys
import torch
sys.path.insert(0, sys.argv[1])
from cuda_zlib import _native
lib = _native.library()
entry = lib.cuda_zlib_compress_noalloc
entry.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_void_p,
                  ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
size, chunk = 1 << 20, 32768
capacity = size + 5 * (size // chunk) + 6
source = (torch.arange(size, device="cuda") % 251).to(torch.uint8)
output = torch.zeros(capacity, dtype=torch.uint8, device="cuda")
metadata = torch.zeros(2, dtype=torch.int32, device="cuda")
stream = torch.cuda.current_stream().cuda_stream
def call():
    code = entry(source.data_ptr(), size, chunk, output.data_ptr(), capacity,
                 metadata.data_ptr(), stream)
    torch.cuda.synchronize()
    return code
first = call()                      # first call on the device: set-up
free_before = torch.cuda.mem_get_info()[0]
codes = [call() for _ in range(3)]  # warm calls
free_after = torch.cuda.mem_get_info()[0]
stats = (ctypes.c_uint64 * 4)()
pool_code = lib.CudaZlibWorkspacePoolStats(0, stats)
print(json.dumps({"codes": [first] + codes, "free_before": free_before,
                  "free_after": free_after, "pool_code": pool_code,
                  "stats": list(stats), "meta": metadata.cpu().tolist()}))
"""


def test_noalloc_allocates_nothing_in_a_fresh_process():
    """The property the entry point exists for: in a process that has made no
    other codec call, warm calls leave the device's free memory unchanged and
    create no workspace pool (CudaZlibWorkspacePoolStats reports none)."""
    import json
    import os
    import subprocess
    import sys
    package = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                           "cuda-zlib_b200")
    result = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, package],
                            capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stderr[-2000:]
    report = json.loads(result.stdout.strip().splitlines()[-1])
    assert report["codes"] == [0, 0, 0, 0]
    assert report["meta"][1] == 0 and report["meta"][0] > 0
    assert report["free_after"] == report["free_before"]
    assert report["pool_code"] == 0
    assert report["stats"][1:] == [0, 0, 0]  # reserved, used, pool count
