"""ctypes front end of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this module, and only as the checker.  The product's CUDA path
never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "_build", "libzlib_oracle.so")
MAX_CANDIDATES = 262144
MAX_BLOCKS = 262144

_lib = None


def build():
    """Compile the oracle with gcc (make), if it is missing or stale."""
    source = os.path.join(HERE, "zlib_oracle.c")
    if (not os.path.exists(LIBRARY)
            or os.path.getmtime(LIBRARY) < os.path.getmtime(source)):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIBRARY


def lib():
    global _lib
    if _lib is None:
        build()
        handle = ctypes.CDLL(LIBRARY)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        handle.oracle_adler32.argtypes = [u8p, ctypes.c_uint64]
        handle.oracle_adler32.restype = ctypes.c_uint32
        handle.oracle_inflate_serial.argtypes = [u8p, ctypes.c_uint64, u8p, ctypes.c_uint64,
                                                 ctypes.c_uint32]
        handle.oracle_inflate_serial.restype = ctypes.c_uint32
        handle.oracle_inflate_general.argtypes = [u8p, ctypes.c_uint64, u8p, ctypes.c_uint64,
                                                  ctypes.c_uint32, ctypes.c_uint32]
        handle.oracle_inflate_general.restype = ctypes.c_uint32
        handle.oracle_decompress.argtypes = [u8p, ctypes.c_uint64, u8p, ctypes.c_uint64,
                                             ctypes.c_uint32, ctypes.c_uint32]
        handle.oracle_decompress.restype = ctypes.c_uint32
        handle.oracle_compress.argtypes = [u8p, ctypes.c_uint64, ctypes.c_uint32, u8p,
                                           ctypes.c_uint64, u32p]
        handle.oracle_compress.restype = ctypes.c_uint32
        handle.oracle_compress_chunks.argtypes = [u8p, ctypes.c_uint64, ctypes.c_uint32,
                                                  ctypes.c_uint64, ctypes.c_uint64, u8p,
                                                  ctypes.c_uint32, u32p]
        handle.oracle_compress_chunks.restype = ctypes.c_uint32
        handle.oracle_compress_level.argtypes = [u8p, ctypes.c_uint64, ctypes.c_uint32,
                                                 ctypes.c_uint32, u8p, ctypes.c_uint64, u32p]
        handle.oracle_compress_level.restype = ctypes.c_uint32
        handle.oracle_compress_chunks_level.argtypes = [u8p, ctypes.c_uint64, ctypes.c_uint32,
                                                        ctypes.c_uint32, ctypes.c_uint64,
                                                        ctypes.c_uint64, u8p, ctypes.c_uint32,
                                                        u32p]
        handle.oracle_compress_chunks_level.restype = ctypes.c_uint32
        _lib = handle
    return _lib


def _u8(array):
    return array.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def _view(data):
    array = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data
    return np.ascontiguousarray(array, dtype=np.uint8)


def adler32(data):
    array = _view(data)
    return lib().oracle_adler32(_u8(array), array.size)


def decompress(payload, expected, max_candidates=MAX_CANDIDATES, max_blocks=MAX_BLOCKS):
    """Single-stream decode with the reference's route semantics: (bytes, status)."""
    source = _view(payload)
    out = np.zeros(max(1, expected), dtype=np.uint8)
    status = lib().oracle_decompress(_u8(source), source.size, _u8(out), expected,
                                     max_candidates, max_blocks)
    return out[:expected].tobytes(), int(status)


def inflate_serial(payload, expected, max_blocks=MAX_BLOCKS):
    """Serial-route decode (small streams, every batch file): (bytes, status)."""
    source = _view(payload)
    out = np.zeros(max(1, expected), dtype=np.uint8)
    status = lib().oracle_inflate_serial(_u8(source), source.size, _u8(out), expected,
                                         max_blocks)
    if status:
        out[:] = 0
    return out[:expected].tobytes(), int(status)


def inflate_general(payload, expected, max_candidates=MAX_CANDIDATES, max_blocks=MAX_BLOCKS):
    source = _view(payload)
    out = np.zeros(max(1, expected), dtype=np.uint8)
    status = lib().oracle_inflate_general(_u8(source), source.size, _u8(out), expected,
                                          max_candidates, max_blocks)
    return out[:expected].tobytes(), int(status)


def stored_blocks(size):
    """Stored blocks of a chunk's stored fallback (several above 65535 bytes)."""
    return max(1, -(-size // 65535))


def capacity(size, chunk_bytes=32768):
    """Padded output size: size + 5 * (stored blocks of every chunk) + 6,
    which is size + 5 * chunks + 6 for chunks of at most 65535 bytes."""
    chunks = max(1, (size + chunk_bytes - 1) // chunk_bytes)
    last = size - (chunks - 1) * chunk_bytes
    return size + 5 * ((chunks - 1) * stored_blocks(chunk_bytes) + stored_blocks(last)) + 6


def slot_bytes(chunk_bytes):
    """Per-chunk slot of oracle_compress_chunks (room for any chunk encoding)."""
    return (chunk_bytes * 9 + 7) // 8 + 16 + 5 * stored_blocks(chunk_bytes)


def compress_padded(data, chunk_bytes=32768, level=1):
    """Reference encoder restated: (padded buffer, [encoded_length, status]).
    level 2 is the codec's opt-in parse (hash chains, lazy evaluation),
    which the reference does not have."""
    source = _view(data)
    cap = capacity(source.size, chunk_bytes)
    out = np.zeros(cap, dtype=np.uint8)
    meta = np.zeros(2, dtype=np.uint32)
    lib().oracle_compress_level(_u8(source), source.size, chunk_bytes, level, _u8(out), cap,
                                meta.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return out, meta


def compress(data, chunk_bytes=32768, level=1):
    out, meta = compress_padded(data, chunk_bytes, level)
    if meta[1]:
        raise ValueError("oracle compression status %d" % meta[1])
    return out[:meta[0]].tobytes()


def compress_parallel(data, chunk_bytes=32768, threads=None, level=1):
    """compress() for large inputs: the chunks are independent, so several
    host threads encode disjoint chunk ranges (ctypes drops the GIL), then
    the stream is assembled as compress() writes it: 78 01, every chunk's
    encoding in order, the big-endian Adler-32."""
    from concurrent.futures import ThreadPoolExecutor
    source = _view(data)
    n = source.size
    chunks = max(1, -(-n // chunk_bytes))
    slot = slot_bytes(chunk_bytes)
    per = 64

    def encode(first):
        count = min(per, chunks - first)
        out = np.zeros(count * slot, dtype=np.uint8)
        sizes = np.zeros(count, dtype=np.uint32)
        failed = lib().oracle_compress_chunks_level(
            _u8(source), n, chunk_bytes, level, first, count, _u8(out), slot,
            sizes.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
        if failed:
            raise ValueError("oracle chunk compression failed")
        return b"".join(out[k * slot:k * slot + int(sizes[k])].tobytes() for k in range(count))

    with ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1) as pool:
        bodies = list(pool.map(encode, range(0, chunks, per)))
    return b"\x78\x01" + b"".join(bodies) + adler32(source).to_bytes(4, "big")


# ---------------------------------------------------------------- gzip / raw
# The reference has no gzip or raw-Deflate path; the checker for this codec's
# wrappers is the stdlib zlib (the RFC 1950-1952 reference implementation)
# plus the restatements below.
GZIP_HEADER = bytes([0x1F, 0x8B, 8, 0, 0, 0, 0, 0, 0, 0xFF])
CRC_POLY = 0xEDB88320


def raw_deflate(data, chunk_bytes=32768, level=1):
    """The codec's raw Deflate stream: the zlib stream's body."""
    source = _view(data)
    whole = compress_parallel(source, chunk_bytes, level=level) if source.size > (4 << 20) \
        else compress(source, chunk_bytes, level)
    return whole[2:-4]


def gzip_member(data, chunk_bytes=32768, crc=None, level=1):
    """The codec's gzip member: fixed header, body, CRC-32, ISIZE (LE)."""
    import zlib
    source = _view(data)
    value = zlib.crc32(source) if crc is None else crc
    return (GZIP_HEADER + raw_deflate(source, chunk_bytes, level) + value.to_bytes(4, "little")
            + (source.size & 0xFFFFFFFF).to_bytes(4, "little"))


def _gf2_times_x(v):
    return (v >> 1) ^ (CRC_POLY if v & 1 else 0)


def gf2_mul(a, b):
    """a * b mod P in the reflected representation (bit 31 is x^0)."""
    product = 0
    for k in range(32):
        if a & (0x80000000 >> k):
            product ^= b
        b = _gf2_times_x(b)
    return product


def gf2_shift_bytes(n):
    """x^(8 n) mod P."""
    result, power = 0x80000000, 0x00800000
    while n:
        if n & 1:
            result = gf2_mul(result, power)
        power = gf2_mul(power, power)
        n >>= 1
    return result


def crc32_segmented(data, segment=65536):
    """CRC-32 as the GPU computes it: zero-register CRCs of segments (the
    buffer padded in front to whole segments), combined by shifts, then the
    initial value and final XOR applied as one shift term."""
    import zlib
    source = _view(data)
    n = source.size
    segments = -(-n // segment)
    pad = segments * segment - n
    reg = 0
    for s in range(segments):
        lo, hi = max(0, s * segment - pad), (s + 1) * segment - pad
        # Zero-register CRC of the piece: crc32 with init 0 and no final XOR.
        part = zlib.crc32(source[lo:hi], 0xFFFFFFFF) ^ 0xFFFFFFFF
        reg = gf2_mul(reg, gf2_shift_bytes(segment)) ^ part
    return reg ^ gf2_mul(0xFFFFFFFF, gf2_shift_bytes(n)) ^ 0xFFFFFFFF
