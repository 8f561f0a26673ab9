"""The CPU oracle against the reference's golden vectors (no GPU).

The oracle is the checker for every GPU parity test, so it is pinned first:
the 38 SHA-256-frozen encoder streams and every decode status the reference
tests assert for hand-built streams must reproduce exactly.
"""
import hashlib
import zlib

import pytest

from golden_io import decode_vectors, encode_vectors
from oracle import oracle

ENCODE = encode_vectors()
DECODE = decode_vectors()


@pytest.mark.parametrize("record", ENCODE, ids=[r["name"] for r in ENCODE])
def test_oracle_encoder_matches_frozen_reference_streams(record):
    stream = oracle.compress(record["input"], record["chunk_bytes"])
    if record["size"] is not None:
        assert len(stream) == record["size"]
    assert hashlib.sha256(stream).hexdigest() == record["sha256"]
    assert zlib.decompress(stream) == record["input"]


@pytest.mark.parametrize("record", DECODE, ids=[r["name"] for r in DECODE])
def test_oracle_decoder_matches_reference_statuses(record):
    out, status = oracle.decompress(record["payload"], record["expected"],
                                    record["max_candidates"], record["max_blocks"])
    if record["want"] >= 0:
        assert status == record["want"]
    else:
        assert status != 0
    if status == 0:
        assert hashlib.sha256(out).hexdigest() == record["sha256"]
        assert out == zlib.decompress(record["payload"])
    else:
        assert out == bytes(record["expected"])


def test_oracle_adler32_matches_stdlib():
    for data in (b"", b"a", bytes(range(256)) * 300, b"\xff" * 70000):
        assert oracle.adler32(data) == zlib.adler32(data)


@pytest.mark.parametrize("size", [0, 1, 255, 256, 257, 32767, 32768, 32769, 65535, 65536, 131073])
@pytest.mark.parametrize("kind", ["random", "repeat", "alphabet"])
def test_oracle_encoder_roundtrips_through_stdlib(size, kind):
    import random
    if kind == "random":
        raw = random.Random(size + 19).randbytes(size)
    elif kind == "repeat":
        raw = b"a" * size
    else:
        raw = (bytes(range(256)) * ((size + 255) // 256))[:size]
    stream = oracle.compress(raw)
    assert zlib.decompress(stream) == raw
    assert len(stream) <= size + 5 * max(1, (size + 32767) // 32768) + 6


def test_serial_route_matches_stdlib_on_block_types():
    import random
    raw = bytes(random.Random(5).choices(range(16), k=40000))
    for level, strategy in ((0, zlib.Z_DEFAULT_STRATEGY), (6, zlib.Z_FIXED), (9, zlib.Z_DEFAULT_STRATEGY)):
        c = zlib.compressobj(level, zlib.DEFLATED, 15, 8, strategy)
        payload = c.compress(raw) + c.flush()
        out, status = oracle.inflate_serial(payload, len(raw))
        assert status == 0 and out == raw
        out, status = oracle.inflate_general(payload, len(raw))
        assert status == 0 and out == raw
