"""Load the committed golden vectors (no reference checkout needed).

Small payloads are stored inline (base64 of zlib-compressed bytes).  The few
fixtures that are megabytes of seeded random bytes are stored as recipes and
rebuilt here; make_golden.py checks every rebuild is byte-identical to the
reference builder's output before writing the file.
"""
import base64
import json
import os
import random
import struct
import zlib

HERE = os.path.dirname(os.path.abspath(__file__))


def unpack(text):
    return zlib.decompress(base64.b64decode(text))


def _stored_blocks(data, final):
    blocks = []
    for index in range(0, len(data), 65535):
        chunk = data[index:index + 65535]
        last = final and index + 65535 >= len(data)
        blocks.append(bytes((int(last),)) + struct.pack("<HH", len(chunk), len(chunk) ^ 0xFFFF)
                      + chunk)
    return b"".join(blocks)


def build_payload(record):
    """Return the payload bytes of one decode record."""
    if "payload" in record:
        payload = unpack(record["payload"])
    else:
        recipe = record["recipe"]
        if recipe["kind"] == "zlib-random":
            data = random.Random(recipe["seed"]).randbytes(recipe["size"])
            compressor = zlib.compressobj(recipe["level"], zlib.DEFLATED, zlib.MAX_WBITS, 8,
                                          zlib.Z_DEFAULT_STRATEGY)
            payload = compressor.compress(data) + compressor.flush()
        elif recipe["kind"] == "stored-prefix":
            prefix = random.Random(recipe["seed"]).randbytes(recipe["size"])
            body = _stored_blocks(prefix, final=False) + unpack(recipe["tail_body"])
            raw = prefix + unpack(recipe["tail_raw"])
            payload = b"\x78\x01" + body + struct.pack(">I", zlib.adler32(raw))
        else:
            raise ValueError(recipe["kind"])
    payload = bytearray(payload)
    for start, stop, data in record.get("edits", []):
        payload[start:stop] = unpack(data)
    return bytes(payload)


def _load(name):
    with open(os.path.join(HERE, name), "rb") as handle:
        return json.loads(zlib.decompress(handle.read()))


def decode_vectors():
    """Records: name, payload (bytes), expected, max_candidates, max_blocks,
    want (reference-asserted status, -1 = any failure), sha256 (successes)."""
    records = _load("decode_vectors.json.zz")
    for record in records:
        record["payload"] = build_payload(record)
    return records


def encode_vectors():
    """Records: name, input (bytes), chunk_bytes, size (or None), sha256."""
    records = _load("encode_vectors.json.zz")
    for record in records:
        record["input"] = unpack(record["input"])
    return records
