"""Regenerate the golden vectors in this directory from the reference tests.

Run in a container that has the reference checkout (its path is the first
argument, or $CUDA_ZLIB_REFERENCE).  The GPU box never runs this script: it
reads only the committed outputs.

Decode vectors
    Payloads come from the reference's own independent bit-level fixture
    builders (tests/test_decode.py:46-455, tests/test_regressions.py:24-313),
    called unchanged, plus stdlib-zlib streams built the way the reference
    tests build them.  Each record keeps the status the reference test
    asserts (`want`, or -1 where the test only asserts some failure), the
    route parameters (expected size, max_candidates, max_blocks) and, for
    successes, the SHA-256 of stdlib zlib's output.

Encode vectors
    The 38 SHA-256 pins of the reference encoder's frozen streams
    (tests/test_encode.py:52-70, tests/test_encode_match.py:26-57,
    tests/test_encode_bounds.py:16-35) with their inputs.

Output files: decode_vectors.json.zz and encode_vectors.json.zz (zlib-
compressed JSON; payloads base64).
"""
import base64
import hashlib
import json
import os
import random
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
MIB = 1 << 20
DEFAULT = (262144, 262144)


def _b64(data):
    return base64.b64encode(zlib.compress(bytes(data), 9)).decode("ascii")


from golden_io import build_payload  # noqa: E402


def _load_reference(root):
    sys.path.insert(0, os.path.join(root, "src"))
    sys.path.insert(0, os.path.join(root, "tests"))
    import test_decode as td  # noqa: E402
    import test_regressions as tr  # noqa: E402
    import test_encode as te  # noqa: E402
    import test_encode_match as tm  # noqa: E402
    import test_encode_bounds as tb  # noqa: E402
    return td, tr, te, tm, tb


def _params(function, name):
    for mark in getattr(function, "pytestmark", []):
        if mark.name == "parametrize" and mark.args[0] == name:
            return list(mark.args[1])
    raise KeyError(name)


def decode_vectors(td, tr):
    records = []

    def add(name, payload, expected, want, source, limits=DEFAULT, raw=None,
            recipe=None, edits=None):
        record = {"name": name, "expected": expected,
                  "max_candidates": limits[0], "max_blocks": limits[1],
                  "want": want, "source": source}
        if recipe is None:
            record["payload"] = _b64(payload)
        else:
            # Seeded recipe (megabytes of random bytes); the loader rebuilds
            # it and the generator checks the rebuild is byte-identical.
            record["recipe"] = recipe
            record["edits"] = edits or []
            assert build_payload(record) == payload, name
        if want == 0:
            assert raw is not None and len(raw) == expected
            record["sha256"] = hashlib.sha256(raw).hexdigest()
        records.append(record)

    # tests/test_decode.py:406-419, 591-597 (tree shapes, all valid)
    for kind in ["literal-only-empty-distance", "single-eob", "single-distance"]:
        payload, raw = td._dynamic_tree_stream(kind)
        add("dynamic-tree-" + kind, payload, len(raw), 0, "test_decode.py:588-597", raw=raw)
    # tests/test_decode.py:687-693 (malformed repeats; expected bytes 0)
    for kind in ["repeat-before-length", "repeat-overflow"]:
        add("invalid-repeat-" + kind, td._invalid_repeat_stream(kind), 0, -1,
            "test_decode.py:687-693")
    add("padded-final", td._padded_final_stream(), 1, 0, "test_decode.py:696-701", raw=b"A")
    payload, small_window, raw = td._distance_window_stream()
    add("distance-window", payload, len(raw), 0, "test_decode.py:704-712", raw=raw)
    add("distance-window-cinfo0", small_window, len(raw), -1, "test_decode.py:710-712")
    tail_payload, _, tail_raw = td._distance_window_stream()
    for prefix_bytes in (65537, 1048577):
        payload, small_window, raw = td._prefixed_distance_window_stream(prefix_bytes)
        recipe = {"kind": "stored-prefix", "seed": prefix_bytes, "size": prefix_bytes,
                  "tail_body": _b64(tail_payload[2:-4]), "tail_raw": _b64(tail_raw)}
        add("prefixed-window-%d" % prefix_bytes, payload, len(raw), 0,
            "test_decode.py:818-850", raw=raw, recipe=recipe)
        add("prefixed-window-%d-cinfo0" % prefix_bytes, small_window, len(raw), 6,
            "test_decode.py:843", recipe=recipe,
            edits=[[0, 2, _b64(td._header(cmf=0x08))]])
        # Damaged bodies: byte 2 becomes 0x07 and the Adler trailer flips.
        damage = [[-1, None, _b64(bytes((payload[-1] ^ 1,)))], [2, 3, _b64(b"\x07")]]
        for label, head, status in (
                ("cmf88", td._header(cmf=0x88), 15),
                ("flg", payload[:1] + bytes((payload[1] ^ 1,)), 15),
                ("gzip", b"\x1f\x8b", 16),
                ("fdict", td._header(flags=0x20), 17)):
            bad = head + b"\x07" + payload[3:-1] + bytes((payload[-1] ^ 1,))
            add("prefixed-window-%d-%s" % (prefix_bytes, label), bad, len(raw), status,
                "test_decode.py:838-842", recipe=recipe,
                edits=damage + [[0, 2, _b64(head)]])
    payload, raw = td._medium_period_stream()
    add("medium-period", payload, len(raw), 0, "test_decode.py:962-973", raw=raw)
    add("medium-period-cinfo0", td._header(cmf=0x08) + payload[2:], len(raw), 6,
        "test_decode.py:959-971")
    payload, raw = td._medium_compound_stream()
    add("medium-compound", payload, len(raw), 0, "test_decode.py:911-948", raw=raw)
    hist, _ = td._medium_compound_stream(history_error=True, reserved=True)
    add("medium-compound-history-reserved", hist, len(raw), 4, "test_decode.py:924")
    wres, wraw = td._medium_compound_stream(window_error=True, reserved=True)
    add("medium-compound-window-reserved", wres, len(wraw), 4, "test_decode.py:925")
    win, wraw2 = td._medium_compound_stream(window_error=True)
    add("medium-compound-window-short", win, len(wraw2) - 1, 7, "test_decode.py:926-927")
    add("medium-compound-adler", payload[:-1] + bytes((payload[-1] ^ 1,)), len(raw), 21,
        "test_decode.py:928")
    for index in range(8):
        payload, raw = td._alignment_stream(index)
        add("alignment-%d" % index, payload, len(raw), 0, "test_decode.py:600-605", raw=raw)
        payload, raw = td._late_code_length_stream(index)
        add("late-code-length-%d" % index, payload, len(raw), 0, "test_decode.py:608-613",
            raw=raw)
        payload, raw = td._truncated_prefix_tail_stream(index)
        add("truncated-prefix-tail-%d" % index, payload, len(raw), 0,
            "test_decode.py:672-677", raw=raw)
    payload, raw = td._embedded_candidate_stream()
    add("embedded-candidates", payload, len(raw), 0, "test_decode.py:630-634", raw=raw)
    add("embedded-candidates-limit1", payload, len(raw), 18, "test_decode.py:1078",
        limits=(1, 256))
    for empty in (True, False):
        payload, raw = td._many_dynamic_stream(empty)
        add("many-dynamic-%s" % ("empty" if empty else "tiny"), payload, len(raw), 0,
            "test_decode.py:637-643", raw=raw)
        add("many-dynamic-%s-limited" % ("empty" if empty else "tiny"), payload, len(raw), 0,
            "test_decode.py:1124-1145", limits=(4096, 256), raw=raw)
    many, _ = td._many_dynamic_stream(True)
    add("many-dynamic-blocks127", many, 0, 9, "test_decode.py:1079", limits=(4096, 127))
    payload, raw = td._long_literal_stream()
    add("long-literal-15bit", payload, len(raw), 0, "test_decode.py:646-650", raw=raw)
    payload, raw = td._grid_stride_stream()
    add("grid-stride", payload, len(raw), 0, "test_decode.py:680-684", raw=raw)
    payload, raw = td._dense_prefix_stored_stream()
    add("dense-prefix-stored", payload, len(raw), 0, "test_decode.py:616-627", raw=raw)
    add("dense-prefix-stored-limited", payload, len(raw), 0, "test_decode.py:1124-1145",
        limits=(4096, 256), raw=raw)
    add("dense-prefix-stored-adler-limited", payload[:-1] + bytes((payload[-1] ^ 1,)),
        len(raw), 21, "test_decode.py:1139", limits=(4096, 256))
    add("dense-prefix-stored-flg", payload[:1] + bytes((payload[1] ^ 1,)) + payload[2:],
        len(raw), 15, "test_decode.py:868-883")
    for blocks in (257, 1050):
        payload, raw = td._deep_reference_stream(blocks)
        add("deep-reference-%d" % blocks, payload, len(raw), 0, "test_decode.py:976-993",
            raw=raw)
    payload, raw = td._fixed_summary_stream()
    add("fixed-summary-limited", payload, len(raw), 0, "test_decode.py:1099-1116",
        limits=(4096, 256), raw=raw)
    add("fixed-summary", payload, len(raw), 0, "test_decode.py:1099-1116", raw=raw)
    invalid, _ = td._fixed_summary_stream(invalid=True)
    add("fixed-summary-invalid-limited", invalid, len(raw), 4, "test_decode.py:1114",
        limits=(4096, 256))
    # tests/test_decode.py:1062-1094: explicit-limit statuses.
    empty, eraw = td._dynamic_tree_stream("single-eob")
    add("limits-empty", empty, 0, 0, "test_decode.py:1080-1094", limits=(4096, 256), raw=eraw)
    add("limits-empty-header0", b"\x00" + empty[1:], 0, 15, "test_decode.py:1076",
        limits=(4096, 256))
    add("limits-empty-payload", b"", 0, 14, "test_decode.py:1075", limits=(4096, 256))
    add("limits-missing-final", td._wrap(td._stored(b"A", final=False), b"A"), 1, 1,
        "test_decode.py:1077", limits=(4096, 256))
    add("missing-final", td._wrap(td._stored(b"A", final=False), b"A"), 1, -1,
        "test_decode.py:453-455")
    # tests/test_decode.py:715-760: stdlib streams with one change each.
    raw = b"a checked fresh compressed stream\x00" * 128
    good = td._compressed(raw)
    add("checked-stream", good, len(raw), 0, "test_decode.py:715-760", raw=raw)
    body = bytearray(td._stored(raw))
    body[3] ^= 1
    for label, bad, expected in (
            ("too-small", good, len(raw) - 1), ("too-large", good, len(raw) + 1),
            ("adler", good[:-1] + bytes((good[-1] ^ 1,)), len(raw)),
            ("truncated-trailer", good[:-1], len(raw)),
            ("truncated-body", good[:-6] + good[-4:], len(raw)),
            ("trailing-byte", good + b"\x00", len(raw)),
            ("concatenated", good + good, len(raw)),
            ("reserved-block", td._wrap(b"\x07\x00", raw), len(raw)),
            ("stored-length", td._wrap(bytes(body), raw), len(raw)),
            ("distance-before-history", td._wrap(b"\x03\x02\x00", b"AAA"), 3)):
        add("checked-stream-" + label, bad, expected, -1, "test_decode.py:734-760")
    # tests/test_decode.py:763-784: checksum seams on each emission path.
    for length in (0, 4095, 4096, 4097):
        for encoding in ("stored", "local-fixed", "literal-dynamic"):
            data = (bytes(i % 251 for i in range(length)) if encoding == "stored"
                    else b"A" * length)
            if encoding == "stored":
                payload = td._wrap(td._stored(data), data)
            elif encoding == "local-fixed":
                payload = td._compressed(data, strategy=zlib.Z_FIXED)
            else:
                payload = td._wrap(td._bits(td._dynamic_literal_fields(data)), data)
            add("seam-%s-%d" % (encoding, length), payload, length, 0,
                "test_decode.py:763-784", raw=data)
            add("seam-%s-%d-adler" % (encoding, length),
                payload[:-1] + bytes((payload[-1] ^ 1,)), length, 21, "test_decode.py:780-782")
    # tests/test_decode.py:798-815: large stored stream with damage.
    for size in (65537, 1048577):
        data = random.Random(size).randbytes(size)
        payload = td._compressed(data, level=0)
        recipe = {"kind": "zlib-random", "seed": size, "size": size, "level": 0}
        add("large-stored-%d" % size, payload, size, 0, "test_decode.py:798-815", raw=data,
            recipe=recipe)
        add("large-stored-%d-header" % size, b"\x00" + payload[1:], size, 15,
            "test_decode.py:799", recipe=recipe, edits=[[0, 1, _b64(b"\x00")]])
        add("large-stored-%d-adler" % size, payload[:-1] + bytes((payload[-1] ^ 1,)), size,
            21, "test_decode.py:800", recipe=recipe,
            edits=[[-1, None, _b64(bytes((payload[-1] ^ 1,)))]])
        add("large-stored-%d-btype3" % size,
            payload[:2] + bytes(((payload[2] & 0xF8) | 7,)) + payload[3:], size, -1,
            "test_decode.py:801-802", recipe=recipe,
            edits=[[2, 3, _b64(bytes(((payload[2] & 0xF8) | 7,)))]])
        add("large-stored-%d-short" % size, payload, size - 1, -1, "test_decode.py:803",
            recipe=recipe)
        add("large-stored-%d-long" % size, payload, size + 1, -1, "test_decode.py:804",
            recipe=recipe)
    for size in (65536, 65537, 262144, 1048576, 1048577):
        data = bytes(size)
        payload = td._compressed(data)
        add("zeros-%d" % size, payload, size, 0, "test_decode.py:886-908", raw=data)
        add("zeros-%d-adler" % size, payload[:-1] + bytes((payload[-1] ^ 1,)), size, 21,
            "test_decode.py:902")
    # tests/test_decode.py:787-795: one bad block before a referencing block.
    literal = [0] * 258
    literal[256] = literal[257] = 1
    lengths = [0] * 19
    lengths[0] = lengths[1] = 1
    length_codes, literal_codes = td._codes(lengths), td._codes(literal)
    fields = []
    for final in [False, True]:
        fields += td._dynamic_header(258, 1, lengths, final)
        fields += [length_codes[w] for w in literal + [1]]
        fields += [literal_codes[257], (0, 1), literal_codes[256]]
    add("external-flag-history", td._wrap(td._bits(fields), b"A" * 6), 6, 6,
        "test_decode.py:787-795")

    # tests/test_regressions.py fixtures.
    payload, raw = tr._long_fixed()
    add("long-fixed", payload, len(raw), 0, "test_regressions.py:539-543", raw=raw)
    changes = {
        "too-small": (payload, len(raw) - 1), "too-large": (payload, len(raw) + 1),
        "adler": (payload[:-1] + bytes((payload[-1] ^ 1,)), len(raw)),
        "truncated-body": (payload[:-11] + payload[-4:], len(raw)),
        "missing-eob": (payload[:-5] + payload[-4:], len(raw)),
        "reserved-symbol": (tr._long_fixed("reserved-symbol")[0], len(raw)),
        "reserved-distance": (tr._long_fixed("reserved-distance")[0], len(raw)),
        "extra-deflate-byte": (payload[:-4] + b"\x00" + payload[-4:], len(raw)),
    }
    for label, (bad, expected) in changes.items():
        add("long-fixed-" + label, bad, expected, -1, "test_regressions.py:562-588")
    for kind, alignment in [("stored", 0)] + [("dynamic", n) for n in range(8)]:
        payload, raw = tr._chained_fixed(kind, alignment)
        add("chained-fixed-%s-%d" % (kind, alignment), payload, len(raw), 0,
            "test_regressions.py:546-552", raw=raw)
    payload, raw = tr._window_matches()
    add("window-matches", payload, len(raw), 0, "test_regressions.py:555-559", raw=raw)
    add("window-matches-cinfo6", td._header(cmf=0x68) + payload[2:], len(raw), -1,
        "test_regressions.py:591-600")
    for distance, length in tr._SEED_BOUNDARIES:
        payload, raw = tr._seed_match_stream("mixed", distance, length)
        add("seed-mixed-%d-%d" % (distance, length), payload, len(raw), 0,
            "test_regressions.py:354-362", raw=raw)
    payload, raw = tr._seed_match_stream("referenced")
    add("seed-referenced", payload, len(raw), 0, "test_regressions.py:365-370", raw=raw)
    for kind in ("local", "external"):
        for value in (0x00, 0x7f, 0xff):
            for length in (3, 258):
                payload, raw = tr._seed_match_stream(kind, 1, length, value)
                add("seed-%s-%d-%d" % (kind, value, length), payload, len(raw), 0,
                    "test_regressions.py:373-383", raw=raw)
    add("match-without-history", tr._match_without_history(), 3, -1,
        "test_regressions.py:386-396")
    for kind in ("fixed", "dynamic"):
        payload, raw = tr._warp_match_stream(kind)
        add("warp-match-%s" % kind, payload, len(raw), 0, "test_regressions.py:425-431",
            raw=raw)
        bad, bad_raw = tr._warp_match_stream(kind, "missing-eob")
        add("warp-match-%s-missing-eob" % kind, bad, len(bad_raw), -1,
            "test_regressions.py:434-450")
        payload, raw = tr._warp_history_stream(kind)
        add("warp-history-%s" % kind, payload, len(raw), 0, "test_regressions.py:453-469",
            raw=raw)
        bad, bad_raw = tr._warp_history_stream(kind, invalid=True)
        add("warp-history-%s-invalid" % kind, bad, len(bad_raw), 6,
            "test_regressions.py:466")
    bad, bad_raw = tr._warp_match_stream("fixed", "reserved-distance")
    add("warp-match-fixed-reserved-distance", bad, len(bad_raw), -1,
        "test_regressions.py:434-450")
    for size in (MIB, MIB + 1):
        payload, raw = tr._warp_match_stream("dynamic", block_size=size)
        add("warp-match-dynamic-%d" % size, payload, len(raw), 0,
            "test_regressions.py:472-482", raw=raw)
    payload, raw = tr._warp_history_stream("dynamic", block_size=MIB + 1)
    add("warp-history-dynamic-large", payload, len(raw), 0, "test_regressions.py:485-501",
        raw=raw)
    bad, bad_raw = tr._warp_history_stream("dynamic", invalid=True, block_size=MIB + 1)
    add("warp-history-dynamic-large-invalid", bad, len(bad_raw), 6,
        "test_regressions.py:497")
    for following in ("fixed", "dynamic"):
        payload, raw = tr._warp_match_stream("dynamic", block_size=MIB + 1,
                                             following=following)
        add("warp-following-%s" % following, payload, len(raw), 0,
            "test_regressions.py:504-515", raw=raw)
    return records


def encode_vectors(te, tm, tb):
    records = []

    def add(name, raw, chunk, size, sha, source):
        records.append({"name": name, "input": _b64(raw), "chunk_bytes": chunk,
                        "size": size, "sha256": sha, "source": source})

    # tests/test_encode.py:52-70 (size, sha) pins, chunk 32768.
    inputs = {
        "empty": b"", "one": b"a", "repeat": b"a" * 32768, "ramp": bytes(range(256)) * 128,
        "mixed": np.random.default_rng(1729).integers(0, 256, 32768, dtype=np.uint8).tobytes()
        + b"a" * 32768,
    }
    for kind, size, sha in _params(te.test_encoder_matches_original_streams,
                                   "kind,encoded_size,encoded_sha256"):
        add("original-" + kind, inputs[kind], 32768, size, sha, "test_encode.py:52-70")
    # tests/test_encode_match.py:26-57.
    unit = random.Random(811).randbytes(258)
    for matched, sha in _params(tm.test_encoder_match_boundaries, "matched,expected"):
        raw = (unit + b"\xff\x00" + unit[:matched] + b"\x01" +
               random.Random(813).randbytes(37) + bytes(4096))
        add("match-%d" % matched, raw, 32768, None, sha, "test_encode_match.py:26-49")
    for alphabet, sha in _params(tm.test_encoder_dictionary_collisions, "alphabet,expected"):
        raw = np.random.default_rng(811).integers(0, alphabet, 4096, dtype=np.uint8).tobytes()
        add("collision-%d" % alphabet, raw, 32768, None, sha, "test_encode_match.py:52-57")
    # tests/test_encode_bounds.py:16-35.
    for size, kind, chunk, encoded_size, sha in tb._CASES:
        if kind == "zeros":
            raw = bytes(size)
        elif kind == "text":
            raw = (b"ABCxyz" * ((size + 5) // 6))[:size]
        else:
            raw = random.Random(123 + size).randbytes(size)
        add("bounds-%d-%s-%d" % (size, kind, chunk), raw, chunk, encoded_size, sha,
            "test_encode_bounds.py:16-35")
    return records


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CUDA_ZLIB_REFERENCE")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    td, tr, te, tm, tb = _load_reference(root)
    decode = decode_vectors(td, tr)
    encode = encode_vectors(te, tm, tb)
    for name, records in (("decode_vectors.json.zz", decode), ("encode_vectors.json.zz", encode)):
        blob = zlib.compress(json.dumps(records, indent=0).encode(), 9)
        with open(os.path.join(HERE, name), "wb") as handle:
            handle.write(blob)
        print(name, len(records), "records", len(blob), "bytes")


if __name__ == "__main__":
    main()
