"""Multi-GPU sharding of the batch codec and of one stream's compression.

Two workloads split across GPUs without any exchange of codec data:

* the independent files of a batch call, assigned to GPUs by greedy
  longest-processing-time (LPT) balancing of their byte counts;
* the independent chunks of one compression stream, split into contiguous
  chunk-aligned ranges.  Each range is encoded as raw Deflate
  (cuda_zlib_compress_range); the host splices the two-byte zlib header, the
  range bodies in order and the Adler-32 combined from the ranges' partial
  checksums.  The result is byte-identical to compressing the whole input on
  one GPU, because every chunk is encoded on its own.

Nothing is reduced across GPUs, so no collective is used: each GPU's results
are copied into disjoint slices of one pinned host buffer.  Single-stream
decompression does not shard (its blocks form one serial chain with
cross-block history); run independent streams on different GPUs instead.

The planners are plain functions of sizes, shared by the in-process
multi-device calls below and by one-process-per-GPU jobs (rank_files,
rank_ranges), so every rank derives the same partition with no communication.
"""
import heapq
import struct
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import _codec, _native
from ._errors import CodecError

_ADLER_MOD = 65521


# ---------------------------------------------------------------- planning
def plan_files(weights, parts):
    """Greedy LPT assignment of items to `parts` bins.

    Items go in decreasing weight order (ties: lower index first) to the bin
    with the least load so far (ties: lower bin).  Returns one ascending index
    list per bin.  Deterministic, so every rank computes the same plan.
    """
    if type(parts) is not int or parts < 1:
        raise ValueError("parts must be a positive integer")
    weights = [int(w) for w in weights]
    if any(w < 0 for w in weights):
        raise ValueError("weights must be nonnegative")
    order = sorted(range(len(weights)), key=lambda i: (-weights[i], i))
    loads = [(0, p) for p in range(parts)]
    bins = [[] for _ in range(parts)]
    for i in order:
        load, p = heapq.heappop(loads)
        bins[p].append(i)
        heapq.heappush(loads, (load + weights[i], p))
    return [sorted(b) for b in bins]


def rank_files(weights, rank, world):
    """This rank's items under plan_files (one process per GPU)."""
    return plan_files(weights, world)[rank]


def plan_ranges(size, chunk_bytes, parts, max_range=None):
    """Split [0, size) into chunk-aligned ranges for `parts` devices.

    Returns one list of (start, stop) per device: contiguous, in stream order
    (device 0 first), the chunks shared as evenly as possible, and each range
    at most `max_range` bytes (rounded down to whole chunks) so every call
    stays inside the single-call bounds.  With fewer chunks than devices
    some devices get no range; an empty input is one empty range.
    """
    if type(parts) is not int or parts < 1:
        raise ValueError("parts must be a positive integer")
    _codec._check_chunk(chunk_bytes)
    chunks = max(1, -(-size // chunk_bytes))
    limit = chunks if max_range is None else max(1, max_range // chunk_bytes)
    plan = []
    for p in range(parts):
        first, last = p * chunks // parts, (p + 1) * chunks // parts
        ranges = []
        for c in range(first, last, limit):
            stop_chunk = min(last, c + limit)
            ranges.append((c * chunk_bytes, min(size, stop_chunk * chunk_bytes)))
        plan.append(ranges)
    return plan


def rank_ranges(size, chunk_bytes, rank, world, max_range=None):
    """This rank's ranges under plan_ranges (one process per GPU)."""
    return plan_ranges(size, chunk_bytes, world, max_range)[rank]


# ---------------------------------------------------------------- splicing
def adler32_combine(first, second, second_length):
    """Adler-32 of A + B from adler32(A), adler32(B) and len(B).

    With A's sums (a1, b1) and B's (a2, b2) over n = len(B) bytes:
    a = a1 + a2 - 1 and b = b1 + b2 + n * (a1 - 1), all mod 65521
    (RFC 1950 section 8.2 defines the sums).
    """
    n = second_length % _ADLER_MOD
    a1, b1 = first & 0xFFFF, first >> 16
    a2, b2 = second & 0xFFFF, second >> 16
    a = (a1 + a2 + _ADLER_MOD - 1) % _ADLER_MOD
    b = (b1 + b2 + n * (a1 + _ADLER_MOD - 1)) % _ADLER_MOD
    return (b << 16) | a


def combine_adlers(adlers, lengths):
    total = 1
    for value, length in zip(adlers, lengths):
        total = adler32_combine(total, value, length)
    return total


def splice_header():
    """The two zlib header bytes the codec writes (CM 8, CINFO 7, FLEVEL 0)."""
    return b"\x78\x01"


def splice_trailer(adler):
    return struct.pack(">I", adler)


# ---------------------------------------------------------------- runners
def _devices(devices):
    torch = _codec._torch()
    if not isinstance(devices, (list, tuple)) or not devices:
        raise ValueError("devices must be a nonempty sequence of CUDA devices")
    return [_codec._select_device(d) for d in devices], torch


def _run_per_device(jobs):
    """Run one callable per device concurrently; re-raise the first error."""
    if len(jobs) == 1:
        return [jobs[0]()]
    with ThreadPoolExecutor(max_workers=len(jobs)) as pool:
        futures = [pool.submit(job) for job in jobs]
        return [f.result() for f in futures]


def _range_call(torch, device, source, start, stop, chunk_bytes, last):
    """Encode input[start:stop) on `device`; returns (body tensor, length, adler)."""
    lib = _native.library()
    size = stop - start
    capacity = _codec._capacity(size, chunk_bytes)[0]
    with torch.cuda.device(device):
        if _codec._is_tensor(source):
            raw = source[start:stop].to(device, non_blocking=False)
        else:
            raw = _codec._device_input(memoryview(source)[start:stop], device)
        output = torch.empty(capacity, dtype=torch.uint8, device=device)
        meta = torch.zeros(3, dtype=torch.uint32, device=device)
        _native.check(lib.cuda_zlib_compress_range(
            _codec._ptr(raw), size, chunk_bytes, int(last), output.data_ptr(), capacity,
            meta.data_ptr(), _codec._stream(device)), "CUDA range compression")
        length, status, adler = (int(v) for v in meta.cpu().numpy())
    _codec._check_value(status, "CUDA range compression")
    return output, length, adler


def compress_zlib_host_sharded(data, devices, *, chunk_bytes=32768):
    """Compress one stream with its chunks split across `devices`.

    Returns a read-only NumPy uint8 array in pinned host memory holding the
    zlib stream, byte-identical to compress_zlib_host on one device.  The
    input may exceed the single-call bound (2**31 bytes): each device encodes
    its share in ranges that fit one call.
    """
    devices, torch = _devices(devices)
    if _codec._is_tensor(data):
        if data.dtype != torch.uint8 or data.ndim != 1:
            raise TypeError("array input must be one-dimensional uint8")
        if data.device.type != "cpu":
            raise ValueError("sharded compression takes host input")
        source, size = data.contiguous(), int(data.shape[0])
    elif isinstance(data, (bytes, bytearray, memoryview, np.ndarray)):
        view = memoryview(data).cast("B") if not isinstance(data, np.ndarray) else \
            memoryview(np.ascontiguousarray(data, dtype=np.uint8)).cast("B")
        source, size = view, view.nbytes
    else:
        raise TypeError("input must be bytes or a one-dimensional uint8 array or tensor")
    _codec._check_chunk(chunk_bytes)
    # Largest range one call takes (whole chunks).
    max_range = _codec._MAX_STREAM // chunk_bytes * chunk_bytes
    plan = plan_ranges(size, chunk_bytes, len(devices), max_range)
    final_range = max((p, len(r) - 1) for p, r in enumerate(plan) if r)

    def encode(p):
        results = []
        for k, (start, stop) in enumerate(plan[p]):
            last = (p, k) == final_range
            results.append(_range_call(torch, devices[p], source, start, stop, chunk_bytes, last))
        return results

    parts = _run_per_device([lambda p=p: encode(p) for p in range(len(devices))])
    flat = [(p, r) for p in range(len(devices)) for r in parts[p]]
    lengths = [r[1] for _, r in flat]
    sizes = [stop - start for p in range(len(devices)) for start, stop in plan[p]]
    adler = combine_adlers([r[2] for _, r in flat], sizes)
    total = 2 + sum(lengths) + 4
    host = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    array = host.numpy()
    array[:2] = np.frombuffer(splice_header(), dtype=np.uint8)
    array[total - 4:] = np.frombuffer(splice_trailer(adler), dtype=np.uint8)
    offsets = np.cumsum([2] + lengths[:-1]).tolist()

    def gather(p):
        with torch.cuda.device(devices[p]):
            for (q, (body, length, _)), offset in zip(flat, offsets):
                if q == p and length:
                    host[offset:offset + length].copy_(body[:length], non_blocking=True)
            torch.cuda.current_stream(devices[p]).synchronize()

    _run_per_device([lambda p=p: gather(p) for p in range(len(devices))])
    array.flags.writeable = False
    return array


def _groups(indices, costs, limits):
    """Consecutive groups of `indices` whose summed costs stay within `limits`.

    costs[i] is a tuple per item (e.g. files, input bytes, output bytes) and
    limits the matching bounds of one batch call.
    """
    groups, current, totals = [], [], [0] * len(limits)
    for i in indices:
        if current and any(t + c > lim for t, c, lim in zip(totals, costs[i], limits)):
            groups.append(current)
            current, totals = [], [0] * len(limits)
        current.append(i)
        totals = [t + c for t, c in zip(totals, costs[i])]
    if current:
        groups.append(current)
    return groups


def decompress_zlib_batch_host_sharded(payloads, expected_sizes, devices):
    """decompress_zlib_batch_host with the files split across `devices`.

    Files are assigned by LPT over compressed + decoded bytes.  Returns one
    read-only NumPy view per file (in input order) into a single pinned host
    buffer that holds each device's outputs in one contiguous slice.
    """
    devices, torch = _devices(devices)
    if not isinstance(payloads, (tuple, list)) or not payloads:
        raise ValueError("inputs must be a nonempty sequence of files")
    blobs = [bytes(p) if not isinstance(p, bytes) else p for p in payloads]
    expected = tuple(expected_sizes)
    if len(expected) != len(blobs):
        raise ValueError("input_sizes and expected_sizes must have matching lengths")
    if any(type(n) is not int or not 0 <= n <= _codec._MAX_BYTES for n in expected):
        raise ValueError("expected_sizes must contain integers in [0, 2**28]")
    weights = [len(b) + n for b, n in zip(blobs, expected)]
    plan = plan_files(weights, len(devices))
    bases, base = [], 0
    for files in plan:
        bases.append(base)
        base += sum(expected[i] for i in files)
    host = torch.empty(base, dtype=torch.uint8, pin_memory=True)
    array = host.numpy()
    where = [0] * len(blobs)

    def decode(p):
        offset = bases[p]
        costs = [(1, len(b), n) for b, n in zip(blobs, expected)]
        limits = (_codec._MAX_BLOCKS, _codec._MAX_BYTES, _codec._MAX_BYTES)
        groups = _groups(plan[p], costs, limits)
        for group in groups:
            sizes = [len(blobs[i]) for i in group]
            outs = [expected[i] for i in group]
            output, meta = _codec.decompress_zlib_batch_checked(
                b"".join(blobs[i] for i in group), sizes, outs, devices[p])
            with torch.cuda.device(devices[p]):
                if output.numel():
                    host[offset:offset + output.numel()].copy_(output, non_blocking=True)
                meta = meta.cpu().numpy()
            for k, i in enumerate(group):
                _codec._check_value(int(meta[k][0]), "CUDA batch decompression file %d" % i)
                where[i] = offset
                offset += expected[i]

    _run_per_device([lambda p=p: decode(p) for p in range(len(devices))])
    array.flags.writeable = False
    return tuple(array[where[i]:where[i] + expected[i]] for i in range(len(blobs)))


def compress_zlib_batch_host_sharded(inputs, devices, *, chunk_bytes=32768):
    """compress_zlib_batch_host with the files split across `devices`.

    Files are assigned by LPT over their sizes; returns a tuple of bytes
    streams in input order, each identical to the one-device result.
    """
    devices, torch = _devices(devices)
    if not isinstance(inputs, (tuple, list)) or not inputs:
        raise ValueError("inputs must be a nonempty sequence of files")
    blobs = [bytes(x) if not isinstance(x, bytes) else x for x in inputs]
    _codec._check_chunk(chunk_bytes)
    sizes = [len(b) for b in blobs]
    capacities = [_codec._capacity(n, chunk_bytes)[0] for n in sizes]
    plan = plan_files(sizes, len(devices))
    streams = [None] * len(blobs)

    def encode(p):
        costs = [(max(1, -(-n // chunk_bytes)), c) for n, c in zip(sizes, capacities)]
        groups = _groups(plan[p], costs, (_codec._MAX_BLOCKS, _codec._MAX_BYTES))
        for group in groups:
            output, meta = _codec.compress_zlib_batch_padded(
                b"".join(blobs[i] for i in group), [sizes[i] for i in group], devices[p],
                chunk_bytes=chunk_bytes)
            with torch.cuda.device(devices[p]):
                packed = _codec._to_pinned_host(output)
                meta = meta.cpu().numpy()
            offset = 0
            for k, i in enumerate(group):
                _codec._check_value(int(meta[k][1]), "CUDA batch compression file %d" % i)
                streams[i] = packed[offset:offset + int(meta[k][0])].tobytes()
                offset += capacities[i]

    _run_per_device([lambda p=p: encode(p) for p in range(len(devices))])
    return tuple(streams)


__all__ = ["plan_files", "rank_files", "plan_ranges", "rank_ranges", "adler32_combine",
           "combine_adlers", "compress_zlib_host_sharded", "decompress_zlib_batch_host_sharded",
           "compress_zlib_batch_host_sharded", "CodecError"]
