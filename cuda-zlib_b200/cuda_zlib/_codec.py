"""Bounded RFC 1950 codec on B200 through the native C ABI.

Mirrors xangma/cuda-zlib's API module (src/cuda_zlib/_codec.py): the same
validation order and errors, the same padded-slot formula and metadata
layouts ([encoded_length, status] for compression, [status, 0] for
decompression), and the same batch bounds (2**28 bytes, 262144 blocks and
files).  Two bounds are deliberate supersets of the reference's: a single
stream may hold up to 2**31 uncompressed bytes (and, to decode, at most
2**29 - 2**16 compressed bytes), where the reference stops at 2**28
(_codec.py:13,28,103); and chunk_bytes may be up to 262144, where the
reference stops at 65535 (_codec.py:158-159).  A chunk above 65535 bytes
falls back to several stored blocks, so the padded slot is
size + 5 * (stored blocks) + 6, which equals the reference's
size + 5 * chunks + 6 whenever chunk_bytes <= 65535.
Device arrays are PyTorch CUDA tensors; host results are read-only NumPy
arrays backed by pinned memory.  Calls run on the device's current PyTorch
stream; the *_padded / *_checked variants never synchronize the host.
"""
import os
import threading
import warnings
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import _hostio, _native
from ._errors import BackendUnavailable, CodecError, UnsupportedStream

_MAX_BYTES = 2**28
_MAX_STREAM = 2**31                  # one stream's uncompressed bytes
_MAX_STREAM_PAYLOAD = 2**29 - 2**16  # one stream's compressed bytes, to decode
_MAX_CHUNK = 262144
_STORED_MAX = 65535
_MAX_CANDIDATES = 262144
_MAX_BLOCKS = 262144
_MESSAGES = {
    0: "success",
    1: "truncated Deflate payload",
    2: "reserved Deflate block type",
    3: "invalid Huffman tree",
    4: "invalid or reserved Huffman symbol",
    5: "invalid code-length repeat",
    6: "invalid backward distance or history",
    7: "decoded output exceeds the declared bound",
    9: "Deflate block workspace capacity exceeded",
    10: "dynamic block boundary was not discovered",
    11: "final decoded size differs from the declared size",
    12: "block endpoint or payload extent mismatch",
    13: "fixed-block tile summaries required",
    14: "truncated zlib payload", 15: "invalid zlib CMF/FLG header",
    16: "native CUDA codec supports RFC 1950 zlib",
    17: "zlib preset dictionaries are unsupported",
    18: "Deflate candidate workspace overflow", 19: "Deflate initial block missing",
    20: "Deflate back-reference depth exceeded", 21: "CUDA Adler32 mismatch",
    22: "CUDA compression workspace overflow", 23: "invalid codec bounds",
    24: "invalid gzip header", 25: "gzip CRC32 mismatch", 26: "gzip ISIZE mismatch",
}


def _torch():
    try:
        import torch
    except ImportError as exc:  # pragma: no cover - torch is part of the image
        raise BackendUnavailable("the CUDA codec requires PyTorch for device memory") from exc
    return torch


def _validate_size(size):
    if type(size) is not int or not 0 <= size <= _MAX_STREAM:
        raise ValueError("expected_bytes must be an integer in [0, 2**31]")


def _check_chunk(chunk_bytes):
    if type(chunk_bytes) is not int or not 256 <= chunk_bytes <= _MAX_CHUNK:
        raise ValueError("chunk_bytes must be an integer in [256, 262144]")


def _validate_device(device):
    torch = _torch()
    if type(device) is int:
        if device >= 0:
            return
    elif isinstance(device, torch.device) and device.type == "cuda":
        return
    raise BackendUnavailable("device must be a nonnegative CUDA ordinal or CUDA torch device")


def _select_device(device):
    """Return a torch.device('cuda', i) for an ordinal or CUDA device."""
    _validate_device(device)
    torch = _torch()
    if not torch.cuda.is_available():
        raise BackendUnavailable("CUDA backend unavailable")
    index = device if type(device) is int else (device.index if device.index is not None
                                               else torch.cuda.current_device())
    if index >= torch.cuda.device_count():
        raise BackendUnavailable("requested CUDA device is unavailable")
    return torch.device("cuda", index)


def _is_tensor(data):
    return type(data).__module__.startswith("torch") and hasattr(data, "dtype")


_LIMIT_TEXT = {_MAX_BYTES: "2**28", _MAX_STREAM: "2**31",
               _MAX_STREAM_PAYLOAD: "2**29 - 2**16"}


def _input_size(data, label="input", limit=_MAX_BYTES):
    if isinstance(data, (bytes, bytearray, memoryview)):
        size = memoryview(data).nbytes
    elif isinstance(data, np.ndarray) or _is_tensor(data):
        torch = _torch() if _is_tensor(data) else None
        dtype_ok = data.dtype == (torch.uint8 if torch else np.uint8)
        if not dtype_ok or data.ndim != 1:
            raise TypeError("array input must be one-dimensional uint8")
        size = int(data.shape[0])
    else:
        raise TypeError(label + " must be bytes or a one-dimensional uint8 array or tensor")
    if size > limit:
        raise ValueError(label + " exceeds size limit (%s bytes)" % _LIMIT_TEXT[limit])
    return size


def _stream(device):
    torch = _torch()
    return torch.cuda.current_stream(device).cuda_stream


_STAGE_PIECE = 4 << 20   # bytes per staging-copy task
_stage_pool = None
_stage_lock = threading.Lock()


def _staging_pool():
    """Host threads that fill pinned staging buffers (NumPy copies drop the GIL)."""
    global _stage_pool
    if _stage_pool is None:
        with _stage_lock:
            if _stage_pool is None:
                workers = max(1, min(16, (os.cpu_count() or 1)))
                _stage_pool = ThreadPoolExecutor(max_workers=workers,
                                                 thread_name_prefix="cuda_zlib_stage")
    return _stage_pool


def _pinned_copy(data, device):
    """Pageable host bytes -> device tensor through one pinned staging buffer.

    Large inputs are copied into the staging buffer by several host threads,
    since one thread's memcpy is several times slower than the H2D link.
    """
    torch = _torch()
    view = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data
    view = np.ascontiguousarray(view, dtype=np.uint8)
    staging = torch.empty(view.size, dtype=torch.uint8, pin_memory=True)
    host = staging.numpy()
    if view.size >= 2 * _STAGE_PIECE:
        pieces = range(0, view.size, _STAGE_PIECE)

        def fill(start):
            host[start:start + _STAGE_PIECE] = view[start:start + _STAGE_PIECE]

        for future in [_staging_pool().submit(fill, start) for start in pieces]:
            future.result()
    elif view.size:
        host[:] = view
    return staging.to(device, non_blocking=True)


def _pinned_tensor(data):
    """A CPU tensor over `data` when it already lives in page-locked memory."""
    torch = _torch()
    if not (isinstance(data, np.ndarray) and data.size and data.flags.c_contiguous):
        return None
    with warnings.catch_warnings():
        # Read-only arrays (e.g. a *_host result) are only read here.
        warnings.simplefilter("ignore", UserWarning)
        tensor = torch.from_numpy(data)
    return tensor if tensor.is_pinned() else None


def _device_input(data, device):
    torch = _torch()
    if _is_tensor(data):
        if data.device.type == "cuda":
            if data.device != device:
                raise ValueError("input array and requested CUDA device differ")
            return data.contiguous()
        # Pinned CPU tensors go straight to the device by DMA.
        return data.contiguous().to(device, non_blocking=False)
    if isinstance(data, np.ndarray):
        pinned = _pinned_tensor(data)
        if pinned is not None:
            return pinned.to(device, non_blocking=False)
    if isinstance(data, (bytes, bytearray, memoryview, np.ndarray)):
        return _pinned_copy(data, device)
    raise TypeError("input must be bytes or a one-dimensional uint8 array or tensor")


def _check_framing(payload, expected_bytes):
    view = memoryview(payload).cast("B")
    _validate_size(expected_bytes)
    if view.nbytes < 8:
        raise CodecError("truncated zlib payload")
    if view.nbytes > _MAX_STREAM_PAYLOAD:
        raise ValueError("compressed payload exceeds 2**29 - 2**16 bytes")
    cmf, flg = view[0], view[1]
    if cmf == 0x1F and flg == 0x8B:
        raise UnsupportedStream("native CUDA codec supports RFC 1950 zlib")
    if cmf & 15 != 8 or cmf >> 4 > 7 or (cmf * 256 + flg) % 31:
        raise CodecError("invalid zlib CMF/FLG header")
    if flg & 32:
        raise UnsupportedStream("zlib preset dictionaries are unsupported")


def _check_value(value, operation):
    if value:
        message = _MESSAGES.get(value, "unknown error")
        error = UnsupportedStream if value in (16, 17) else CodecError
        raise error("%s: %s (Deflate status %d)" % (operation, message, value))


def _ptr(tensor):
    return tensor.data_ptr() if tensor.numel() else None


def compile_kernels(device=0):
    """Load the native library and prepare `device` (pool, kernel attributes)."""
    selected = _select_device(device)
    torch = _torch()
    lib = _native.library()
    with torch.cuda.device(selected):
        meta = torch.empty(2, dtype=torch.uint32, device=selected)
        out = torch.empty(11, dtype=torch.uint8, device=selected)
        _native.check(lib.cuda_zlib_compress(None, 0, 32768, out.data_ptr(), 11, meta.data_ptr(),
                                             _stream(selected)), "CUDA compression")


def workspace_pool_stats(device=0):
    """Return retention, reserved/live bytes and pool count for a CUDA device.

    Scratch pools retain up to a 1 GiB release threshold by default. Set
    CUDA_ZLIB_WORKSPACE_RETENTION_BYTES before the first call to change it;
    zero disables retention. The threshold is not a hard allocation cap.
    """
    import ctypes
    selected = _select_device(device)
    values = (ctypes.c_uint64 * 4)()
    _native._check_pool_error(_native.library().CudaZlibWorkspacePoolStats(selected.index, values))
    return dict(zip(("retention_bytes", "reserved_bytes", "used_bytes", "pool_count"), values))


def trim_workspace_pool(device=0):
    """Try to release unused codec scratch memory on the requested device."""
    selected = _select_device(device)
    _native._check_pool_error(_native.library().CudaZlibTrimWorkspacePool(selected.index))


def _stored_blocks(size):
    return max(1, -(-size // _STORED_MAX))


def _layout(size, chunk_bytes):
    """(capacity, chunks, most Deflate blocks) of one stream.

    The capacity is size + 5 * (stored blocks of every chunk's stored
    fallback) + 6: size + 5 * chunks + 6 for chunks of at most 65535 bytes
    (the reference's formula, _codec.py:151-177).  Every nonfinal chunk can
    end with an empty stored block, so the stream holds at most
    2 * chunks - 1 blocks, or the stored blocks when a chunk needs more.
    """
    chunks = max(1, (size + chunk_bytes - 1) // chunk_bytes)
    full, tail = _stored_blocks(chunk_bytes), _stored_blocks(size - (chunks - 1) * chunk_bytes)
    stored = (chunks - 1) * full + tail
    blocks = (chunks - 1) * max(full, 2) + tail
    return size + 5 * stored + 6, chunks, blocks


def _capacity(size, chunk_bytes):
    capacity, chunks, _ = _layout(size, chunk_bytes)
    return capacity, chunks


def _check_level(level):
    if type(level) is not int or level not in (1, 2):
        raise ValueError("level must be 1 (the reference encoder) or 2")


def compress_zlib_padded(data, device=0, *, chunk_bytes=32768, level=1):
    """Return ``(buffer, [encoded_length, status])`` without a host sync.

    The fixed-size buffer holds a zlib stream followed by zero padding.
    Status zero means success; check it before using the stream.  level 1
    (the default) is the reference's encoder, byte for byte; level 2, which
    the reference does not have, searches hash chains with lazy evaluation
    for smaller streams at a lower rate.
    """
    _check_level(level)
    if level != 1:
        from . import formats
        return formats._compress_padded(data, device, chunk_bytes, formats.FORMAT_ZLIB, level)
    _check_chunk(chunk_bytes)
    size = _input_size(data, limit=_MAX_STREAM)
    capacity, chunks, blocks = _layout(size, chunk_bytes)
    if blocks > _MAX_BLOCKS:
        raise ValueError("chunk count exceeds decoder block limit")
    selected = _select_device(device)
    torch = _torch()
    lib = _native.library()
    raw = _device_input(data, selected)
    with torch.cuda.device(selected):
        output = torch.empty(capacity, dtype=torch.uint8, device=selected)
        metadata = torch.empty(2, dtype=torch.uint32, device=selected)
        _native.check(lib.cuda_zlib_compress(_ptr(raw), size, chunk_bytes, output.data_ptr(),
                                             capacity, metadata.data_ptr(), _stream(selected)),
                      "CUDA compression")
    return output, metadata


def _batch_sizes(sizes, label):
    if not isinstance(sizes, (tuple, list)) or not 1 <= len(sizes) <= _MAX_BLOCKS:
        raise ValueError(label + " must contain between 1 and 262144 static sizes")
    sizes = tuple(sizes)
    # Exact ints only (bool and NumPy integers are refused), each in range;
    # checked by C-level passes, a batch call issues thousands of sizes.
    if (not set(map(type, sizes)) <= {int} or min(sizes) < 0 or
            max(sizes) > _MAX_BYTES):
        raise ValueError(label + " must contain integers in [0, 2**28]")
    if sum(sizes) > _MAX_BYTES:
        raise ValueError(label + " total exceeds 2**28 bytes")
    return sizes


def _batch_capacities(sizes, chunk_bytes):
    """Padded slot sizes of a batch (_layout per file, vectorised)."""
    _check_chunk(chunk_bytes)
    sizes = np.asarray(sizes, dtype=np.int64)
    chunks = np.maximum(1, -(-sizes // chunk_bytes))
    full = max(1, -(-chunk_bytes // _STORED_MAX))
    tail = np.maximum(1, -(-(sizes - (chunks - 1) * chunk_bytes) // _STORED_MAX))
    blocks = (chunks - 1) * max(full, 2) + tail
    if int(chunks.sum()) > _MAX_BLOCKS or (blocks.size and int(blocks.max()) > _MAX_BLOCKS):
        raise ValueError("batch chunk count exceeds workspace limit")
    capacities = sizes + 5 * ((chunks - 1) * full + tail) + 6
    if int(capacities.sum()) > _MAX_BYTES:
        raise ValueError("batch compressed capacity exceeds 2**28 bytes")
    return tuple(capacities.tolist())


def _i64_array(values):
    """The values as a C int64 array (one C-level copy through NumPy; the
    ctypes array keeps its buffer alive)."""
    return np.ctypeslib.as_ctypes(np.array(values, dtype=np.int64))


def _batch_encode_call(data, input_sizes, device, chunk_bytes, entry):
    sizes = _batch_sizes(input_sizes, "input_sizes")
    if _input_size(data) != sum(sizes):
        raise ValueError("packed input length differs from input_sizes total")
    capacities = _batch_capacities(sizes, chunk_bytes)
    selected = _select_device(device)
    torch = _torch()
    lib = _native.library()
    raw = _device_input(data, selected)
    total = sum(capacities)
    with torch.cuda.device(selected):
        output = torch.empty(total, dtype=torch.uint8, device=selected)
        metadata = torch.empty((len(sizes), 2), dtype=torch.uint32, device=selected)
        _native.check(getattr(lib, entry)(
            _ptr(raw), sum(sizes), _i64_array(sizes), len(sizes), chunk_bytes,
            _ptr(output), total, metadata.data_ptr(), _stream(selected)),
            "CUDA batch compression")
    return output, metadata


def compress_zlib_batch_packed(data, input_sizes, device=0, *, chunk_bytes=32768):
    """compress_zlib_batch_padded with the streams back to back.

    No reference counterpart.  Same arguments, bounds and metadata; the
    output buffer has the padded size, but file k's stream starts at the sum
    of the earlier files' encoded lengths (failed files take no bytes) and the
    rest is zero, so copying ``output[:metadata[:, 0].sum()]`` moves only the
    encoded bytes.  No host sync.
    """
    return _batch_encode_call(data, input_sizes, device, chunk_bytes,
                              "cuda_zlib_compress_batch_packed")


def compress_zlib_batch_padded(data, input_sizes, device=0, *, chunk_bytes=32768):
    """Compress packed independent files in one call, without a host sync.

    ``input_sizes`` lists the file lengths (their sum is len(data)).  Returns a
    flat uint8 buffer of consecutive padded slots and uint32 metadata of shape
    (files, 2) with [encoded_length, status] per file.  A slot has
    ``size + 5 * max(1, ceil(size / chunk_bytes)) + 6`` bytes for chunk_bytes
    up to 65535 (larger chunks count ceil(chunk / 65535) stored blocks each).
    """
    return _batch_encode_call(data, input_sizes, device, chunk_bytes,
                              "cuda_zlib_compress_batch")


def decompress_zlib_batch_checked(payload, input_sizes, expected_sizes, device=0,
                                  *, encoded_metadata=None):
    """Decode packed independent streams in one call, without a host sync.

    Input streams and returned outputs are packed back to back.  To decode
    padded compression slots directly, pass their capacities as input_sizes
    and compression's (files, 2) uint32 metadata as encoded_metadata.
    Returns a flat output and (files, 2) uint32 [status, 0] metadata.
    """
    sizes = _batch_sizes(input_sizes, "input_sizes")
    expected = _batch_sizes(expected_sizes, "expected_sizes")
    if len(sizes) != len(expected):
        raise ValueError("input_sizes and expected_sizes must have matching lengths")
    if _input_size(payload, "compressed payload") != sum(sizes):
        raise ValueError("packed input length differs from input_sizes total")
    selected = _select_device(device)
    torch = _torch()
    lib = _native.library()
    raw = _device_input(payload, selected)
    lengths = None
    if encoded_metadata is not None:
        if (not _is_tensor(encoded_metadata) or encoded_metadata.dtype != torch.uint32 or
                tuple(encoded_metadata.shape) != (len(sizes), 2)):
            raise TypeError("encoded_metadata must be a uint32 tensor with shape (files, 2)")
        if encoded_metadata.device != selected:
            raise ValueError("input array and requested CUDA device differ")
        lengths = encoded_metadata.contiguous()
    total = sum(expected)
    with torch.cuda.device(selected):
        output = torch.empty(total, dtype=torch.uint8, device=selected)
        metadata = torch.empty((len(sizes), 2), dtype=torch.uint32, device=selected)
        _native.check(lib.cuda_zlib_decompress_batch(
            _ptr(raw), sum(sizes), _i64_array(sizes), _i64_array(expected), len(sizes),
            None if lengths is None else lengths.data_ptr(), _ptr(output), total,
            metadata.data_ptr(), _stream(selected)), "CUDA batch decompression")
    return output, metadata


def _pack_batch(inputs, device):
    if not isinstance(inputs, (tuple, list)) or not inputs:
        raise ValueError("inputs must be a nonempty sequence of files")
    sizes = _batch_sizes(tuple(_input_size(data) for data in inputs), "input_sizes")
    if all(isinstance(data, (bytes, bytearray, memoryview)) for data in inputs):
        return b"".join(bytes(data) for data in inputs), sizes
    torch = _torch()
    parts = [_device_input(data, device) for data in inputs]
    return torch.cat(parts) if parts else torch.empty(0, dtype=torch.uint8, device=device), sizes


def _check_batch(metadata, operation, compression=False):
    metadata = metadata.cpu().numpy()
    for i, row in enumerate(metadata):
        _check_value(int(row[1 if compression else 0]), "%s file %d" % (operation, i))
    return metadata


def _split_batch(buffer, sizes, extents=None):
    offset = 0
    results = []
    for i, size in enumerate(sizes):
        length = size if extents is None else int(extents[i])
        results.append(buffer[offset:offset + length])
        offset += size
    return tuple(results)


def _to_pinned_host(tensor):
    """One D2H transfer into pinned memory; returns a read-only NumPy view."""
    torch = _torch()
    host = torch.empty(tensor.numel(), dtype=torch.uint8, pin_memory=True)
    if tensor.numel():
        host.copy_(tensor, non_blocking=True)
    torch.cuda.current_stream(tensor.device).synchronize()
    array = host.numpy()
    array.flags.writeable = False
    return array


def compress_zlib_batch(inputs, device=0, *, chunk_bytes=32768):
    """Return completed exact-length device streams for a sequence of files."""
    selected = _select_device(device)
    packed, sizes = _pack_batch(inputs, selected)
    output, metadata = compress_zlib_batch_padded(packed, sizes, selected, chunk_bytes=chunk_bytes)
    lengths = _check_batch(metadata, "CUDA batch compression", True)[:, 0]
    return _split_batch(output, _batch_capacities(sizes, chunk_bytes), lengths)


def decompress_zlib_batch(payloads, expected_sizes, device=0):
    """Return completed device outputs for independent streams; checks statuses once."""
    selected = _select_device(device)
    packed, sizes = _pack_batch(payloads, selected)
    expected = _batch_sizes(expected_sizes, "expected_sizes")
    output, metadata = decompress_zlib_batch_checked(packed, sizes, expected, selected)
    _check_batch(metadata, "CUDA batch decompression")
    return _split_batch(output, expected)


def _host_sizes(sizes, label):
    """Per-file sizes of a host batch call as int64 (each in [0, 2**28]; the
    total is not bounded: the call splits into device calls)."""
    if isinstance(sizes, np.ndarray):
        if sizes.ndim != 1 or sizes.dtype.kind not in "iu":
            raise ValueError(label + " must contain integers in [0, 2**28]")
        values = sizes.astype(np.int64)
    elif isinstance(sizes, (tuple, list)) and all(type(v) is int for v in sizes):
        values = np.array(sizes, dtype=np.int64) if sizes else np.empty(0, np.int64)
    else:
        raise ValueError(label + " must contain integers in [0, 2**28]")
    if values.size and (values.min() < 0 or values.max() > _MAX_BYTES):
        raise ValueError(label + " must contain integers in [0, 2**28]")
    if not 1 <= values.size:
        raise ValueError(label + " must contain at least one size")
    return values


def _host_packed(data, sizes, label):
    packed = _hostio.as_host_array(data)
    if packed is None:
        raise ValueError(label + " must be in host memory")
    if packed.size != int(sizes.sum()):
        raise ValueError("packed input length differs from input_sizes total")
    return packed


_HOST_LIMITS = (_MAX_BLOCKS, _MAX_BYTES, _MAX_BYTES)


def decompress_zlib_batch_checked_host(payload, input_sizes, expected_sizes, device=0):
    """Host-buffer counterpart of decompress_zlib_batch_checked.

    Packed streams in host memory (bytes, NumPy uint8 or a CPU tensor; page-
    locked memory is copied in directly) -> ``(output, metadata)``: the packed
    outputs and (files, 2) uint32 [status, 0], read-only NumPy arrays in
    pinned memory.  The files go through in pipelined groups (see _hostio),
    so the batch may exceed one device call's 2**28-byte totals; each file
    keeps the per-file bounds.  Statuses are returned, not raised.
    """
    sizes = _host_sizes(input_sizes, "input_sizes")
    expected = _host_sizes(expected_sizes, "expected_sizes")
    if sizes.size != expected.size:
        raise ValueError("input_sizes and expected_sizes must have matching lengths")
    packed = _host_packed(payload, sizes, "compressed payload")
    selected = _select_device(device)
    host, meta = _hostio.decode(_torch(), selected, packed, sizes, expected, _HOST_LIMITS)
    output = host.numpy()[:int(expected.sum())]
    output.flags.writeable = False
    meta = meta.view(np.uint32)
    meta.flags.writeable = False
    return output, meta


def compress_zlib_batch_padded_host(data, input_sizes, device=0, *, chunk_bytes=32768):
    """Host-buffer counterpart of compress_zlib_batch_padded.

    Packed files in host memory -> ``(slots, metadata)``: consecutive padded
    slots (the same layout as the device call's) and (files, 2) uint32
    [encoded_length, status], read-only NumPy arrays in pinned memory.
    Pipelined in groups like decompress_zlib_batch_checked_host; statuses
    are returned, not raised.
    """
    sizes = _host_sizes(input_sizes, "input_sizes")
    _check_chunk(chunk_bytes)
    packed = _host_packed(data, sizes, "input")
    capacities, chunks, blocks = _host_layouts(sizes, chunk_bytes)
    selected = _select_device(device)
    host, meta = _hostio.encode(_torch(), selected, packed, sizes, capacities, chunks,
                                chunk_bytes, _HOST_LIMITS)
    slots = host.numpy()[:int(capacities.sum())]
    slots.flags.writeable = False
    meta = meta.view(np.uint32)
    meta.flags.writeable = False
    return slots, meta


def compress_zlib_batch_packed_host(data, input_sizes, device=0, *, chunk_bytes=32768):
    """Host-buffer batch compression returning the streams back to back.

    No reference counterpart.  Packed files in host memory -> ``(streams,
    metadata)``: every file's stream in file order with nothing between them
    (a failed file takes no bytes) and (files, 2) uint32 [encoded_length,
    status], read-only NumPy arrays in pinned memory.  Pipelined like
    compress_zlib_batch_padded_host, but each group copies only its encoded
    bytes back (the device packs them with compress_zlib_batch_packed).
    """
    sizes = _host_sizes(input_sizes, "input_sizes")
    _check_chunk(chunk_bytes)
    packed = _host_packed(data, sizes, "input")
    capacities, chunks, blocks = _host_layouts(sizes, chunk_bytes)
    selected = _select_device(device)
    host, meta = _hostio.encode(_torch(), selected, packed, sizes, capacities, chunks,
                                chunk_bytes, _HOST_LIMITS, compact=True)
    streams = host.numpy()
    streams.flags.writeable = False
    meta = meta.view(np.uint32)
    meta.flags.writeable = False
    return streams, meta


def _host_layouts(sizes, chunk_bytes):
    """Vectorised _layout: (capacities, chunks, blocks) per file."""
    chunks = np.maximum(1, -(-sizes // chunk_bytes))
    full = max(1, -(-chunk_bytes // _STORED_MAX))
    tail = np.maximum(1, -(-(sizes - (chunks - 1) * chunk_bytes) // _STORED_MAX))
    stored = (chunks - 1) * full + tail
    blocks = (chunks - 1) * max(full, 2) + tail
    if blocks.max() > _MAX_BLOCKS or chunks.max() > _MAX_BLOCKS:
        raise ValueError("batch chunk count exceeds workspace limit")
    return sizes + 5 * stored + 6, chunks, blocks


def _first_failure(meta, column, operation):
    """Raise for the first nonzero status of a (files, 2) metadata array."""
    statuses = meta[:, column]
    bad = np.flatnonzero(statuses)
    if bad.size:
        i = int(bad[0])
        _check_value(int(statuses[i]), "%s file %d" % (operation, i))


def _host_files(inputs, label):
    """Host views of a batch's files, or None when some file is a CUDA tensor."""
    if not isinstance(inputs, (tuple, list)) or not inputs:
        raise ValueError(label + " must be a nonempty sequence of files")
    views = []
    for item in inputs:
        view = _hostio.as_host_array(item)
        if view is None:
            return None
        views.append(view)
    return views


def compress_zlib_batch_host(inputs, device=0, *, chunk_bytes=32768):
    """Return a tuple of bytes streams, one per file, through pinned memory.

    Host files go through compress_zlib_batch_padded_host (pipelined groups;
    the batch may exceed one device call's 2**28-byte totals, each file keeps
    the per-file bounds).  Files given as CUDA tensors take one device call.
    """
    views = _host_files(inputs, "inputs")
    if views is None:
        selected = _select_device(device)
        packed, sizes = _pack_batch(inputs, selected)
        capacities = _batch_capacities(sizes, chunk_bytes)
        output, metadata = compress_zlib_batch_padded(packed, sizes, selected,
                                                      chunk_bytes=chunk_bytes)
        lengths = _check_batch(metadata, "CUDA batch compression", True)[:, 0]
        host = _to_pinned_host(output)
        return tuple(view.tobytes() for view in _split_batch(host, capacities, lengths))
    sizes = np.fromiter((v.size for v in views), dtype=np.int64, count=len(views))
    if sizes.max() > _MAX_BYTES:
        raise ValueError("inputs exceeds size limit (2**28 bytes)")
    packed = _hostio.pack(views, _torch())
    streams, meta = compress_zlib_batch_packed_host(packed, sizes, device,
                                                    chunk_bytes=chunk_bytes)
    _first_failure(meta, 1, "CUDA batch compression")
    bounds = np.concatenate(([0], np.cumsum(meta[:, 0], dtype=np.int64))).tolist()
    return tuple(streams[bounds[i]:bounds[i + 1]].tobytes() for i in range(len(views)))


def decompress_zlib_batch_host(payloads, expected_sizes, device=0):
    """Return read-only NumPy views into one pinned host buffer.

    Every stream is decoded and checked independently on CUDA.  Host
    payloads go through decompress_zlib_batch_checked_host (pipelined groups;
    the batch may exceed one device call's 2**28-byte totals, each file keeps
    the per-file bounds).  Payloads given as CUDA tensors take one device call.
    """
    views = _host_files(payloads, "payloads")
    expected = _host_sizes(expected_sizes, "expected_sizes")
    if len(payloads) != expected.size:
        raise ValueError("input_sizes and expected_sizes must have matching lengths")
    if views is None:
        selected = _select_device(device)
        packed, sizes = _pack_batch(payloads, selected)
        expected = _batch_sizes(tuple(int(v) for v in expected), "expected_sizes")
        output, metadata = decompress_zlib_batch_checked(packed, sizes, expected, selected)
        _check_batch(metadata, "CUDA batch decompression")
        return _split_batch(_to_pinned_host(output), expected)
    sizes = np.fromiter((v.size for v in views), dtype=np.int64, count=len(views))
    if sizes.max() > _MAX_BYTES:
        raise ValueError("payloads exceeds size limit (2**28 bytes)")
    output, meta = decompress_zlib_batch_checked_host(_hostio.pack(views, _torch()), sizes,
                                                      expected, device)
    _first_failure(meta, 0, "CUDA batch decompression")
    bounds = np.concatenate(([0], np.cumsum(expected))).tolist()
    return tuple(output[bounds[i]:bounds[i + 1]] for i in range(len(views)))


def decompress_zlib_checked(payload, expected_bytes, device=0, *,
                            max_candidates=_MAX_CANDIDATES, max_blocks=_MAX_BLOCKS):
    """Return ``(output, [status, 0])`` without a host sync.

    Status zero validates the stream, the output extent and Adler-32; check it
    before using the output.  A failed output is all zero.  max_candidates
    and max_blocks are the reference handler's attributes (default 262144).
    """
    _validate_size(expected_bytes)
    size = _input_size(payload, "compressed payload", _MAX_STREAM_PAYLOAD)
    if isinstance(payload, (bytes, bytearray, memoryview)):
        _check_framing(payload, expected_bytes)
    elif size < 8:
        raise CodecError("truncated zlib payload")
    selected = _select_device(device)
    torch = _torch()
    lib = _native.library()
    raw = _device_input(payload, selected)
    with torch.cuda.device(selected):
        output = torch.empty(expected_bytes, dtype=torch.uint8, device=selected)
        metadata = torch.empty(2, dtype=torch.uint32, device=selected)
        _native.check(lib.cuda_zlib_decompress(_ptr(raw), size, int(max_candidates),
                                               int(max_blocks), _ptr(output), expected_bytes,
                                               metadata.data_ptr(), _stream(selected)),
                      "CUDA decompression")
    return output, metadata


def compress_zlib(data, device=0, *, chunk_bytes=32768, level=1):
    """Encode bytes/uint8 data to a completed, exact-length CUDA tensor."""
    output, metadata = compress_zlib_padded(data, device, chunk_bytes=chunk_bytes, level=level)
    length, status = (int(v) for v in metadata.cpu().numpy())
    _check_value(status, "CUDA compression")
    return output[:length]


_PIPE_MIN = 32 << 20     # host inputs at least this large are pipelined
_PIPE_PIECE = 16 << 20   # bytes per pipelined piece (rounded down to whole chunks)


def _host_view(data):
    """A host input as a flat uint8 CPU tensor (no copy), or None."""
    torch = _torch()
    if _is_tensor(data):
        return data.contiguous() if data.device.type == "cpu" else None
    if isinstance(data, (bytes, bytearray, memoryview, np.ndarray)):
        view = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data
        view = np.ascontiguousarray(view, dtype=np.uint8).reshape(-1)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore", UserWarning)  # read-only inputs are only read
            return torch.from_numpy(view)
    return None


def _compress_host_pipelined(source, size, selected, chunk_bytes):
    """compress_zlib_host for large host inputs, copies overlapping kernels.

    The input goes through in chunk-aligned pieces: a piece is staged into
    pinned memory by the host threads and copied in on a copy stream,
    encoded on the caller's stream by the range entry point while the next
    piece is staged, and its body copied out at its exact length as soon as
    its metadata is in.  Header, bodies and the combined Adler-32 trailer
    are byte-identical to the one-call stream.  (Inputs already in pinned
    memory take the one-call path: their copy-in is a single DMA and the
    pieces measured no faster.)
    """
    from . import sharding  # Adler-32 combination of the pieces
    torch = _torch()
    lib = _native.library()
    piece = max(chunk_bytes, _PIPE_PIECE // chunk_bytes * chunk_bytes)
    bounds = [(a, min(a + piece, size)) for a in range(0, size, piece)]
    pinned = source.is_pinned()
    with torch.cuda.device(selected):
        compute = torch.cuda.current_stream(selected)
        copy_in, copy_out = torch.cuda.Stream(selected), torch.cuda.Stream(selected)
        host_meta = torch.empty(3 * len(bounds), dtype=torch.int32, pin_memory=True)
        kept, done = [], []
        for k, (a, b) in enumerate(bounds):
            with torch.cuda.stream(copy_in):
                part = source[a:b]
                raw = (part.to(selected, non_blocking=True) if pinned else
                       _pinned_copy(part.numpy(), selected))
                ready = torch.cuda.Event()
                ready.record(copy_in)
            compute.wait_event(ready)
            capacity = _capacity(b - a, chunk_bytes)[0]
            output = torch.empty(capacity, dtype=torch.uint8, device=selected)
            meta = torch.zeros(3, dtype=torch.uint32, device=selected)
            _native.check(lib.cuda_zlib_compress_range(
                _ptr(raw), b - a, chunk_bytes, int(k == len(bounds) - 1), output.data_ptr(),
                capacity, meta.data_ptr(), compute.cuda_stream), "CUDA compression")
            finished = torch.cuda.Event()
            finished.record(compute)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(finished)
                host_meta[3 * k:3 * k + 3].copy_(meta.view(torch.int32), non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(copy_out)
            kept.append((raw, output, meta))
            done.append(arrived)
        host = torch.empty(_capacity(size, chunk_bytes)[0], dtype=torch.uint8, pin_memory=True)
        body_out = torch.cuda.Stream(selected)
        at, adlers = 2, []
        with torch.cuda.stream(body_out):
            for k, arrived in enumerate(done):
                arrived.synchronize()
                length, status, adler = (int(v) & 0xFFFFFFFF for v in host_meta[3 * k:3 * k + 3])
                if status:
                    body_out.synchronize()
                    _check_value(status, "CUDA compression")
                host[at:at + length].copy_(kept[k][1][:length], non_blocking=True)
                at += length
                adlers.append(adler)
            body_out.synchronize()
        compute.wait_stream(copy_in)  # the caller's stream orders after this call's work
    array = host.numpy()
    array[:2] = np.frombuffer(sharding.splice_header(), dtype=np.uint8)
    trailer = sharding.splice_trailer(sharding.combine_adlers(adlers, [b - a for a, b in bounds]))
    array[at:at + 4] = np.frombuffer(trailer, dtype=np.uint8)
    array = array[:at + 4]
    array.flags.writeable = False
    return array


def compress_zlib_host(data, device=0, *, chunk_bytes=32768, level=1) -> np.ndarray:
    """Encode to a completed, read-only NumPy uint8 array in pinned memory.

    The single-stream counterpart of compress_zlib_batch_host (the reference
    has no single-stream host variant): same encoding as compress_zlib, then
    one transfer of exactly the encoded length into pinned host memory.
    Pageable host inputs of at least _PIPE_MIN bytes go through in pieces, so
    that staging them into pinned memory and copying them in overlap the
    kernels; the stream is the same byte for byte.
    """
    _check_chunk(chunk_bytes)
    _check_level(level)
    size = _input_size(data, limit=_MAX_STREAM)
    if size >= _PIPE_MIN and level == 1:
        _, _, blocks = _layout(size, chunk_bytes)
        source = _host_view(data)
        if source is not None and not source.is_pinned() and blocks <= _MAX_BLOCKS:
            if source.dtype != _torch().uint8 or source.ndim != 1:
                raise TypeError("array input must be one-dimensional uint8")
            return _compress_host_pipelined(source, size, _select_device(device), chunk_bytes)
    output, metadata = compress_zlib_padded(data, device, chunk_bytes=chunk_bytes, level=level)
    length, status = (int(v) for v in metadata.cpu().numpy())
    _check_value(status, "CUDA compression")
    return _to_pinned_host(output[:length])


def decompress_zlib(payload, expected_bytes, device=0):
    """Decode to a completed CUDA tensor; every call checks Adler-32."""
    output, metadata = decompress_zlib_checked(payload, expected_bytes, device)
    _check_value(int(metadata.cpu().numpy()[0]), "CUDA decompression")
    return output


def decompress_zlib_host(payload, expected_bytes, device=0) -> np.ndarray:
    """Decode to a completed, read-only, contiguous NumPy uint8 array.

    Same decoding, limits and validation as decompress_zlib, then one transfer
    into pinned host memory that the returned array keeps alive.
    """
    output = decompress_zlib(payload, expected_bytes, device)
    return _to_pinned_host(output)
