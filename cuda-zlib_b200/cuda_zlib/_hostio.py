"""Pipelined host-to-host batch calls.

The batch calls with host buffers (decompress_zlib_batch_checked_host,
compress_zlib_batch_padded_host, and the per-file decompress_zlib_batch_host
and compress_zlib_batch_host built on them) take packed files in host
memory and return packed results in pinned host memory.  Done as one device
call, the copies and the kernels would run one after another.  Here the
files go through in groups (consecutive files within one batch call's
bounds: 2**28 bytes in and out, 262144 files or chunks) and each group
moves through four stages that overlap with the neighbouring groups':

  stage     host threads copy the group's bytes into a pinned buffer
            (skipped when the packed input already lives in pinned memory);
  copy in   one cudaMemcpyAsync on a copy stream;
  codec     the batch entry point on the caller's stream;
  copy out  results and metadata to pinned host memory on a third stream.

Two sets of buffers alternate between groups; events order each reuse after
the work that last read the buffer.  Because the groups are separate device
calls, a batch may exceed one call's 2**28-byte totals; every file keeps the
per-file bounds.  All per-file bookkeeping is vectorised (numpy), so a batch
of many small files costs no per-file Python work.
"""
import ctypes
import os
import warnings
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import _native

_GROUP_MIN = 32 << 20   # a group holds at least this many bytes (unless the batch is smaller)
_TAIL_FILES = 2048      # decode groups hold at least this many of the batch's largest files
_STAGE_PIECE = 8 << 20  # bytes per host staging task
_STAGE_THREADS = max(1, min(16, os.cpu_count() or 1))
_pool = None


def _stage_pool():
    global _pool
    if _pool is None:
        _pool = ThreadPoolExecutor(max_workers=_STAGE_THREADS, thread_name_prefix="cuda_zlib_io")
    return _pool


def as_host_array(data):
    """A flat uint8 host array over `data` without copying (bytes-like,
    NumPy array or CPU tensor); None for a CUDA tensor."""
    if isinstance(data, (bytes, bytearray, memoryview)):
        return np.frombuffer(data, dtype=np.uint8)
    if isinstance(data, np.ndarray):
        if data.dtype != np.uint8 or data.ndim != 1:
            raise TypeError("array input must be one-dimensional uint8")
        return np.ascontiguousarray(data)
    if type(data).__module__.startswith("torch") and hasattr(data, "device"):
        if data.device.type != "cpu":
            return None
        if data.dtype.is_floating_point or data.element_size() != 1 or data.ndim != 1:
            raise TypeError("array input must be one-dimensional uint8")
        return data.contiguous().numpy().view(np.uint8)
    raise TypeError("input must be bytes or a one-dimensional uint8 array or tensor")


def _tensor(torch, array):
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)  # read-only arrays are only read
        return torch.from_numpy(array)


def plan_groups(in_sizes, out_sizes, units, limits, floor=0):
    """Boundaries [a, b) of consecutive files whose totals stay within
    `limits` = (units, input bytes, output bytes) of one call; groups are cut
    at about a quarter of the batch (at least _GROUP_MIN output bytes) so
    that a large batch has stages to overlap; the first two groups are a
    quarter and a half of that.  No group is cut below `floor` output bytes
    (the batch decoder gives each file one warp, so a group's time has a tail
    set by its largest file; a group must be large enough to hide it)."""
    n = len(in_sizes)
    if n == 0:
        return []
    cin = np.concatenate(([0], np.cumsum(in_sizes, dtype=np.int64)))
    cout = np.concatenate(([0], np.cumsum(out_sizes, dtype=np.int64)))
    cunit = np.concatenate(([0], np.cumsum(units, dtype=np.int64)))
    target = min(limits[2], max(_GROUP_MIN, -(-int(cout[-1]) // 4)))
    groups, a = [], 0
    while a < n:
        # The first two groups take a quarter and a half of the target, so
        # the kernels start after a short first copy.
        want = max(1, target >> max(0, 2 - len(groups)), min(int(floor), limits[2]))
        # Largest b with every total within its limit (at least one file).
        b = min(int(np.searchsorted(cin, cin[a] + limits[1], "right")) - 1,
                int(np.searchsorted(cout, cout[a] + limits[2], "right")) - 1,
                int(np.searchsorted(cunit, cunit[a] + limits[0], "right")) - 1,
                int(np.searchsorted(cout, cout[a] + want, "left")))
        b = max(a + 1, min(b, n))
        groups.append((a, b))
        a = b
    return groups


class _Source:
    """Each group's input as a pinned tensor: slices of the packed input when
    it is pinned, else copies into two alternating pinned buffers."""

    def __init__(self, torch, packed, groups, offsets):
        self.packed, self.offsets = packed, offsets
        tensor = _tensor(torch, packed)
        self.tensor = tensor if packed.size and tensor.is_pinned() else None
        need = max((int(offsets[b] - offsets[a]) for a, b in groups), default=0)
        self.buffers = [] if self.tensor is not None else [
            torch.empty(max(1, need), dtype=torch.uint8, pin_memory=True)
            for _ in range(2 if len(groups) > 1 else 1)]
        self.released = [None, None]

    def get(self, k, a, b):
        lo, hi = int(self.offsets[a]), int(self.offsets[b])
        if self.tensor is not None:
            return self.tensor[lo:hi]
        j = k % len(self.buffers)
        if self.released[j] is not None:
            self.released[j].synchronize()  # the copy of group k - 2 has left this buffer
        buf = self.buffers[j][:hi - lo]
        host, src = buf.numpy(), self.packed[lo:hi]
        pieces = range(0, hi - lo, _STAGE_PIECE)
        if len(pieces) > 1:
            def fill(s):
                host[s:s + _STAGE_PIECE] = src[s:s + _STAGE_PIECE]
            for future in [_stage_pool().submit(fill, s) for s in pieces]:
                future.result()
        elif hi > lo:
            host[:] = src
        return buf

    def mark(self, k, event):
        if self.buffers:
            self.released[k % len(self.buffers)] = event


def _i64(values):
    """A ctypes int64 pointer over a contiguous int64 NumPy slice (no copy)."""
    return values.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))


def run(torch, device, packed, in_sizes, out_sizes, units, limits, call, compact=False,
        floor=0):
    """Push the packed files through stage -> copy in -> call -> copy out.

    call(a, b, dev_in, in_bytes, dev_out, out_bytes, dev_meta, stream) issues
    the batch call of files [a, b).  Returns (pinned host output holding every
    group's dev_out, int32 metadata of shape (files, 2)).

    compact: the call packs its files' streams at the front of dev_out
    (metadata [length, status]); each group's copy out then takes only the
    sum of its lengths, read from its metadata.  The host waits for a
    group's metadata only after issuing the next group's call, so the GPU
    stays busy; the returned output holds the streams back to back.
    """
    in_sizes = np.asarray(in_sizes, dtype=np.int64)
    out_sizes = np.asarray(out_sizes, dtype=np.int64)
    groups = plan_groups(in_sizes, out_sizes, units, limits, floor)
    in_off = np.concatenate(([0], np.cumsum(in_sizes)))
    out_off = np.concatenate(([0], np.cumsum(out_sizes)))
    files = len(in_sizes)
    host_out = torch.empty(max(1, int(out_off[-1])), dtype=torch.uint8, pin_memory=True)
    host_meta = torch.empty((max(1, files), 2), dtype=torch.int32, pin_memory=True)
    if not groups:
        return host_out, host_meta.numpy()[:0]
    source = _Source(torch, packed, groups, in_off)
    with torch.cuda.device(device):
        compute = torch.cuda.current_stream(device)
        copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
        # Compact mode: metadata goes out on its own stream, so that a group's
        # stream copy, issued once the host has read that group's metadata,
        # never queues behind the next group's metadata copy (which waits for
        # the next group's kernels).
        meta_out = torch.cuda.Stream(device) if compact else copy_out
        sets = 2 if len(groups) > 1 else 1
        most_in = max(int(in_off[b] - in_off[a]) for a, b in groups)
        most_out = max(int(out_off[b] - out_off[a]) for a, b in groups)
        most_files = max(b - a for a, b in groups)
        dev_in = [torch.empty(max(1, most_in), dtype=torch.uint8, device=device)
                  for _ in range(sets)]
        dev_out = [torch.empty(max(1, most_out), dtype=torch.uint8, device=device)
                   for _ in range(sets)]
        dev_meta = [torch.empty((most_files, 2), dtype=torch.int32, device=device)
                    for _ in range(sets)]
        consumed = [None] * sets   # the call that last read dev_in[j]
        drained = [None] * sets    # the copy out that last read dev_out[j]
        waiting = None             # compact: (j, a, b, metadata event) of the last group
        written = 0

        def copy_compact(j, a, b, meta_ready):
            nonlocal written
            meta_ready.synchronize()
            meta = host_meta.numpy()[a:b]
            n = int(meta[:, 0][meta[:, 1] == 0].astype(np.int64).sum())
            with torch.cuda.stream(copy_out):
                if n:
                    host_out[written:written + n].copy_(dev_out[j][:n], non_blocking=True)
                finished = torch.cuda.Event()
                finished.record(copy_out)
            drained[j] = finished
            written += n

        for k, (a, b) in enumerate(groups):
            j = k % sets
            src = source.get(k, a, b)
            n_in, n_out = int(in_off[b] - in_off[a]), int(out_off[b] - out_off[a])
            with torch.cuda.stream(copy_in):
                if consumed[j] is not None:
                    copy_in.wait_event(consumed[j])
                if n_in:
                    dev_in[j][:n_in].copy_(src, non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(copy_in)
            source.mark(k, arrived)
            compute.wait_event(arrived)
            if drained[j] is not None:
                compute.wait_event(drained[j])
            call(a, b, dev_in[j], n_in, dev_out[j], n_out, dev_meta[j], compute)
            done = torch.cuda.Event()
            done.record(compute)
            consumed[j] = done
            with torch.cuda.stream(meta_out):
                meta_out.wait_event(done)
                if n_out and not compact:
                    host_out[int(out_off[a]):int(out_off[b])].copy_(dev_out[j][:n_out],
                                                                    non_blocking=True)
                host_meta[a:b].copy_(dev_meta[j][:b - a], non_blocking=True)
                finished = torch.cuda.Event()
                finished.record(meta_out)
            if not compact:
                drained[j] = finished
                continue
            if waiting is not None:
                copy_compact(*waiting)
            waiting = (j, a, b, finished)
        if waiting is not None:
            copy_compact(*waiting)
        copy_out.synchronize()
        meta_out.synchronize()
        compute.wait_stream(copy_in)
    if compact:
        return host_out[:written], host_meta.numpy()[:files]
    return host_out, host_meta.numpy()[:files]


def decode(torch, device, packed, in_sizes, out_sizes, limits):
    """Packed host streams -> (pinned packed outputs, int32 [status, 0] pairs)."""
    lib = _native.library()
    ins = np.ascontiguousarray(in_sizes, dtype=np.int64)
    outs = np.ascontiguousarray(out_sizes, dtype=np.int64)

    def call(a, b, dev_in, n_in, dev_out, n_out, dev_meta, stream):
        _native.check(lib.cuda_zlib_decompress_batch(
            dev_in.data_ptr(), n_in, _i64(ins[a:b]), _i64(outs[a:b]), b - a, None,
            dev_out.data_ptr(), n_out, dev_meta.data_ptr(), stream.cuda_stream),
            "CUDA batch decompression")

    # One warp decodes a file: groups of at least 2048 largest files keep a
    # group's tail (its largest file) small against its throughput time.
    floor = _TAIL_FILES * int(outs.max()) if outs.size else 0
    return run(torch, device, packed, ins, outs, np.ones(ins.size, np.int64), limits, call,
               floor=floor)


def encode(torch, device, packed, in_sizes, capacities, chunks, chunk_bytes, limits,
           compact=False):
    """Packed host files -> (pinned padded slots, int32 [length, status] pairs);
    compact: the streams back to back instead of padded slots."""
    lib = _native.library()
    ins = np.ascontiguousarray(in_sizes, dtype=np.int64)
    entry = lib.cuda_zlib_compress_batch_packed if compact else lib.cuda_zlib_compress_batch

    def call(a, b, dev_in, n_in, dev_out, n_out, dev_meta, stream):
        _native.check(entry(
            dev_in.data_ptr(), n_in, _i64(ins[a:b]), b - a, chunk_bytes,
            dev_out.data_ptr(), n_out, dev_meta.data_ptr(), stream.cuda_stream),
            "CUDA batch compression")

    return run(torch, device, packed, ins, capacities, chunks, limits, call, compact)


def pack(views, torch):
    """The files back to back in one array: the owner's span when they
    already lie back to back in one array (e.g. slices of one buffer), else
    a pinned concatenation."""
    if not views:
        return np.empty(0, dtype=np.uint8)
    sizes = np.fromiter((v.size for v in views), dtype=np.int64, count=len(views))
    addresses = np.fromiter((v.__array_interface__["data"][0] for v in views), dtype=np.uint64,
                            count=len(views))
    owner = views[0]
    while isinstance(owner.base, np.ndarray):
        owner = owner.base
    start = owner.__array_interface__["data"][0]
    nonempty = sizes > 0
    expected = addresses[0] + np.concatenate(([0], np.cumsum(sizes[:-1]))).astype(np.uint64)
    if (owner.dtype == np.uint8 and owner.ndim == 1 and owner.flags.c_contiguous and
            addresses[0] >= start and
            int(addresses[0]) + int(sizes.sum()) <= start + owner.size and
            np.array_equal(addresses[nonempty], expected[nonempty])):
        first = int(addresses[0]) - start
        return owner[first:first + int(sizes.sum())]
    out = torch.empty(max(1, int(sizes.sum())), dtype=torch.uint8, pin_memory=True).numpy()
    out = out[:int(sizes.sum())]
    if len(views):
        np.concatenate(views, out=out)
    return out
