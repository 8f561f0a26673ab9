"""Pipelined host-to-host batch calls.

decompress_zlib_batch_host and compress_zlib_batch_host take files in host
memory and return results in pinned host memory.  Done as one device call,
the copies and the kernels run one after another.  Here the files go
through in groups (consecutive files within the batch call's bounds, 2**28
bytes and 262144 files or chunks per call) and each group moves through
four stages that overlap with the neighbouring groups' stages:

  stage     host threads copy the group's files into a pinned buffer
            (skipped when the files already lie back to back in pinned
            memory, e.g. views of one page-locked array);
  copy in   one cudaMemcpyAsync on a copy stream;
  codec     the batch entry point on the caller's stream;
  copy out  results and metadata to one pinned host buffer on a third stream.

Two sets of buffers alternate between groups; events order each reuse after
the work that last read the buffer.  Because the groups are separate device
calls, a batch may exceed one call's 2**28-byte totals (the reference's
host calls stop there); every file keeps the per-file bounds.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import _native

_GROUP_MIN = 32 << 20   # a group holds at least this many bytes (unless the batch is smaller)
_STAGE_THREADS = max(1, min(16, os.cpu_count() or 1))
_pool = None


def _stage_pool():
    global _pool
    if _pool is None:
        _pool = ThreadPoolExecutor(max_workers=_STAGE_THREADS, thread_name_prefix="cuda_zlib_io")
    return _pool


def host_views(items):
    """Each item as a flat uint8 NumPy array without copying, or None if some
    item is not a host buffer (e.g. a CUDA tensor)."""
    views = []
    for item in items:
        if isinstance(item, (bytes, bytearray, memoryview)):
            views.append(np.frombuffer(item, dtype=np.uint8))
        elif isinstance(item, np.ndarray):
            if item.dtype != np.uint8 or item.ndim != 1:
                raise TypeError("array input must be one-dimensional uint8")
            views.append(np.ascontiguousarray(item))
        elif type(item).__module__.startswith("torch") and hasattr(item, "device"):
            if item.device.type != "cpu":
                return None
            if item.dtype.is_floating_point or item.element_size() != 1 or item.ndim != 1:
                raise TypeError("array input must be one-dimensional uint8")
            views.append(item.contiguous().numpy().view(np.uint8))
        else:
            raise TypeError("input must be bytes or a one-dimensional uint8 array or tensor")
    return views


def _address(view):
    return view.__array_interface__["data"][0]


def _packed_span(views):
    """(owner array, byte offset) when the views lie back to back in one
    array's memory (e.g. slices of one packed buffer), else None."""
    if not views:
        return None
    owner = views[0]
    while isinstance(owner.base, np.ndarray):
        owner = owner.base
    if owner.dtype != np.uint8 or owner.ndim != 1 or not owner.flags.c_contiguous:
        return None
    start = _address(owner)
    at = _address(views[0])
    if at < start:
        return None
    for view in views:
        if view.size and _address(view) != at:
            return None
        at += view.size
    if at > start + owner.size:
        return None
    return owner, _address(views[0]) - start


def plan_groups(in_sizes, out_sizes, units, limits):
    """Consecutive groups [a, b) of files whose totals stay within `limits`
    = (units, input bytes, output bytes) of one call, cut into at least four
    groups of at least _GROUP_MIN output bytes when the batch is large
    enough to overlap its stages."""
    total = sum(out_sizes)
    target = min(limits[2], max(_GROUP_MIN, -(-total // 4)))
    groups, a = [], 0
    n = len(in_sizes)
    while a < n:
        b, used_u, used_in, used_out = a, 0, 0, 0
        while b < n:
            u, i, o = units[b], in_sizes[b], out_sizes[b]
            if b > a and (used_u + u > limits[0] or used_in + i > limits[1] or
                          used_out + o > limits[2] or used_out >= target):
                break
            used_u, used_in, used_out = used_u + u, used_in + i, used_out + o
            b += 1
        groups.append((a, b))
        a = b
    return groups


class _Staging:
    """Where each group's input comes from: views of pinned memory as they
    are, else copies into two alternating pinned buffers by host threads."""

    def __init__(self, torch, views, groups, offsets):
        self.torch, self.views, self.offsets = torch, views, offsets
        span = _packed_span(views)
        self.owner = None
        if span is not None:
            owner, base = span
            import warnings
            with warnings.catch_warnings():
                warnings.simplefilter("ignore", UserWarning)  # read-only owners are only read
                tensor = torch.from_numpy(owner)
            self.owner, self.base, self.pinned = tensor, base, tensor.is_pinned()
        need = max((offsets[b] - offsets[a] for a, b in groups), default=0)
        self.buffers = []
        if self.owner is None or not self.pinned:
            self.buffers = [torch.empty(max(1, need), dtype=torch.uint8, pin_memory=True)
                            for _ in range(2 if len(groups) > 1 else 1)]
        self.released = [None] * 2  # event after the last copy out of buffer j

    def source(self, k, a, b):
        """Pinned host tensor holding files [a, b) back to back."""
        lo, hi = self.offsets[a], self.offsets[b]
        if self.owner is not None and self.pinned:
            return self.owner[self.base + lo:self.base + hi]
        j = k % len(self.buffers)
        if self.released[j] is not None:
            self.released[j].synchronize()
        buf = self.buffers[j][:hi - lo]
        host = buf.numpy()
        if self.owner is not None:
            packed = self.owner.numpy()[self.base + lo:self.base + hi]
            pieces = [(s, min(s + (8 << 20), hi - lo)) for s in range(0, hi - lo, 8 << 20)]

            def fill(piece):
                host[piece[0]:piece[1]] = packed[piece[0]:piece[1]]
        else:
            per = max(1, -(-(b - a) // _STAGE_THREADS))
            pieces = [(i, min(i + per, b)) for i in range(a, b, per)]

            def fill(piece):
                for i in range(piece[0], piece[1]):
                    at = self.offsets[i] - lo
                    host[at:at + self.views[i].size] = self.views[i]
        if hi - lo >= (4 << 20) and len(pieces) > 1:
            for future in [_stage_pool().submit(fill, p) for p in pieces]:
                future.result()
        else:
            for p in pieces:
                fill(p)
        return buf

    def mark(self, k, event):
        if self.buffers:
            self.released[k % len(self.buffers)] = event


def _offsets(sizes):
    offsets = [0]
    for size in sizes:
        offsets.append(offsets[-1] + size)
    return offsets


def run_groups(torch, device, views, groups, in_offsets, out_offsets, dev_out_sizes, call,
               host_out, meta_words):
    """Push every group through stage -> copy in -> call -> copy out.

    call(k, a, b, dev_in, dev_out, dev_meta, stream) issues the codec call of
    group k; its results are dev_out[:out_offsets[b] - out_offsets[a]] and
    dev_meta (2 u32 per file).  Results land in host_out at out_offsets[a]
    and host metadata (returned, int32 pairs) at 2 a.
    """
    staging = _Staging(torch, views, groups, in_offsets)
    host_meta = torch.empty(max(1, meta_words), dtype=torch.int32, pin_memory=True)
    with torch.cuda.device(device):
        compute = torch.cuda.current_stream(device)
        copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
        sets = 2 if len(groups) > 1 else 1
        max_in = max(in_offsets[b] - in_offsets[a] for a, b in groups)
        max_files = max(b - a for a, b in groups)
        dev_in = [torch.empty(max(1, max_in), dtype=torch.uint8, device=device)
                  for _ in range(sets)]
        dev_out = [torch.empty(max(1, dev_out_sizes), dtype=torch.uint8, device=device)
                   for _ in range(sets)]
        dev_meta = [torch.empty((max_files, 2), dtype=torch.uint32, device=device)
                    for _ in range(sets)]
        consumed = [None] * sets   # the call that last read dev_in[j]
        drained = [None] * sets    # the copy out that last read dev_out[j]
        for k, (a, b) in enumerate(groups):
            j = k % sets
            source = staging.source(k, a, b)
            size_in = in_offsets[b] - in_offsets[a]
            with torch.cuda.stream(copy_in):
                if consumed[j] is not None:
                    copy_in.wait_event(consumed[j])
                if size_in:
                    dev_in[j][:size_in].copy_(source, non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(copy_in)
            staging.mark(k, arrived)
            compute.wait_event(arrived)
            if drained[j] is not None:
                compute.wait_event(drained[j])
            call(k, a, b, dev_in[j], dev_out[j], dev_meta[j], compute)
            done = torch.cuda.Event()
            done.record(compute)
            consumed[j] = done
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done)
                size_out = out_offsets[b] - out_offsets[a]
                if size_out:
                    host_out[out_offsets[a]:out_offsets[b]].copy_(dev_out[j][:size_out],
                                                                  non_blocking=True)
                host_meta[2 * a:2 * b].copy_(dev_meta[j][:b - a].view(torch.int32).reshape(-1),
                                             non_blocking=True)
                finished = torch.cuda.Event()
                finished.record(copy_out)
            drained[j] = finished
        copy_out.synchronize()
        compute.wait_stream(copy_in)
    return host_meta.numpy()


def decode(views, expected, device, torch, limits):
    """decompress_zlib_batch_host over host views: (pinned output, int32 meta)."""
    lib = _native.library()
    in_sizes = [v.size for v in views]
    groups = plan_groups(in_sizes, expected, [1] * len(views), limits)
    in_offsets, out_offsets = _offsets(in_sizes), _offsets(expected)
    host_out = torch.empty(max(1, out_offsets[-1]), dtype=torch.uint8, pin_memory=True)
    import ctypes

    def call(k, a, b, dev_in, dev_out, dev_meta, stream):
        sizes = (ctypes.c_int64 * (b - a))(*in_sizes[a:b])
        outs = (ctypes.c_int64 * (b - a))(*expected[a:b])
        _native.check(lib.cuda_zlib_decompress_batch(
            dev_in.data_ptr(), in_offsets[b] - in_offsets[a], sizes, outs, b - a, None,
            dev_out.data_ptr(), out_offsets[b] - out_offsets[a], dev_meta.data_ptr(),
            stream.cuda_stream), "CUDA batch decompression")

    most_out = max(out_offsets[b] - out_offsets[a] for a, b in groups)
    meta = run_groups(torch, device, views, groups, in_offsets, out_offsets, most_out, call,
                      host_out, 2 * len(views))
    return host_out, meta


def encode(views, capacities, chunk_units, chunk_bytes, device, torch, limits):
    """compress_zlib_batch_host over host views: (pinned slots, int32 meta)."""
    lib = _native.library()
    in_sizes = [v.size for v in views]
    groups = plan_groups(in_sizes, capacities, chunk_units, limits)
    in_offsets, out_offsets = _offsets(in_sizes), _offsets(capacities)
    host_out = torch.empty(max(1, out_offsets[-1]), dtype=torch.uint8, pin_memory=True)
    import ctypes

    def call(k, a, b, dev_in, dev_out, dev_meta, stream):
        sizes = (ctypes.c_int64 * (b - a))(*in_sizes[a:b])
        _native.check(lib.cuda_zlib_compress_batch(
            dev_in.data_ptr(), in_offsets[b] - in_offsets[a], sizes, b - a, chunk_bytes,
            dev_out.data_ptr(), out_offsets[b] - out_offsets[a], dev_meta.data_ptr(),
            stream.cuda_stream), "CUDA batch compression")

    most_out = max(out_offsets[b] - out_offsets[a] for a, b in groups)
    meta = run_groups(torch, device, views, groups, in_offsets, out_offsets, most_out, call,
                      host_out, 2 * len(views))
    return host_out, meta, out_offsets
