"""The XLA FFI handlers (cuda-zlib_b200/ffi/cuda_zlib_xla.cc).

CPU: the handler library builds (against the stand-in FFI header here, where
jaxlib is absent; the build's static_assert checks every handler against its
binding) and exports the reference's four handler names
(src/cuda_zlib/native/codec_ffi.cu:1144-1182); a malformed metadata buffer is
InvalidArgument before any CUDA work.  GPU: each handler, called through the
stand-in's call frame, returns what the Python API returns for the same input.
"""
import ctypes
import importlib.util
import os
import zlib

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HANDLERS = ("CudaZlibCompress", "CudaZlibDecompress", "CudaZlibCompressBatch",
            "CudaZlibDecompressBatch")


class Buffer(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("rank", ctypes.c_int64),
                ("dims", ctypes.POINTER(ctypes.c_int64))]


class Span(ctypes.Structure):
    _fields_ = [("data", ctypes.POINTER(ctypes.c_int64)), ("size", ctypes.c_int64)]


class Frame(ctypes.Structure):
    _fields_ = [("stream", ctypes.c_void_p), ("num_attrs", ctypes.c_int64),
                ("attrs", ctypes.POINTER(ctypes.c_void_p)), ("num_args", ctypes.c_int64),
                ("args", ctypes.POINTER(Buffer)), ("num_rets", ctypes.c_int64),
                ("rets", ctypes.POINTER(Buffer))]


class Error(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int), ("message", ctypes.c_char * 256)]


@pytest.fixture(scope="module")
def handlers():
    from cuda_zlib import _native
    _native.library()  # the package configures the codec library before any handler runs
    spec = importlib.util.spec_from_file_location(
        "cuda_zlib_b200_build", os.path.join(ROOT, "cuda-zlib_b200", "build.py"))
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    path = build.build_xla()
    lib = ctypes.CDLL(path)
    for name in HANDLERS:
        getattr(lib, name).argtypes = [ctypes.POINTER(Frame)]
        getattr(lib, name).restype = ctypes.POINTER(Error)
    return lib


class Call:
    """A stand-in call frame; keeps every ctypes object it points to alive."""

    def __init__(self, stream, attrs, args, rets):
        self.keep = []
        attr_ptrs = []
        for value in attrs:
            if isinstance(value, (list, tuple)):
                data = (ctypes.c_int64 * max(1, len(value)))(*value)
                span = Span(ctypes.cast(data, ctypes.POINTER(ctypes.c_int64)), len(value))
                self.keep += [data, span]
                attr_ptrs.append(ctypes.cast(ctypes.pointer(span), ctypes.c_void_p))
            else:
                scalar = ctypes.c_int64(value)
                self.keep.append(scalar)
                attr_ptrs.append(ctypes.cast(ctypes.pointer(scalar), ctypes.c_void_p))
        self.attrs = (ctypes.c_void_p * max(1, len(attr_ptrs)))(*attr_ptrs)
        self.args = self._buffers(args)
        self.rets = self._buffers(rets)
        self.frame = Frame(stream, len(attrs), self.attrs, len(args), self.args, len(rets),
                           self.rets)

    def _buffers(self, items):
        array = (Buffer * max(1, len(items)))()
        for i, (pointer, shape) in enumerate(items):
            dims = (ctypes.c_int64 * max(1, len(shape)))(*shape)
            self.keep.append(dims)
            array[i] = Buffer(pointer, len(shape), dims)
        return array

    def __call__(self, fn):
        error = fn(ctypes.byref(self.frame))
        return (0, "") if not error else (error.contents.code, error.contents.message.decode())


def test_handler_library_exports_the_reference_handler_names(handlers):
    for name in HANDLERS:
        assert hasattr(handlers, name)


def test_malformed_metadata_is_invalid_argument_before_cuda(handlers):
    # Metadata of shape (3,) instead of (2,): rejected before any device call.
    call = Call(None, [32768], [(None, (0,))], [(None, (11,)), (None, (3,))])
    code, message = call(handlers.CudaZlibCompress)
    assert code == 3 and "shape (2,)" in message
    call = Call(None, [32768, [1, 2]], [(None, (3,))], [(None, (30,)), (None, (2, 2, 1))])
    code, message = call(handlers.CudaZlibCompressBatch)
    assert code == 3 and "(files, 2)" in message


@pytest.mark.gpu
def test_handlers_match_the_python_api_on_the_gpu(handlers):
    import torch
    import cuda_zlib as codec
    device = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(device)
    rng = np.random.default_rng(7)
    raw = np.concatenate([rng.integers(0, 8, 200000, dtype=np.uint8),
                          np.frombuffer(b"xla ffi handler " * 5000, dtype=np.uint8)])
    src = torch.from_numpy(raw).to(device)
    capacity = raw.size + 5 * -(-raw.size // 32768) + 6
    out = torch.zeros(capacity, dtype=torch.uint8, device=device)
    meta = torch.zeros(2, dtype=torch.int32, device=device)
    code, _ = Call(stream.cuda_stream, [32768], [(src.data_ptr(), (raw.size,))],
                   [(out.data_ptr(), (capacity,)), (meta.data_ptr(), (2,))])(
        handlers.CudaZlibCompress)
    torch.cuda.synchronize()
    length, status = (int(v) for v in meta.cpu())
    assert code == 0 and status == 0
    want, want_meta = codec.compress_zlib_padded(src, device)
    assert out.cpu().numpy().tobytes() == want.cpu().numpy().tobytes()
    stream_bytes = out[:length].cpu().numpy().tobytes()
    assert zlib.decompress(stream_bytes) == raw.tobytes()

    payload = torch.from_numpy(np.frombuffer(stream_bytes, dtype=np.uint8).copy()).to(device)
    dec = torch.zeros(raw.size, dtype=torch.uint8, device=device)
    code, _ = Call(stream.cuda_stream, [262144, 262144], [(payload.data_ptr(), (length,))],
                   [(dec.data_ptr(), (raw.size,)), (meta.data_ptr(), (2,))])(
        handlers.CudaZlibDecompress)
    torch.cuda.synchronize()
    assert code == 0 and [int(v) for v in meta.cpu()] == [0, 0]
    assert torch.equal(dec, src)

    files = [raw[:1000], raw[1000:1000], raw[1000:150000], raw[150000:]]
    sizes = [f.size for f in files]
    caps = [n + 5 * max(1, -(-n // 32768)) + 6 for n in sizes]
    slots = torch.zeros(sum(caps), dtype=torch.uint8, device=device)
    bmeta = torch.zeros((len(files), 2), dtype=torch.int32, device=device)
    code, _ = Call(stream.cuda_stream, [32768, sizes], [(src.data_ptr(), (raw.size,))],
                   [(slots.data_ptr(), (sum(caps),)), (bmeta.data_ptr(), (len(files), 2))])(
        handlers.CudaZlibCompressBatch)
    torch.cuda.synchronize()
    assert code == 0
    want, want_meta = codec.compress_zlib_batch_padded(src, sizes, device)
    assert slots.cpu().numpy().tobytes() == want.cpu().numpy().tobytes()
    assert np.array_equal(bmeta.cpu().numpy().view(np.uint32), want_meta.cpu().numpy())

    # Decode the padded slots directly with the encoded lengths (the
    # encoded-metadata argument), then with an empty one and packed streams.
    outs = torch.zeros(raw.size, dtype=torch.uint8, device=device)
    dmeta = torch.full((len(files), 2), 99, dtype=torch.int32, device=device)
    code, _ = Call(stream.cuda_stream, [caps, sizes],
                   [(slots.data_ptr(), (sum(caps),)), (bmeta.data_ptr(), (len(files), 2))],
                   [(outs.data_ptr(), (raw.size,)), (dmeta.data_ptr(), (len(files), 2))])(
        handlers.CudaZlibDecompressBatch)
    torch.cuda.synchronize()
    assert code == 0 and not dmeta.cpu().numpy().any()
    assert torch.equal(outs, src)
    host = slots.cpu().numpy()
    lengths = bmeta.cpu().numpy()[:, 0]
    starts = np.concatenate(([0], np.cumsum(caps)))
    packed = b"".join(host[starts[i]:starts[i] + lengths[i]].tobytes() for i in range(len(files)))
    z = torch.from_numpy(np.frombuffer(packed, dtype=np.uint8).copy()).to(device)
    outs.zero_()
    code, _ = Call(stream.cuda_stream, [[int(n) for n in lengths], sizes],
                   [(z.data_ptr(), (len(packed),)), (None, (0,))],
                   [(outs.data_ptr(), (raw.size,)), (dmeta.data_ptr(), (len(files), 2))])(
        handlers.CudaZlibDecompressBatch)
    torch.cuda.synchronize()
    assert code == 0 and not dmeta.cpu().numpy().any()
    assert torch.equal(outs, src)
