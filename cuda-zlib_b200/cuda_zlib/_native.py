"""ctypes binding of libcuda_zlib_b200.so (include/cuda_zlib_b200.h).

The library is built in-tree by cuda-zlib_b200/build.py.  If it is missing,
loading raises BackendUnavailable: there is no other implementation to fall
back to.  Workspace retention follows the reference's environment variable
(src/cuda_zlib/_ffi.py:21-40).
"""
import ctypes
import os
import threading

from ._errors import BackendUnavailable

LIBRARY = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libcuda_zlib_b200.so")
_LOCK = threading.Lock()
_library = None

_u8p = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)


def _workspace_retention():
    value = os.environ.get("CUDA_ZLIB_WORKSPACE_RETENTION_BYTES", str(1 << 30))
    if not value.isascii() or not value.isdecimal() or int(value) >= 1 << 64:
        raise ValueError("CUDA_ZLIB_WORKSPACE_RETENTION_BYTES must be an integer in [0, 2**64-1]")
    return int(value)


def _check_pool_error(code):
    if code:
        raise BackendUnavailable(f"native CUDA workspace pool operation failed (CUDA error {code})")


def _configure(library):
    library.cuda_zlib_compress.argtypes = [_u8p, ctypes.c_uint64, ctypes.c_int64, _u8p,
                                           ctypes.c_uint64, _u8p, ctypes.c_void_p]
    library.cuda_zlib_decompress.argtypes = [_u8p, ctypes.c_uint64, ctypes.c_int64,
                                             ctypes.c_int64, _u8p, ctypes.c_uint64, _u8p,
                                             ctypes.c_void_p]
    library.cuda_zlib_compress_batch.argtypes = [_u8p, ctypes.c_uint64, _i64p, ctypes.c_uint64,
                                                 ctypes.c_int64, _u8p, ctypes.c_uint64, _u8p,
                                                 ctypes.c_void_p]
    library.cuda_zlib_compress_batch_packed.argtypes = [_u8p, ctypes.c_uint64, _i64p,
                                                        ctypes.c_uint64, ctypes.c_int64, _u8p,
                                                        ctypes.c_uint64, _u8p, ctypes.c_void_p]
    library.cuda_zlib_decompress_batch.argtypes = [_u8p, ctypes.c_uint64, _i64p, _i64p,
                                                   ctypes.c_uint64, _u8p, _u8p, ctypes.c_uint64,
                                                   _u8p, ctypes.c_void_p]
    library.cuda_zlib_compress_range.argtypes = [_u8p, ctypes.c_uint64, ctypes.c_int64,
                                                 ctypes.c_int32, _u8p, ctypes.c_uint64, _u8p,
                                                 ctypes.c_void_p]
    library.cuda_zlib_compress_format.argtypes = [_u8p, ctypes.c_uint64, ctypes.c_int64,
                                                  ctypes.c_int32, ctypes.c_int32, _u8p,
                                                  ctypes.c_uint64, _u8p, ctypes.c_void_p]
    library.cuda_zlib_decompress_format.argtypes = [_u8p, ctypes.c_uint64, ctypes.c_int32,
                                                    ctypes.c_uint64, ctypes.c_int64,
                                                    ctypes.c_int64, _u8p, ctypes.c_uint64, _u8p,
                                                    ctypes.c_void_p]
    library.cuda_zlib_gzip_header.argtypes = [ctypes.c_void_p, ctypes.c_uint64,
                                              ctypes.POINTER(ctypes.c_uint64)]
    for name in ("cuda_zlib_compress", "cuda_zlib_decompress", "cuda_zlib_compress_batch",
                 "cuda_zlib_decompress_batch", "cuda_zlib_compress_range",
                 "cuda_zlib_compress_batch_packed",
                 "cuda_zlib_compress_format", "cuda_zlib_decompress_format",
                 "cuda_zlib_gzip_header"):
        getattr(library, name).restype = ctypes.c_int
    library.CudaZlibSetWorkspaceRetention.argtypes = [ctypes.c_uint64]
    library.CudaZlibSetWorkspaceRetention.restype = ctypes.c_int
    library.CudaZlibWorkspacePoolStats.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint64)]
    library.CudaZlibWorkspacePoolStats.restype = ctypes.c_int
    library.CudaZlibTrimWorkspacePool.argtypes = [ctypes.c_int]
    library.CudaZlibTrimWorkspacePool.restype = ctypes.c_int
    library.cuda_zlib_b200_version.restype = ctypes.c_char_p
    retention = _workspace_retention()
    code = library.CudaZlibSetWorkspaceRetention(retention)
    if code:
        # Retention is fixed once a pool exists (e.g. the library was already
        # loaded and used through its XLA FFI handlers); that is fine when the
        # value in force is the one asked for.
        stats = (ctypes.c_uint64 * 4)()
        if library.CudaZlibWorkspacePoolStats(0, stats) == 0 and stats[0] == retention:
            code = 0
    _check_pool_error(code)


def library():
    """Load (once) and return the native codec library."""
    global _library
    if _library is None:
        with _LOCK:
            if _library is None:
                if not os.path.exists(LIBRARY):
                    raise BackendUnavailable(
                        "native CUDA codec library missing: build it with cuda-zlib_b200/build.py")
                try:
                    handle = ctypes.CDLL(LIBRARY)
                except OSError as exc:
                    raise BackendUnavailable(f"native CUDA codec library failed to load: {exc}")
                _configure(handle)
                _library = handle
    return _library


def check(code, operation):
    """Raise for a nonzero CUDA error returned by an entry point."""
    if code:
        if code == 1:
            raise ValueError(f"{operation}: invalid arguments (cudaErrorInvalidValue)")
        raise BackendUnavailable(f"{operation}: native CUDA codec error {code}")
