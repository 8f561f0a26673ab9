"""B200-native zlib/Deflate codec with the cuda_zlib Python API.

Importing this package does not initialize CUDA.  The API mirrors
xangma/cuda-zlib (src/cuda_zlib/__init__.py:14-20): the same functions,
bounds, errors and metadata layouts, with PyTorch CUDA tensors where the
reference returns JAX arrays.  formats.py adds gzip (RFC 1952) and raw
Deflate (RFC 1951) wrappers around the same body codec.  Every codec call
runs hand-written sm_100a kernels through libcuda_zlib_b200.so; there is no
CPU codec fallback.
"""

from ._codec import (compress_zlib, compress_zlib_host, decompress_zlib, compile_kernels,
                     compress_zlib_padded, decompress_zlib_checked,
                     decompress_zlib_host, workspace_pool_stats, trim_workspace_pool)
from ._codec import (compress_zlib_batch_padded_host, decompress_zlib_batch_checked_host,
                     compress_zlib_batch_packed, compress_zlib_batch_packed_host)
from ._codec import (compress_zlib_batch_padded, decompress_zlib_batch_checked,
                     compress_zlib_batch, decompress_zlib_batch,
                     compress_zlib_batch_host, decompress_zlib_batch_host)
from .formats import (compress_deflate, compress_deflate_padded, decompress_deflate,
                      decompress_deflate_checked, compress_gzip, compress_gzip_padded,
                      compress_gzip_host, decompress_gzip, decompress_gzip_checked,
                      decompress_gzip_host, gzip_header_size)
from ._errors import BackendUnavailable, CodecError, UnsupportedStream

__all__ = ["compress_zlib", "compress_zlib_host", "decompress_zlib", "compile_kernels",
           "compress_zlib_padded", "decompress_zlib_checked", "decompress_zlib_host",
           "workspace_pool_stats", "trim_workspace_pool",
           "compress_zlib_batch_padded", "decompress_zlib_batch_checked",
           "compress_zlib_batch", "decompress_zlib_batch",
           "compress_zlib_batch_host", "decompress_zlib_batch_host",
           "compress_zlib_batch_padded_host", "decompress_zlib_batch_checked_host",
           "compress_zlib_batch_packed", "compress_zlib_batch_packed_host",
           "compress_deflate", "compress_deflate_padded", "decompress_deflate",
           "decompress_deflate_checked", "compress_gzip", "compress_gzip_padded",
           "compress_gzip_host", "decompress_gzip", "decompress_gzip_checked",
           "decompress_gzip_host", "gzip_header_size",
           "BackendUnavailable", "CodecError", "UnsupportedStream"]
__version__ = "0.1.0"
