// XLA FFI handlers of the codec: the reference's four typed handlers
// (src/cuda_zlib/native/codec_ffi.cu:1144-1182), same names, bindings and
// attribute names, each a thin wrapper of the C ABI in
// include/cuda_zlib_b200.h on the JAX-supplied stream.
//
// A JAX front end registers them exactly as the reference does
// (src/cuda_zlib/_ffi.py:127-131):
//   jax.ffi.register_ffi_target("cuda_zlib_compress_sm_100a",
//       jax.ffi.pycapsule(lib.CudaZlibCompress), platform="CUDA")
// and likewise CudaZlibDecompress, CudaZlibCompressBatch and
// CudaZlibDecompressBatch.
//
// Error convention (codec_ffi.cu:952-977): codec failures are statuses in the
// metadata buffer and return Success; malformed buffer shapes and invalid
// arguments (the C ABI's cudaErrorInvalidValue) are InvalidArgument; other
// CUDA errors are Internal.
//
// Built against jaxlib's xla/ffi/api/ffi.h when jaxlib is installed, else
// against the stand-in header in ffi/standin (same declarations, no call
// frame decoding), which checks every binding against its handler.
#include <cuda_runtime_api.h>

#include <cstdint>
#include <string>
#include <vector>

#include "xla/ffi/api/ffi.h"
#include "cuda_zlib_b200.h"

namespace ffi = xla::ffi;

namespace {

using Sizes = ffi::Span<const std::int64_t>;

ffi::Error FromCode(int code, const char* what) {
  if (code == 0) return ffi::Error::Success();
  if (code == int(cudaErrorInvalidValue))
    return ffi::Error::InvalidArgument(std::string(what) + ": invalid codec arguments");
  return ffi::Error::Internal(std::string(what) + ": native CUDA codec error " +
                              std::to_string(code));
}

template <typename Result>
bool Vector(const Result& buffer, std::size_t count) {
  const auto dims = buffer->dimensions();
  return dims.size() == 1 && std::size_t(dims[0]) == count;
}

template <typename Result>
bool Pairs(const Result& buffer, std::size_t files) {
  const auto dims = buffer->dimensions();
  return dims.size() == 2 && std::size_t(dims[0]) == files && dims[1] == 2;
}

template <typename Body>
ffi::Error Guard(Body&& body) {
  try {
    return body();
  } catch (...) {
    return ffi::Error::Internal("native CUDA codec handler exception");
  }
}

ffi::Error CompressImpl(cudaStream_t stream, std::int64_t chunk_bytes,
                        ffi::Buffer<ffi::U8> input, ffi::ResultBuffer<ffi::U8> output,
                        ffi::ResultBuffer<ffi::U32> metadata) {
  return Guard([&] {
    if (!Vector(metadata, 2))
      return ffi::Error::InvalidArgument("codec metadata must have shape (2,)");
    return FromCode(cuda_zlib_compress(input.typed_data(), input.element_count(), chunk_bytes,
                                       output->typed_data(), output->element_count(),
                                       metadata->typed_data(), stream),
                    "CudaZlibCompress");
  });
}

ffi::Error DecompressImpl(cudaStream_t stream, std::int64_t max_candidates,
                          std::int64_t max_blocks, ffi::Buffer<ffi::U8> input,
                          ffi::ResultBuffer<ffi::U8> output,
                          ffi::ResultBuffer<ffi::U32> metadata) {
  return Guard([&] {
    if (!Vector(metadata, 2))
      return ffi::Error::InvalidArgument("codec metadata must have shape (2,)");
    return FromCode(cuda_zlib_decompress(input.typed_data(), input.element_count(),
                                         max_candidates, max_blocks, output->typed_data(),
                                         output->element_count(), metadata->typed_data(),
                                         stream),
                    "CudaZlibDecompress");
  });
}

ffi::Error CompressBatchImpl(cudaStream_t stream, std::int64_t chunk_bytes, Sizes input_sizes,
                             ffi::Buffer<ffi::U8> input, ffi::ResultBuffer<ffi::U8> output,
                             ffi::ResultBuffer<ffi::U32> metadata) {
  return Guard([&] {
    const std::size_t files = input_sizes.size();
    if (!Pairs(metadata, files))
      return ffi::Error::InvalidArgument("batch codec metadata must have shape (files, 2)");
    const std::vector<std::int64_t> sizes(input_sizes.begin(), input_sizes.end());
    return FromCode(cuda_zlib_compress_batch(input.typed_data(), input.element_count(),
                                             sizes.data(), files, chunk_bytes,
                                             output->typed_data(), output->element_count(),
                                             metadata->typed_data(), stream),
                    "CudaZlibCompressBatch");
  });
}

ffi::Error DecompressBatchImpl(cudaStream_t stream, Sizes input_sizes, Sizes output_sizes,
                               ffi::Buffer<ffi::U8> input, ffi::Buffer<ffi::U32> encoded,
                               ffi::ResultBuffer<ffi::U8> output,
                               ffi::ResultBuffer<ffi::U32> metadata) {
  return Guard([&] {
    const std::size_t files = input_sizes.size();
    if (output_sizes.size() != files || !Pairs(metadata, files))
      return ffi::Error::InvalidArgument("batch codec metadata must have shape (files, 2)");
    // An empty encoded-metadata buffer means "use input_sizes"
    // (decompress_zlib_batch_checked without encoded_metadata).
    const bool has_lengths = encoded.element_count() != 0;
    if (has_lengths && encoded.element_count() != 2 * files)
      return ffi::Error::InvalidArgument("encoded metadata must have shape (files, 2)");
    const std::vector<std::int64_t> in(input_sizes.begin(), input_sizes.end());
    const std::vector<std::int64_t> out(output_sizes.begin(), output_sizes.end());
    return FromCode(cuda_zlib_decompress_batch(input.typed_data(), input.element_count(),
                                               in.data(), out.data(), files,
                                               has_lengths ? encoded.typed_data() : nullptr,
                                               output->typed_data(), output->element_count(),
                                               metadata->typed_data(), stream),
                    "CudaZlibDecompressBatch");
  });
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(
    CudaZlibCompress, CompressImpl,
    ffi::Ffi::Bind()
        .Ctx<ffi::PlatformStream<cudaStream_t>>()
        .Attr<std::int64_t>("chunk_bytes")
        .Arg<ffi::Buffer<ffi::U8>>()
        .Ret<ffi::Buffer<ffi::U8>>()
        .Ret<ffi::Buffer<ffi::U32>>());

XLA_FFI_DEFINE_HANDLER_SYMBOL(
    CudaZlibDecompress, DecompressImpl,
    ffi::Ffi::Bind()
        .Ctx<ffi::PlatformStream<cudaStream_t>>()
        .Attr<std::int64_t>("max_candidates")
        .Attr<std::int64_t>("max_blocks")
        .Arg<ffi::Buffer<ffi::U8>>()
        .Ret<ffi::Buffer<ffi::U8>>()
        .Ret<ffi::Buffer<ffi::U32>>());

XLA_FFI_DEFINE_HANDLER_SYMBOL(
    CudaZlibCompressBatch, CompressBatchImpl,
    ffi::Ffi::Bind()
        .Ctx<ffi::PlatformStream<cudaStream_t>>()
        .Attr<std::int64_t>("chunk_bytes")
        .Attr<Sizes>("input_sizes")
        .Arg<ffi::Buffer<ffi::U8>>()
        .Ret<ffi::Buffer<ffi::U8>>()
        .Ret<ffi::Buffer<ffi::U32>>());

XLA_FFI_DEFINE_HANDLER_SYMBOL(
    CudaZlibDecompressBatch, DecompressBatchImpl,
    ffi::Ffi::Bind()
        .Ctx<ffi::PlatformStream<cudaStream_t>>()
        .Attr<Sizes>("input_sizes")
        .Attr<Sizes>("output_sizes")
        .Arg<ffi::Buffer<ffi::U8>>()
        .Arg<ffi::Buffer<ffi::U32>>()
        .Ret<ffi::Buffer<ffi::U8>>()
        .Ret<ffi::Buffer<ffi::U32>>());
