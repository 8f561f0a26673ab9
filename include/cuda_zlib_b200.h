/*
 * cuda_zlib_b200.h -- C ABI of the B200 (sm_100a) zlib/Deflate codec.
 *
 * The four codec entry points are the reference's four XLA FFI handlers
 * (xangma/cuda-zlib, src/cuda_zlib/native/codec_ffi.cu) with the FFI buffers
 * and attributes spelled out as plain pointers and sizes:
 *
 *   - input, output and metadata are DEVICE pointers on the device that
 *     owns `stream` (a cudaStream_t passed as void*; NULL = legacy stream);
 *   - size lists (the handlers' span attributes) are HOST arrays;
 *   - codec results go to device metadata exactly as in the reference:
 *     compression [encoded_length, status], decompression [status, 0], one
 *     pair per file for the batch calls;
 *   - the return value is a cudaError_t: 0 on success, cudaErrorInvalidValue
 *     (1) where the reference handler returns ffi::Error::InvalidArgument or
 *     cudaErrorInvalidValue, other CUDA errors as-is.  A nonzero return means
 *     the metadata was not written.
 *
 * Calls are asynchronous on `stream` (one host read of nothing; scratch comes
 * from a per-device stream-ordered pool, like the reference's
 * cudaMemPool workspace, codec_ffi.cu:132-273).  Concurrent calls from
 * several host threads are allowed.
 *
 * Bounds.  Batch calls keep the reference's (totals of 2**28 bytes, 262144
 * files and chunks).  Two bounds are deliberate supersets of the
 * reference's (_codec.py:13,28,103,158-166): one stream may hold up to 2**31
 * uncompressed bytes (decoding also needs at most 2**29 - 2**16 compressed
 * bytes), and chunk_bytes may be up to 262144.  A chunk above 65535 bytes
 * falls back to several stored blocks of at most 65535 bytes, so the padded
 * capacity is size + 5 * S + 6 where S counts ceil(len / 65535) stored
 * blocks per chunk -- exactly size + 5 * chunks + 6 for chunk_bytes up to
 * 65535, the reference's formula.
 *
 * Status codes: 0 ok; 1-13 Deflate parser (_decode_kernels.py:36-50);
 * 14 truncated zlib, 15 bad CMF/FLG, 16 gzip, 17 preset dictionary,
 * 18 candidate overflow, 19 initial block missing, 20 reference depth,
 * 21 Adler-32 mismatch, 22 compression overflow, 23 invalid bounds
 * (codec_ffi.cu:51-62); gzip wrapper only: 24 invalid gzip header,
 * 25 gzip CRC-32 mismatch, 26 gzip ISIZE mismatch.
 */
#ifndef CUDA_ZLIB_B200_H
#define CUDA_ZLIB_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces CudaZlibCompress / CompressImpl (codec_ffi.cu:1144-1151, 981-988,
 * 551-612).  output must have capacity = size + 5*max(1,ceil(size/chunk))+6
 * bytes for chunk <= 65535 (compress_zlib_padded, _codec.py:151-177; the
 * stored-block count above); it is zero-filled past the stream.  metadata:
 * u32[2] = [encoded_length, status]. */
int cuda_zlib_compress(const uint8_t* input, uint64_t size, int64_t chunk_bytes,
                       uint8_t* output, uint64_t capacity, uint32_t* metadata, void* stream);

/* One contiguous range of a longer stream, for splitting a stream's chunks
 * across GPUs.  No counterpart in the reference, which compresses a stream
 * on one device.  Writes the range's raw Deflate chunks with no zlib header
 * or trailer; the last chunk is final only when `last` is nonzero, and a
 * range that is not last must hold a whole number of chunks.  Capacity as
 * for cuda_zlib_compress.  metadata: u32[3] = [body_length, status,
 * adler32 of the range's input].  Bodies of consecutive ranges, with the
 * two-byte header before them and the combined Adler-32 after, are
 * byte-identical to cuda_zlib_compress on the whole input.  Invalid bounds
 * return cudaErrorInvalidValue (1). */
int cuda_zlib_compress_range(const uint8_t* input, uint64_t size, int64_t chunk_bytes,
                             int32_t last, uint8_t* output, uint64_t capacity,
                             uint32_t* metadata, void* stream);

/* Replaces CudaZlibDecompress / DecompressImpl (codec_ffi.cu:1153-1161,
 * 990-998, 662-950).  expected = exact output size (at most 2**31; size
 * at most 2**29 - 2**16); max_candidates and
 * max_blocks in [1, 262144] (defaults 262144 select the small route for
 * outputs <= 64 KiB with inputs <= 128 KiB).  metadata: u32[2] =
 * [status, 0].  A failed output is all zero. */
int cuda_zlib_decompress(const uint8_t* input, uint64_t size, int64_t max_candidates,
                         int64_t max_blocks, uint8_t* output, uint64_t expected,
                         uint32_t* metadata, void* stream);

/* Replaces CudaZlibCompressBatch / CompressBatchImpl (codec_ffi.cu:1163-1171,
 * 1002-1063).  input: the files packed back to back; input_sizes: host
 * int64[files].  output: consecutive padded slots of size_i + 5*chunks_i + 6
 * bytes; metadata: u32[files][2] = [encoded_length, status]. */
int cuda_zlib_compress_batch(const uint8_t* input, uint64_t input_bytes,
                             const int64_t* input_sizes, uint64_t files, int64_t chunk_bytes,
                             uint8_t* output, uint64_t output_bytes, uint32_t* metadata,
                             void* stream);

/* Replaces CudaZlibDecompressBatch / DecompressBatchImpl (codec_ffi.cu:
 * 1173-1182, 1065-1107).  input_sizes / output_sizes: host int64[files]
 * (packed layouts).  encoded_metadata: NULL, or a device u32[files][2] of
 * compression metadata whose encoded lengths replace input_sizes (slots
 * keep their static offsets).  metadata: u32[files][2] = [status, 0]. */
int cuda_zlib_decompress_batch(const uint8_t* input, uint64_t input_bytes,
                               const int64_t* input_sizes, const int64_t* output_sizes,
                               uint64_t files, const uint32_t* encoded_metadata, uint8_t* output,
                               uint64_t output_bytes, uint32_t* metadata, void* stream);

/* Batch compression with packed output.  No counterpart in the reference.
 * Same arguments, bounds and metadata as cuda_zlib_compress_batch (output
 * sized for the padded slots), but the streams go back to back from
 * output[0] in file order (a failed file takes no bytes; the rest of output
 * is zero), so a caller copying the streams to the host copies only the
 * encoded bytes: the sum of metadata's lengths. */
int cuda_zlib_compress_batch_packed(const uint8_t* input, uint64_t input_bytes,
                                    const int64_t* input_sizes, uint64_t files,
                                    int64_t chunk_bytes, uint8_t* output,
                                    uint64_t output_bytes, uint32_t* metadata, void* stream);

/* gzip (RFC 1952) and raw Deflate (RFC 1951) wrappers around the same body
 * codec.  No counterpart in the reference, which supports RFC 1950 only and
 * rejects gzip members with status 16 (_codec.py:105-111).
 * format: 0 zlib (exactly cuda_zlib_compress / cuda_zlib_decompress),
 * 1 raw Deflate, 2 gzip (one member).  Any other format returns
 * cudaErrorInvalidValue (1).
 *
 * cuda_zlib_compress_format: a zlib stream (format 0), its body bare
 * (format 1) or as a gzip member (format 2: header 1f 8b 08 00, MTIME 0,
 * XFL 0, OS 255, then the body, CRC-32 and ISIZE).  level 1 is the
 * reference's encoder (format 0 at level 1 is exactly cuda_zlib_compress);
 * level 2, with no reference counterpart, searches up to 32 hash-chain
 * candidates per position with one-step lazy evaluation (smaller output,
 * slower; the chunking, block choice and trees are level 1's).  Any other
 * level returns cudaErrorInvalidValue (1).  capacity = size + 5 * S + W
 * with S as for cuda_zlib_compress and W = 6 (zlib), 0 (raw) or 18 (gzip);
 * metadata u32[2] = [encoded_length, status], bounds failures [0, 23] as
 * cuda_zlib_compress. */
int cuda_zlib_compress_format(const uint8_t* input, uint64_t size, int64_t chunk_bytes,
                              int32_t format, int32_t level, uint8_t* output,
                              uint64_t capacity, uint32_t* metadata, void* stream);

/* cuda_zlib_decompress_format: decodes a raw Deflate stream (its final
 * block ends in its last byte) or one gzip member whose header is
 * header_bytes long (from cuda_zlib_gzip_header; ignored for formats 0 and
 * 1).  Same bounds, routes and statuses as cuda_zlib_decompress, except that
 * the Adler-32 check is replaced by none (raw) or by CRC-32 (25) and ISIZE
 * (26) checks (gzip); a member shorter than header_bytes + 8 is 24 and a
 * body shorter than two bytes is 1.  metadata u32[2] = [status, 0]; a failed
 * output is all zero. */
int cuda_zlib_decompress_format(const uint8_t* input, uint64_t size, int32_t format,
                                uint64_t header_bytes, int64_t max_candidates,
                                int64_t max_blocks, uint8_t* output, uint64_t expected,
                                uint32_t* metadata, void* stream);

/* Host-side gzip header parse over HOST bytes [0, available): checks the
 * magic bytes, CM = 8, the reserved flag bits and, with FHCRC, the header
 * CRC-16, and skips FEXTRA, FNAME and FCOMMENT.  Returns 0 and the header
 * length in *header_bytes, or 24 (invalid, or not complete within
 * `available` bytes: pass more of the member). */
int cuda_zlib_gzip_header(const uint8_t* bytes, uint64_t available, uint64_t* header_bytes);

/* Compression that allocates no device memory.  No counterpart in the
 * reference: it exists for callers that cannot allocate while they run, such
 * as a service whose allocator reserves the whole device at start-up and
 * lends out only its own buffers, or a latency-critical loop that must not
 * wait on an allocation.  Same arguments, output and metadata as
 * cuda_zlib_compress (byte-identical streams), restricted to
 * size <= CUDA_ZLIB_NOALLOC_MAX_INPUT and
 * 256 <= chunk_bytes <= CUDA_ZLIB_NOALLOC_MAX_CHUNK; anything else returns
 * cudaErrorInvalidValue (1) and leaves output and metadata untouched.  The
 * chunk must also fit the encoder's shared-memory path (every chunk up to
 * 32 KiB does on a B200; a device with less shared memory per block rejects
 * larger chunks the same way), because this entry point has no room for the
 * global spill arrays larger chunks use.
 * Scratch lives in one static device array (about 1.6 MB) that every GPU
 * loading the library keeps until exit.  All calls share it: calls that
 * overlap on the GPU race with each other, so order them (one stream, or
 * events).  The first call on a device also looks up that array's device
 * address and sets kernel attributes for that device; make that first call
 * before any stream capture. */
#define CUDA_ZLIB_NOALLOC_MAX_INPUT (1u << 20)
#define CUDA_ZLIB_NOALLOC_MAX_CHUNK 32768
int cuda_zlib_compress_noalloc(const uint8_t* input, uint64_t size, int64_t chunk_bytes,
                               uint8_t* output, uint64_t capacity, uint32_t* metadata,
                               void* stream);

/* Workspace pool controls, same names and meaning as the reference's C
 * exports (codec_ffi.cu:1113-1142).  Retention is the pools' release
 * threshold in bytes (default 1 GiB); it can only be set before the first
 * pool exists.  stats: [retention, reserved bytes, used bytes, pool count]. */
int CudaZlibSetWorkspaceRetention(uint64_t bytes);
int CudaZlibWorkspacePoolStats(int device, uint64_t* stats);
int CudaZlibTrimWorkspacePool(int device);

/* Library version string, e.g. "0.1.0".  No reference counterpart. */
const char* cuda_zlib_b200_version(void);

/* Kernel launches this library has issued since it was loaded, all devices
 * and threads together (benchmarks report it per timed region). */
uint64_t cuda_zlib_b200_launches(void);

/* Opt-in kernel timing, no reference counterpart (the reference profiles
 * with Nsight Systems only, PROFILING.md).  enable != 0 clears the totals,
 * creates a supply of events on the current device (so that timing a region
 * creates none) and brackets every named kernel launch with CUDA events on
 * its stream;
 * profile_read waits for the recorded events and returns the summed device
 * time and launch count of one kernel ("serial_inflate_kernel",
 * "encode_chunks_kernel", ...).  Off by default; costs two events a launch. */
int cuda_zlib_b200_profile(int enable);
int cuda_zlib_b200_profile_read(const char* kernel, double* total_ms, uint64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* CUDA_ZLIB_B200_H */
