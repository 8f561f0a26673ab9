// Shared definitions for the B200 zlib codec kernels (sm_100a).
//
// Status codes are the reference's metadata values: 1..13 from the Deflate
// parser (src/cuda_zlib/_decode_kernels.py:36-50) and 14..23 from its host
// handlers (src/cuda_zlib/native/codec_ffi.cu:51-62).  Callers read them from
// device metadata, exactly as with the reference.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace cz {

typedef uint8_t u8;
typedef uint16_t u16;
typedef uint32_t u32;
typedef uint64_t u64;

constexpr u32 kMaxBytes = 1u << 28;      // _codec.py:13
constexpr u32 kMaxCandidates = 262144;   // _codec.py:14
constexpr u32 kMaxBlocks = 262144;       // _codec.py:15

enum Status : u32 {
  kOk = 0,
  kTruncated = 1,
  kReservedType = 2,
  kBadTree = 3,
  kBadSymbol = 4,
  kBadRepeat = 5,
  kBadDistance = 6,
  kOutputOverflow = 7,
  kBlockLimit = 9,
  kUndiscovered = 10,
  kSizeMismatch = 11,
  kExtentMismatch = 12,
  kFixedTiles = 13,
  kTruncatedZlib = 14,
  kInvalidHeader = 15,
  kUnsupportedGzip = 16,
  kUnsupportedDictionary = 17,
  kCandidateOverflow = 18,
  kInitialBlockMissing = 19,
  kReferenceDepthExceeded = 20,
  kAdlerMismatch = 21,
  kCompressionOverflow = 22,
  kInvalidBounds = 23,
  // gzip wrapper (this codec only; the reference rejects gzip with 16).
  kGzipHeader = 24,
  kGzipCrcMismatch = 25,
  kGzipSizeMismatch = 26,
};

constexpr u32 kFullMask = 0xffffffffu;

__host__ __device__ inline u32 min_u32(u32 a, u32 b) { return a < b ? a : b; }
__host__ __device__ inline u32 max_u32(u32 a, u32 b) { return a > b ? a : b; }
__host__ __device__ inline u64 min_u64(u64 a, u64 b) { return a < b ? a : b; }

// zlib wrapper check shared by every decode route (DecompressionFraming,
// codec_ffi.cu:304-329; DecodeOneFile, batch_decode.cuh:145-164).
__device__ inline u32 zlib_framing(const u8* in, u64 size, u32* window, u32* wanted) {
  if (size < 8) return kTruncatedZlib;
  const u32 cmf = in[0], flg = in[1];
  if (cmf == 0x1f && flg == 0x8b) return kUnsupportedGzip;
  if ((cmf & 15) != 8 || (cmf >> 4) > 7 || (cmf * 256 + flg) % 31) return kInvalidHeader;
  if (flg & 32) return kUnsupportedDictionary;
  *window = 1u << ((cmf >> 4) + 8);
  *wanted = (u32(in[size - 4]) << 24) | (u32(in[size - 3]) << 16) |
            (u32(in[size - 2]) << 8) | u32(in[size - 1]);
  return kOk;
}

// Adler-32 pieces.  A segment of `n` bytes contributes (s1 = sum x_i,
// s2 = sum (n - i) x_i); segments combine as
//   S1 = sum s1_k,  S2 = sum (s2_k + s1_k * bytes_after_k),
// and adler = ((S2 + N) mod 65521) << 16 | ((S1 + 1) mod 65521).
// Partial sums stay reduced mod 65521 so any stream length composes.
constexpr u32 kAdlerMod = 65521u;

__host__ __device__ inline u32 adler_finish(u64 s1, u64 s2, u64 n) {
  const u32 a = u32((s1 % kAdlerMod + 1) % kAdlerMod);
  const u32 b = u32((s2 % kAdlerMod + n % kAdlerMod) % kAdlerMod);
  return (b << 16) | a;
}

}  // namespace cz
