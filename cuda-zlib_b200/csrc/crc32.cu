// CRC-32 (the gzip / RFC 1952 checksum: reflected polynomial 0xEDB88320,
// initial value and final XOR 0xFFFFFFFF) over device buffers, and the gzip
// member's header and trailer steps.
//
// The reference codec has no gzip path (it rejects gzip members with status
// 16); these kernels serve this codec's gzip wrapper.  The method is the
// linear one: with R(M) the CRC register after M from a zero register,
//   R(A || B) = R(A) * x^(8|B|) + R(B)          (mod P, over GF(2))
//   crc32(M)  = R(M) + 0xFFFFFFFF * x^(8|M|) + 0xFFFFFFFF,
// so a buffer splits into 64 KiB segments whose registers combine in any
// order once each is shifted by the bytes after it.  The buffer is read as if
// zero-padded in front to whole segments (leading zero bytes leave a zero
// register unchanged), so every segment, and every thread's piece of a
// segment, has the same length and the same shift constants.
#include "kernels.h"
#include "common.cuh"

namespace cz {
namespace {

constexpr u32 kCrcPoly = 0xEDB88320u;  // x^32 + ... reflected: bit 31 is x^0
constexpr u32 kCrcOne = 0x80000000u;   // the polynomial 1
constexpr u32 kCrcThreads = 256;
constexpr u32 kCrcPiece = kCrcSegment / kCrcThreads;  // bytes per thread
constexpr u32 kCombineThreads = 1024;

// v * x mod P.
__host__ __device__ inline u32 gf2_times_x(u32 v) { return (v >> 1) ^ ((v & 1u) ? kCrcPoly : 0u); }

// a * b mod P: b times each term x^k of a, accumulated.
__host__ __device__ inline u32 gf2_mul(u32 a, u32 b) {
  u32 product = 0;
  for (u32 k = 0; k < 32 && a; ++k, b = gf2_times_x(b)) {
    const u32 term = kCrcOne >> k;
    if (a & term) {
      product ^= b;
      a &= ~term;
    }
  }
  return product;
}

// x^(8 n) mod P by repeated squaring of x^8.
__host__ __device__ inline u32 gf2_shift_bytes(u64 n) {
  u32 result = kCrcOne, power = kCrcOne >> 8;  // x^8
  for (; n; n >>= 1, power = gf2_mul(power, power))
    if (n & 1u) result = gf2_mul(result, power);
  return result;
}

// The four slice tables: table[k][b] = register of byte b followed by k zero
// bytes.  Built by the CTA in shared memory.
__device__ void build_tables(u32 (*table)[256]) {
  const u32 b = threadIdx.x;
  if (b < 256) {
    u32 r = b;
    for (u32 i = 0; i < 8; ++i) r = gf2_times_x(r);
    table[0][b] = r;
  }
  __syncthreads();
  if (b < 256) {
    u32 r = table[0][b];
    for (u32 k = 1; k < 4; ++k) {
      r = table[0][r & 255u] ^ (r >> 8);
      table[k][b] = r;
    }
  }
  __syncthreads();
}

__device__ inline u32 crc_byte(const u32 (*table)[256], u32 r, u32 byte) {
  return table[0][(r ^ byte) & 255u] ^ (r >> 8);
}

__device__ inline u32 crc_word(const u32 (*table)[256], u32 r, u32 word) {
  r ^= word;  // little-endian: the first byte is the low one
  return table[3][r & 255u] ^ table[2][(r >> 8) & 255u] ^ table[1][(r >> 16) & 255u] ^
         table[0][r >> 24];
}

// Register of bytes [a, b) of buf from a zero register.
__device__ u32 crc_range(const u32 (*table)[256], const u8* buf, u64 a, u64 b) {
  u32 r = 0;
  while (a < b && ((reinterpret_cast<uintptr_t>(buf + a) & 15u) != 0)) r = crc_byte(table, r, buf[a++]);
  for (; a + 16 <= b; a += 16) {
    const uint4 v = *reinterpret_cast<const uint4*>(buf + a);
    r = crc_word(table, r, v.x);
    r = crc_word(table, r, v.y);
    r = crc_word(table, r, v.z);
    r = crc_word(table, r, v.w);
  }
  for (; a < b; ++a) r = crc_byte(table, r, buf[a]);
  return r;
}

// Combine the block's per-thread registers, thread t holding the t-th of
// blockDim.x equal pieces, each `piece` bytes: returns, on thread 0,
// sum_t reg_t * x^(8 piece (blockDim.x - 1 - t)).  `shift` (shared) holds
// x^(8 piece 2^l) for l = 0..log2(blockDim.x) - 1.
__device__ u32 block_combine(u32 reg, const u32* shift, u32* warp_regs) {
  const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  for (u32 l = 0; l < 5; ++l) {
    const u32 o = 1u << l;
    const u32 right = __shfl_down_sync(kFullMask, reg, o);
    if ((lane & (2 * o - 1)) == 0) reg = gf2_mul(reg, shift[l]) ^ right;
  }
  if (lane == 0) warp_regs[warp] = reg;
  __syncthreads();
  if (warp == 0) {
    reg = lane < warps ? warp_regs[lane] : 0u;
    for (u32 l = 0; (1u << l) < warps; ++l) {
      const u32 o = 1u << l;
      const u32 right = __shfl_down_sync(kFullMask, reg, o);
      if ((lane & (2 * o - 1)) == 0) reg = gf2_mul(reg, shift[5 + l]) ^ right;
    }
  }
  return reg;
}

// One CTA per 64 KiB segment (grid-stride): parts[s] = R(segment s).
__global__ void __launch_bounds__(kCrcThreads)
crc_parts_kernel(const u8* buf, u64 n, u32 segments, u32* parts) {
  __shared__ u32 table[4][256];
  __shared__ u32 shift[8], warp_regs[kCrcThreads / 32];
  build_tables(table);
  if (threadIdx.x == 0) {
    shift[0] = gf2_shift_bytes(kCrcPiece);
    for (u32 l = 1; l < 8; ++l) shift[l] = gf2_mul(shift[l - 1], shift[l - 1]);
  }
  __syncthreads();
  const u64 pad = u64(segments) * kCrcSegment - n;
  for (u32 s = blockIdx.x; s < segments; s += gridDim.x) {
    const u64 v0 = u64(s) * kCrcSegment + u64(threadIdx.x) * kCrcPiece;
    const u64 a = v0 < pad ? 0 : v0 - pad;
    const u64 b = v0 + kCrcPiece < pad ? 0 : v0 + kCrcPiece - pad;
    const u32 reg = block_combine(crc_range(table, buf, a, b), shift, warp_regs);
    if (threadIdx.x == 0) parts[s] = reg;
    __syncthreads();
  }
}

// One CTA: crc32 of the whole buffer from its segment registers.  Thread t
// folds virtual segments [t g, (t + 1) g) (segments padded in front to
// kCombineThreads * g), then the block combines the thread registers.
__global__ void __launch_bounds__(kCombineThreads)
crc_combine_kernel(const u32* parts, u32 segments, u64 n, u32* crc) {
  __shared__ u32 shift[10], step[1], warp_regs[kCombineThreads / 32];
  const u32 g = (segments + kCombineThreads - 1) / kCombineThreads;
  if (threadIdx.x == 0) {
    step[0] = gf2_shift_bytes(kCrcSegment);
    shift[0] = gf2_shift_bytes(u64(kCrcSegment) * (g ? g : 1));
    for (u32 l = 1; l < 10; ++l) shift[l] = gf2_mul(shift[l - 1], shift[l - 1]);
  }
  __syncthreads();
  const u64 offset = u64(kCombineThreads) * g - segments;
  u32 reg = 0;
  for (u32 j = 0; j < g; ++j) {
    const u64 v = u64(threadIdx.x) * g + j;
    reg = gf2_mul(reg, step[0]) ^ (v < offset ? 0u : parts[v - offset]);
  }
  reg = block_combine(reg, shift, warp_regs);
  if (threadIdx.x == 0) *crc = reg ^ gf2_mul(0xFFFFFFFFu, gf2_shift_bytes(n)) ^ 0xFFFFFFFFu;
}

// gzip trailer of an encoded member: CRC-32 and ISIZE (input size mod 2^32),
// little-endian, in the last 8 bytes of meta[0] (skipped when meta[1] != 0).
__global__ void gzip_trailer_kernel(u8* out, const u32* meta, const u32* crc, u64 isize) {
  if (threadIdx.x != 0 || meta[1]) return;
  u8* t = out + meta[0] - 8;
  const u32 c = *crc, s = u32(isize);
  for (u32 i = 0; i < 4; ++i) {
    t[i] = u8(c >> (8 * i));
    t[4 + i] = u8(s >> (8 * i));
  }
}

// gzip member check after its body decoded: the magic and method bytes,
// then CRC-32, then ISIZE.  Only a decode that succeeded is checked.
__global__ void gzip_check_kernel(const u8* member, u64 size, u64 expected, const u32* crc,
                                  u32* meta) {
  if (threadIdx.x != 0 || meta[0]) return;
  const u8* t = member + size - 8;
  u32 want = 0, isize = 0;
  for (u32 i = 0; i < 4; ++i) {
    want |= u32(t[i]) << (8 * i);
    isize |= u32(t[4 + i]) << (8 * i);
  }
  u32 status = 0;
  if (member[0] != 0x1f || member[1] != 0x8b || member[2] != 8) status = kGzipHeader;
  else if (want != *crc) status = kGzipCrcMismatch;
  else if (isize != u32(expected)) status = kGzipSizeMismatch;
  meta[0] = status;
}

}  // namespace

u32 crc_segments(u64 n) { return u32((n + kCrcSegment - 1) / kCrcSegment); }

cudaError_t launch_crc32(const u8* buf, u64 n, u32* parts, u32* crc, const DeviceInfo& dev,
                         cudaStream_t stream) {
  const u32 segments = crc_segments(n);
  if (segments) {
    const u32 grid = std::min<u32>(segments, u32(dev.sms) * 8);
    profile_begin("crc_parts_kernel", stream);
    note_launch();
    crc_parts_kernel<<<grid, kCrcThreads, 0, stream>>>(buf, n, segments, parts);
    profile_end(stream);
  }
  note_launch();
  crc_combine_kernel<<<1, kCombineThreads, 0, stream>>>(parts, segments, n, crc);
  return cudaGetLastError();
}

cudaError_t launch_gzip_trailer(u8* out, const u32* meta, const u32* crc, u64 isize,
                                cudaStream_t stream) {
  note_launch();
  gzip_trailer_kernel<<<1, 32, 0, stream>>>(out, meta, crc, isize);
  return cudaGetLastError();
}

cudaError_t launch_gzip_check(const u8* member, u64 size, u64 expected, const u32* crc, u32* meta,
                              cudaStream_t stream) {
  note_launch();
  gzip_check_kernel<<<1, 32, 0, stream>>>(member, size, expected, crc, meta);
  return cudaGetLastError();
}

}  // namespace cz
