// One warp per zlib stream: the reference's serial decode route.
//
// Semantics follow DecodeOneFile (src/cuda_zlib/native/batch_decode.cuh:123-296):
// the small single-stream route (output <= 64 KiB, input <= 128 KiB, default
// limits; codec_ffi.cu:681-695) and every file of a batch decode
// (BatchDecode, batch_decode.cuh:298-328) use it.  Lane 0 parses the bit
// stream; the warp builds Huffman tables, copies stored blocks and long
// matches, computes Adler-32 and clears a failed output.
//
// Work distribution: a persistent grid; each warp pops stream indices from a
// device counter in largest-first order, so a few long streams never sit
// behind a queue of short ones.
//
// History: every produced byte is written to the output and to a per-warp
// shared-memory ring of kRing bytes.  Matches within the ring read shared
// memory; farther matches read the output in global memory (written earlier
// by this warp, ordered by program order or __syncwarp).
#include "kernels.h"
#include "inflate_core.cuh"

namespace cz {

constexpr u32 kSerialWarps = 4;
constexpr u32 kRing = 8192;
constexpr u32 kRingMask = kRing - 1;

struct SerialShared {
  Tables fixed;
  Tables dyn[kSerialWarps];
  u8 ring[kSerialWarps][kRing];
};

enum Action : u32 { kNone = 0, kStored = 1, kCopy = 2, kDynamic = 3 };

// Adler-32 of data[0..n) by one warp (lanes stride bytes; coalesced).
__device__ u32 warp_adler(const u8* data, u64 n) {
  const u32 lane = threadIdx.x & 31u;
  u64 s1 = 0, s2 = 0;
  u32 since = 0;
  for (u64 i = lane; i < n; i += 32) {
    const u32 x = data[i];
    s1 += x;
    s2 += (n - i) * x;
    if (++since == (1u << 16)) {  // keep the sums far from 2^64 for any n
      s1 %= kAdlerMod;
      s2 %= kAdlerMod;
      since = 0;
    }
  }
  s1 %= kAdlerMod;
  s2 %= kAdlerMod;
  for (u32 o = 16; o; o >>= 1) {
    s1 += __shfl_xor_sync(kFullMask, s1, o);
    s2 += __shfl_xor_sync(kFullMask, s2, o);
  }
  return adler_finish(s1, s2, n);
}

__device__ void warp_fill_zero(u8* out, u64 n) {
  const u32 lane = threadIdx.x & 31u;
  for (u64 i = lane; i < n; i += 32) out[i] = 0;
}

// Decode one stream.  All 32 lanes call; returns the status on every lane.
__device__ u32 warp_inflate_one(const u8* in, u64 in_size, u8* out, u64 out_size, u32 max_blocks,
                                const Tables& fixed, Tables& dyn, u8* ring) {
  const u32 lane = threadIdx.x & 31u;
  if (in_size > kMaxBytes || out_size > kMaxBytes || !max_blocks || max_blocks > kMaxBlocks)
    return kInvalidBounds;
  u32 window = 0, wanted = 0;
  u32 error = zlib_framing(in, in_size, &window, &wanted);
  BitCursor c;
  u64 produced = 0;
  u32 blocks = 0, final = 0;
  bool need_header = true, complete = false, use_dyn = false;
  if (!error && lane == 0) c.init(in + 2, in_size - 6, 0);
  while (!error) {
    u32 action = kNone, len = 0, dist = 0;
    u64 src = 0, dst = 0;
    if (lane == 0) {
      while (!complete) {
        if (need_header) {
          if (blocks >= max_blocks) { error = kBlockLimit; break; }
          ++blocks;
          final = c.take(1, &error);
          const u32 type = c.take(2, &error);
          if (error) break;
          if (type == 3) { error = kReservedType; break; }
          if (type == 0) {
            c.seek((c.pos + 7) & ~7ull);
            const u32 n = c.take(16, &error), comp = c.take(16, &error);
            if (error) break;
            if ((n ^ comp) != 0xffffu) { error = kBadSymbol; break; }
            if (n > out_size - produced) { error = kOutputOverflow; break; }
            if (c.pos > c.end || u64(n) * 8 > c.end - c.pos) { error = kTruncated; break; }
            action = kStored;
            src = 2 + (c.pos >> 3);
            dst = produced;
            len = n;
            produced += n;
            c.seek(c.pos + u64(n) * 8);
            complete = final != 0;
            break;
          }
          if (type == 2) { action = kDynamic; break; }
          use_dyn = false;
          need_header = false;
        }
        const Token tok = decode_token(c, use_dyn ? dyn : fixed);
        if (tok.kind == kTokError) { error = tok.error; break; }
        if (tok.kind == kTokMatch && tok.dist > window) { error = kBadDistance; break; }
        c.skip(tok.bits);
        if (tok.kind == kTokEnd) {
          complete = final != 0;
          need_header = true;
          continue;
        }
        if (tok.kind == kTokLiteral) {
          if (produced >= out_size) { error = kOutputOverflow; break; }
          const u8 b = u8(tok.value);
          out[produced] = b;
          ring[produced & kRingMask] = b;
          ++produced;
          continue;
        }
        if (tok.length > out_size - produced) { error = kOutputOverflow; break; }
        if (tok.dist > produced) { error = kBadDistance; break; }
        if (tok.length >= 32) {
          action = kCopy;
          dst = produced;
          len = tok.length;
          dist = tok.dist;
          produced += tok.length;
          break;
        }
        const u64 from = produced - tok.dist;
        if (tok.dist <= kRing) {
          for (u32 j = 0; j < tok.length; ++j) {
            const u8 b = ring[(from + j) & kRingMask];
            ring[(produced + j) & kRingMask] = b;
            out[produced + j] = b;
          }
        } else {
          for (u32 j = 0; j < tok.length; ++j) {
            const u8 b = out[from + j];
            ring[(produced + j) & kRingMask] = b;
            out[produced + j] = b;
          }
        }
        produced += tok.length;
      }
    }
    error = __shfl_sync(kFullMask, error, 0);
    if (error) break;
    action = __shfl_sync(kFullMask, action, 0);
    const bool done = __shfl_sync(kFullMask, complete ? 1u : 0u, 0) != 0;
    if (action == kDynamic) {
      const u32 st = warp_dynamic_header(c, dyn);
      if (st) { error = st; break; }
      if (lane == 0) { use_dyn = true; need_header = false; }
    } else if (action != kNone) {
      len = __shfl_sync(kFullMask, len, 0);
      src = __shfl_sync(kFullMask, src, 0);
      dst = __shfl_sync(kFullMask, dst, 0);
      if (action == kStored) {
        for (u32 j = lane; j < len; j += 32) {
          const u8 b = in[src + j];
          out[dst + j] = b;
          ring[(dst + j) & kRingMask] = b;
        }
      } else {
        dist = __shfl_sync(kFullMask, dist, 0);
        // Only the dist-byte seed before dst is read, so lanes never read a
        // byte another lane writes in this copy.  Near-ring distances read
        // global memory so no ring slot is overwritten before it is read.
        const u64 first = dst - dist;
        const bool from_ring = dist + 258 <= kRing;
        u32 s = lane % dist;
        const u32 step = 32 % dist;
        for (u32 j = lane; j < len; j += 32) {
          const u8 b = from_ring ? ring[(first + s) & kRingMask] : out[first + s];
          out[dst + j] = b;
          ring[(dst + j) & kRingMask] = b;
          s += step;
          if (s >= dist) s -= dist;
        }
      }
    }
    __syncwarp();
    if (done) break;
  }
  if (!error && lane == 0) {
    if (produced != out_size) error = kSizeMismatch;
    else if ((c.pos + 7) / 8 != in_size - 6) error = kExtentMismatch;
  }
  error = __shfl_sync(kFullMask, error, 0);
  if (!error) {
    __syncwarp();
    if (warp_adler(out, out_size) != wanted) error = kAdlerMismatch;
  }
  return error;
}

__global__ void __launch_bounds__(kSerialWarps * 32)
serial_inflate_kernel(const u8* in, u8* out, const StreamDesc* descs, StreamDesc single,
                      u32 count, const u32* order, u32* next, u32* meta, const u32* encoded,
                      u32 max_blocks) {
  extern __shared__ __align__(16) u8 smem_raw[];
  SerialShared& sh = *reinterpret_cast<SerialShared*>(smem_raw);
  const u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  if (warp == 0) warp_build_fixed(sh.fixed);
  __syncthreads();
  for (;;) {
    u32 item = 0;
    if (lane == 0) item = atomicAdd(next, 1u);
    item = __shfl_sync(kFullMask, item, 0);
    if (item >= count) break;
    const u32 f = order ? order[item] : item;
    const StreamDesc d = descs ? descs[f] : single;
    u64 in_size = d.in_size;
    u32 status = 0;
    if (encoded) {
      // Compression slots keep static offsets while their encoded lengths
      // vary (BatchDecode, batch_decode.cuh:306-324).
      const u32 length = encoded[2 * f], encode_status = encoded[2 * f + 1];
      status = encode_status ? u32(kCompressionOverflow)
                             : (length > d.in_size ? u32(kInvalidBounds) : 0u);
      if (d.out_size > kMaxBytes) status = kInvalidBounds;
      in_size = length;
    }
    if (!status)
      status = warp_inflate_one(in + d.in_offset, in_size, out + d.out_offset, d.out_size,
                                max_blocks, sh.fixed, sh.dyn[warp], sh.ring[warp]);
    // A failed stream publishes an all-zero output.
    if (status && d.out_size <= kMaxBytes) warp_fill_zero(out + d.out_offset, d.out_size);
    if (lane == 0) {
      meta[2 * f] = status;
      meta[2 * f + 1] = 0;
    }
    __syncwarp();
  }
}

cudaError_t configure_serial_inflate(int* per_sm) {
  const size_t smem = sizeof(SerialShared);
  cudaError_t e = cudaFuncSetAttribute(serial_inflate_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, serial_inflate_kernel,
                                                       kSerialWarps * 32, smem);
}

cudaError_t launch_serial_inflate(const u8* in, u8* out, const StreamDesc* descs,
                                  const StreamDesc& single, u32 count, const u32* order, u32* next,
                                  u32* meta, const u32* encoded, u32 max_blocks,
                                  const DeviceInfo& dev, cudaStream_t stream) {
  const size_t smem = sizeof(SerialShared);
  u32 grid = u32(dev.sms) * u32(dev.serial_per_sm > 0 ? dev.serial_per_sm : 1);
  const u32 needed = (count + kSerialWarps - 1) / kSerialWarps;
  if (grid > needed) grid = needed;
  if (grid < 1) grid = 1;
  serial_inflate_kernel<<<grid, kSerialWarps * 32, smem, stream>>>(
      in, out, descs, single, count, order, next, meta, encoded, max_blocks);
  return cudaGetLastError();
}

}  // namespace cz
