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
// device counter in order of estimated decode cost, costliest first (the
// host's order in decompress_batch), so a few long streams never sit behind
// a queue of short ones and the last streams taken are quick.
//
// History: every produced byte is written to the output and to a per-warp
// shared-memory ring of kRing bytes.  Matches within the ring read shared
// memory; farther matches read the output in global memory (written earlier
// by this warp, ordered by program order or __syncwarp).
#include "kernels.h"
#include "inflate_core.cuh"

namespace cz {

constexpr u32 kSerialWarps = 4;
// History bytes cached per warp (a power of two).  8 KiB keeps four 4-warp
// CTAs on an SM; a batch of 64 KiB files decoded 35% faster than with 16 KiB
// (two CTAs), because farther matches are rare and more warps hide latency.
constexpr u32 kRing = 8192;
constexpr u32 kRingMask = kRing - 1;
constexpr u32 kFlushBytes = 2048; // produced bytes that trigger a warp flush

struct SerialShared {
  Tables dyn[kSerialWarps];
  __align__(16) u8 ring[kSerialWarps][kRing];
};

// Adler-32 partial sums of one lane: s1 = sum x, s2 = sum (n - p) x over the
// positions p this lane flushed.  Kept reduced so they never overflow.
struct AdlerLane {
  u64 s1 = 0, s2 = 0;
  __device__ __forceinline__ void add(u32 x, u32 weight) {
    s1 += x;
    s2 += u64(weight) * x;
  }
  __device__ __forceinline__ void reduce() {
    s1 %= kAdlerMod;
    s2 %= kAdlerMod;
  }
};

__device__ __forceinline__ void add_word(AdlerLane& a, u32 w, u32 weight) {
  // Four bytes at positions with weights weight, weight-1, weight-2, weight-3.
  const u32 b0 = w & 255u, b1 = (w >> 8) & 255u, b2 = (w >> 16) & 255u, b3 = w >> 24;
  const u32 sum = b0 + b1 + b2 + b3;
  a.s1 += sum;
  a.s2 += u64(weight) * sum - (b1 + 2 * b2 + 3 * b3);
}

// Copy output [from, to) from the ring to global memory with the whole warp,
// adding every byte to the lanes' Adler sums.  16-byte vectors when `out` is
// 16-byte aligned; bytes at the ragged ends.
__device__ void warp_flush(const u8* ring, u8* out, u32 from, u32 to, u32 n, AdlerLane& adler,
                           bool vec) {
  const u32 lane = threadIdx.x & 31u;
  if (from >= to) return;
  u32 head_end = to, tail_start = to;
  if (vec) {
    head_end = min_u32(to, (from + 15) & ~15u);
    tail_start = head_end + ((to - head_end) & ~15u);
  }
  for (u32 p = from + lane; p < head_end; p += 32) {
    const u8 b = ring[p & kRingMask];
    out[p] = b;
    adler.add(b, n - p);
  }
  for (u32 p = head_end + 16 * lane; p < tail_start; p += 512) {
    const uint4 v = *reinterpret_cast<const uint4*>(ring + (p & kRingMask));
    *reinterpret_cast<uint4*>(out + p) = v;
    add_word(adler, v.x, n - p);
    add_word(adler, v.y, n - p - 4);
    add_word(adler, v.z, n - p - 8);
    add_word(adler, v.w, n - p - 12);
  }
  for (u32 p = tail_start + lane; p < to; p += 32) {
    const u8 b = ring[p & kRingMask];
    out[p] = b;
    adler.add(b, n - p);
  }
  adler.reduce();
}

__device__ void warp_fill_zero(u8* out, u64 n) {
  const u32 lane = threadIdx.x & 31u;
  for (u64 i = lane; i < n; i += 32) out[i] = 0;
}

// Decode one stream.  All 32 lanes call; returns the status on every lane.
// Output bytes are staged in `ring` and flushed by the warp; `produced -
// flushed` stays below kFlushBytes + 258, so every byte older than the ring
// is already in global memory when a far match reads it.
__device__ u32 warp_inflate_one(const u8* in, u64 in_size64, u8* out, u64 out_size64,
                                u32 max_blocks, bool checksum, const Tables& fixed, Tables& dyn,
                                u8* ring) {
  const u32 lane = threadIdx.x & 31u;
  if (in_size64 > kMaxBytes || out_size64 > kMaxBytes || !max_blocks || max_blocks > kMaxBlocks)
    return kInvalidBounds;
  const u32 in_size = u32(in_size64), out_size = u32(out_size64);
  u32 window = 0, wanted = 0;
  u32 error = zlib_framing(in, in_size, &window, &wanted);
  Bits c;
  u32 produced = 0, flushed = 0, blocks = 0, final = 0, full_words = 0;
  bool need_header = true, complete = false;
  AdlerLane adler;
  const bool vec = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  if (!error && lane == 0) {
    c.init(in + 2, in_size - 6);
    full_words = (c.shift + c.end) >> 5;
  }
  while (!error) {
    u32 action = kNone, len = 0, dist = 0, src = 0, dst = 0;
    if (lane == 0) {
      while (!complete) {
        if (produced - flushed >= kFlushBytes) { action = kFlush; break; }
        if (need_header) {
          if (blocks >= max_blocks) { error = kBlockLimit; break; }
          ++blocks;
          final = c.take(1, &error);
          const u32 type = c.take(2, &error);
          if (error) break;
          if (type == 3) { error = kReservedType; break; }
          if (type == 0) {
            c.seek((c.pos() + 7) & ~7u);
            const u32 n = c.take(16, &error), comp = c.take(16, &error);
            if (error) break;
            if ((n ^ comp) != 0xffffu) { error = kBadSymbol; break; }
            if (n > out_size - produced) { error = kOutputOverflow; break; }
            const u32 at = c.pos();
            if (at > c.end || n * 8 > c.end - at) { error = kTruncated; break; }
            action = kStored;
            src = 2 + (at >> 3);
            dst = produced;
            len = n;
            produced += n;
            c.seek(at + n * 8);
            complete = final != 0;
            break;
          }
          action = type == 2 ? kDynamic : kFixed;
          break;
        }
        const Tables& t = dyn;
        // Fast loop: every bit it reads lies inside the body and every token
        // fits the output, so only history and table kinds are checked.
        // Anything unusual goes to the exact path below, unconsumed.
        const u32 stop_at =
            min_u32(out_size >= 258 ? out_size - 258 : 0, flushed + kFlushBytes);
        const u32 idx_limit = full_words >= 2 ? full_words - 1 : 0;
        // The next input word is loaded one refill ahead, so a refill
        // appends a register instead of waiting on its load.
        u32 ahead = c.load(c.idx);
        auto refill_ahead = [&]() {
          if (c.nbits <= 32) {
            c.append(ahead);
            ++c.idx;
            ahead = c.load(c.idx);
          }
        };
        while (c.idx < idx_limit && produced < stop_at) {
          refill_ahead();
          const u32 v = c.lo;
          const u32 e = t.ll.lut[v & kLLMask];
          const u32 kind = entry_kind(e);
          if (kind == kLiteral) {
            c.consume(entry_len(e));
            ring[produced & kRingMask] = u8(entry_value(e));
            ++produced;
            continue;
          }
          if (kind != kLength) break;
          const u32 saved_lo = c.lo, saved_hi = c.hi;
          const u32 saved_bits = c.nbits, saved_idx = c.idx;
          const u32 L = entry_len(e), E = entry_extra(e);
          const u32 length = entry_value(e) + ((v >> L) & ((1u << E) - 1u));
          c.consume(L + E);
          refill_ahead();
          const u32 w = c.lo;
          const u32 d = t.d.lut[w & 255u];
          const u32 Ld = entry_len(d), Ed = entry_extra(d);
          const u32 span = entry_value(d) + ((w >> Ld) & ((1u << Ed) - 1u));
          if (entry_kind(d) != kLiteral || span > window || span > produced) {
            c.lo = saved_lo;
            c.hi = saved_hi;
            c.nbits = saved_bits;
            c.idx = saved_idx;
            break;
          }
          c.consume(Ld + Ed);
          if (length >= 32) {
            action = kCopy;
            dst = produced;
            len = length;
            dist = span;
            produced += length;
            break;
          }
          const u32 from = produced - span;
          if (span <= kRing) {
            for (u32 j = 0; j < length; ++j)
              ring[(produced + j) & kRingMask] = ring[(from + j) & kRingMask];
          } else {
            for (u32 j = 0; j < length; ++j) ring[(produced + j) & kRingMask] = out[from + j];
          }
          produced += length;
        }
        if (action != kNone) break;
        if (produced - flushed >= kFlushBytes) continue;
        // Exact path: one token with the serial route's checks and order
        // (DecodeOneFile, batch_decode.cuh:230-283).
        const Token tok = take_token(c, t);
        if (tok.kind == kTokError) { error = tok.error; break; }
        if (tok.kind == kTokMatch && tok.dist > window) { error = kBadDistance; break; }
        if (tok.kind == kTokEnd) {
          complete = final != 0;
          need_header = true;
          continue;
        }
        if (tok.kind == kTokLiteral) {
          if (produced >= out_size) { error = kOutputOverflow; break; }
          ring[produced & kRingMask] = u8(tok.value);
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
        const u32 from = produced - tok.dist;
        if (tok.dist <= kRing) {
          for (u32 j = 0; j < tok.length; ++j)
            ring[(produced + j) & kRingMask] = ring[(from + j) & kRingMask];
        } else {
          for (u32 j = 0; j < tok.length; ++j) ring[(produced + j) & kRingMask] = out[from + j];
        }
        produced += tok.length;
      }
    }
    error = __shfl_sync(kFullMask, error, 0);
    if (error) break;
    action = __shfl_sync(kFullMask, action, 0);
    const u32 now = __shfl_sync(kFullMask, produced, 0);
    const bool done = __shfl_sync(kFullMask, complete ? 1u : 0u, 0) != 0;
    if (action == kDynamic) {
      const u32 st = warp_dynamic_header(c, dyn);
      if (st) { error = st; break; }
      if (lane == 0) need_header = false;
    } else if (action == kFixed) {
      warp_load_fixed(dyn, fixed);
      if (lane == 0) need_header = false;
    } else if (action == kFlush) {
      const u32 to = now & ~15u;
      warp_flush(ring, out, flushed, to, out_size, adler, vec);
      flushed = to;
    } else if (action == kStored) {
      len = __shfl_sync(kFullMask, len, 0);
      src = __shfl_sync(kFullMask, src, 0);
      dst = __shfl_sync(kFullMask, dst, 0);
      warp_flush(ring, out, flushed, dst, out_size, adler, vec);
      for (u32 j = lane; j < len; j += 32) {
        const u8 b = in[src + j];
        out[dst + j] = b;
        ring[(dst + j) & kRingMask] = b;
        adler.add(b, out_size - (dst + j));
      }
      adler.reduce();
      flushed = dst + len;
    } else if (action == kCopy) {
      len = __shfl_sync(kFullMask, len, 0);
      dst = __shfl_sync(kFullMask, dst, 0);
      dist = __shfl_sync(kFullMask, dist, 0);
      // Only the dist-byte seed before dst is read, so lanes never read a
      // byte another lane writes in this copy.  Near-ring distances read the
      // flushed global copy, so no ring slot is overwritten before it is read.
      const u32 first = dst - dist;
      const bool from_ring = dist + 258 <= kRing;
      u32 s = lane % dist;
      const u32 step = 32 % dist;
      for (u32 j = lane; j < len; j += 32) {
        const u8 b = from_ring ? ring[(first + s) & kRingMask] : out[first + s];
        ring[(dst + j) & kRingMask] = b;
        s += step;
        if (s >= dist) s -= dist;
      }
    }
    __syncwarp();
    if (done) break;
  }
  if (!error) {
    const u32 end_bits = __shfl_sync(kFullMask, c.pos(), 0);
    const u32 total = __shfl_sync(kFullMask, produced, 0);
    if (total != out_size) error = kSizeMismatch;
    else if ((end_bits + 7) / 8 != in_size - 6) error = kExtentMismatch;
  }
  if (!error) {
    warp_flush(ring, out, flushed, out_size, out_size, adler, vec);
    u64 s1 = adler.s1, s2 = adler.s2;
    for (u32 o = 16; o; o >>= 1) {
      s1 += __shfl_xor_sync(kFullMask, s1, o);
      s2 += __shfl_xor_sync(kFullMask, s2, o);
    }
    if (checksum && adler_finish(s1, s2, out_size) != wanted) error = kAdlerMismatch;
  }
  return error;
}

__global__ void __launch_bounds__(kSerialWarps * 32)
serial_inflate_kernel(const u8* in, u8* out, const StreamDesc* descs, StreamDesc single,
                      u32 count, const u32* order, u32* next, u32* meta, const u32* encoded,
                      u32 max_blocks, u32 checksum, const Tables* fixed) {
  extern __shared__ __align__(16) u8 smem_raw[];
  SerialShared& sh = *reinterpret_cast<SerialShared*>(smem_raw);
  const u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
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
                                max_blocks, checksum != 0, *fixed, sh.dyn[warp], sh.ring[warp]);
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
                                  const DeviceInfo& dev, cudaStream_t stream, bool checksum) {
  const size_t smem = sizeof(SerialShared);
  u32 grid = u32(dev.sms) * u32(dev.serial_per_sm > 0 ? dev.serial_per_sm : 1);
  const u32 needed = (count + kSerialWarps - 1) / kSerialWarps;
  if (grid > needed) grid = needed;
  if (grid < 1) grid = 1;
  profile_begin("serial_inflate_kernel", stream);
  note_launch();
  serial_inflate_kernel<<<grid, kSerialWarps * 32, smem, stream>>>(
      in, out, descs, single, count, order, next, meta, encoded, max_blocks, checksum ? 1u : 0u,
      static_cast<const Tables*>(dev.fixed_tables));
  profile_end(stream);
  return cudaGetLastError();
}

}  // namespace cz
