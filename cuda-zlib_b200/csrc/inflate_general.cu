// General-route semantics for single streams outside the small route.
//
// The reference decodes large streams speculatively (codec_ffi.cu:755-950):
// it discovers candidate block starts, describes every candidate, walks the
// exact block chain (with a fixed-Huffman tile retry), emits with history and
// finally checks Adler-32.  Its statuses therefore follow that order: framing
// (14-17), candidate overflow (18), the first structural error of the chain
// (parse_block semantics: output bound before window; undiscovered dynamic
// headers are status 10), then history/window errors (6), then Adler (21).
//
// Here the fast decode path owns success; this file provides
//   * discover_kernel: the reference's candidate rule and raw event count
//     (discover, _decode_kernels.py:998-1054), always run, because a count
//     above the capacity fails even a valid stream with status 18;
//   * general_status_kernel: one thread restating the chain walk and the
//     emission history check, run only after the fast path failed before
//     its checksum, to report the status the reference's route reports.
#include <algorithm>

#include "kernels.h"
#include "inflate_core.cuh"

namespace cz {

// ---------------------------------------------------------------------------
// Candidate discovery
// ---------------------------------------------------------------------------
// Validity of a dynamic header at `start` (BTYPE 2 and dynamic_tables()==0;
// dynamic_valid, _decode_kernels.py:359-366), per thread and without tables:
// the code lengths are checked as they are decoded, so a random bit pattern
// is usually rejected after a few symbols (an over-subscribed code).  The
// code-length code is kept in registers and decoded through `lut`, 128
// bytes of the caller's scratch; every rejection is the one the reference's
// bitwise reads and checks make, in the same cases.  The check runs as
// init (the header and the code-length code) and then one step per
// code-length symbol, so a warp can keep its lanes on different offsets.
struct HeaderCheck {
  BitCursor c;
  u32 nl, nd, i, previous;
  u32 ks0, ks1, nz0, nz1, mx0, mx1;  // per part: Kraft sum (2^-15 units), nonzero count, maximum
  bool eob;
};
enum HeaderStep : u32 { kHeaderMore = 0, kHeaderBad = 1, kHeaderGood = 2 };

__device__ u32 header_init(HeaderCheck& h, const u8* body, u64 bytes, u64 start, u8* lut) {
  BitCursor& c = h.c;
  c.init(body, bytes, start);
  u32 err = 0;
  c.take(1, &err);
  const u32 type = c.take(2, &err);
  if (err || type != 2) return kHeaderBad;
  h.nl = c.take(5, &err) + 257;
  h.nd = c.take(5, &err) + 1;
  const u32 nc = c.take(4, &err) + 4;
  if (err || h.nl > 286) return kHeaderBad;
  // Code-length code lengths: 3 bits each, in the RFC 1951 order, read at once.
  if (c.avail() < 3 * nc) return kHeaderBad;
  const u64 fields = c.peek() & ((1ull << (3 * nc)) - 1);
  c.skip(3 * nc);
  // Position of symbol s in the transmission order 16 17 18 0 8 7 9 6 10 5 11 4 12 3 13 2 14 1 15.
  constexpr u32 kOrderPos[19] = {3, 17, 15, 13, 11, 9, 7, 5, 4, 6, 8, 10, 12, 14, 16, 18, 0, 1, 2};
  u32 clen[19];
  u32 kraft = 0;
#pragma unroll
  for (u32 s = 0; s < 19; ++s) {
    clen[s] = u32(fields >> (3 * kOrderPos[s])) & 7u;  // zero beyond nc: masked above
    kraft += clen[s] ? 128u >> clen[s] : 0u;
  }
  // Complete code-length code (Kraft sum exactly one, in units of 2^-7).
  if (kraft != 128) return kHeaderBad;
  // Canonical codes, then the 7-bit lookup: entry = symbol | length << 5.
  u32 first = 0, prior = 0;
#pragma unroll
  for (u32 l = 1; l < 8; ++l) {
    u32 count = 0;
#pragma unroll
    for (u32 s = 0; s < 19; ++s) count += clen[s] == l ? 1u : 0u;
    first = (first + prior) << 1;  // first code of length l
    u32 next = first;
#pragma unroll
    for (u32 s = 0; s < 19; ++s) {
      if (clen[s] == l) {
        const u32 lo = next << (7 - l), hi = (next + 1) << (7 - l);
        for (u32 k = lo; k < hi; ++k) lut[k] = u8(s | (l << 5));
        ++next;
      }
    }
    prior = count;
  }
  h.i = 0;
  h.previous = 0;
  h.ks0 = h.ks1 = h.nz0 = h.nz1 = h.mx0 = h.mx1 = 0;
  h.eob = false;
  return kHeaderMore;
}

// One code-length symbol (literal/length lengths i < nl, distance lengths
// after).  Each symbol and its extra bits come from one 64-bit peek; a
// symbol whose bits (code and extra) run past the body end fails as the
// bitwise reads would.
__device__ u32 header_step(HeaderCheck& h, const u8* lut) {
  BitCursor& c = h.c;
  const u32 total = h.nl + h.nd;
  const u64 w = c.peek();
  const u64 avail = c.avail();
  const u32 e = lut[__brev(u32(w)) >> 25];  // first 7 bits, MSB-first
  const u32 sym = e & 31u, len = e >> 5;
  if (len > avail) return kHeaderBad;
  u32 repeat = 1, value = sym, extra = 0;
  if (sym == 16) {
    if (!h.i) return kHeaderBad;
    extra = 2;
    repeat = u32((w >> len) & 3u) + 3;
    value = h.previous;
  } else if (sym == 17) {
    extra = 3;
    repeat = u32((w >> len) & 7u) + 3;
    value = 0;
  } else if (sym == 18) {
    extra = 7;
    repeat = u32((w >> len) & 127u) + 11;
    value = 0;
  }
  if (len + extra > avail) return kHeaderBad;
  c.skip(len + extra);
  const u32 i = h.i;
  if (repeat > total - i) return kHeaderBad;
  if (value) {
    // The run [i, i + repeat) splits at most once at nl.  Kraft sums only
    // grow, so checking after the run rejects exactly when some element
    // of it would have over-subscribed.
    const u32 n0 = i < h.nl ? min_u32(repeat, h.nl - i) : 0u, n1 = repeat - n0;
    const u32 weight = 32768u >> value;
    h.ks0 += n0 * weight;
    h.ks1 += n1 * weight;
    h.nz0 += n0;
    h.nz1 += n1;
    if (n0 && value > h.mx0) h.mx0 = value;
    if (n1 && value > h.mx1) h.mx1 = value;
    if (h.ks0 > 32768u || h.ks1 > 32768u) return kHeaderBad;  // over-subscribed
    if (i <= 256 && 256 < i + repeat) h.eob = true;
  }
  h.i = i + repeat;
  h.previous = value;
  if (h.i < total) return kHeaderMore;
  if (!h.eob) return kHeaderBad;
  // Literal/length: complete, or a single length-1 code.  Distance: empty,
  // complete, or a single length-1 code.
  if (!h.nz0) return kHeaderBad;
  if (h.ks0 != 32768u && !(h.mx0 == 1 && h.nz0 == 1)) return kHeaderBad;
  if (h.nz1 && h.ks1 != 32768u && !(h.mx1 == 1 && h.nz1 == 1)) return kHeaderBad;
  return kHeaderGood;
}

__device__ bool dynamic_header_valid(const u8* body, u64 bytes, u64 start, u8* lut) {
  HeaderCheck h;
  u32 st = header_init(h, body, bytes, start, lut);
  while (st == kHeaderMore) st = header_step(h, lut);
  return st == kHeaderGood;
}

// Stored-block endpoint seed at body byte `byte` (discover, :1009-1035).
__device__ bool stored_seed(const u8* body, u64 bytes, u64 byte, u64* endpoint) {
  const u64 available = bytes - byte;
  if (!byte || available < 5) return false;
  const u32 n = u32(body[byte]) | (u32(body[byte + 1]) << 8);
  const u32 comp = u32(body[byte + 2]) | (u32(body[byte + 3]) << 8);
  if ((n ^ comp) != 0xffffu || u64(n) + 4 >= available) return false;
  u32 before = u32(body[byte - 1]) << 8;
  if (byte >= 2) before |= body[byte - 2];
  bool possible = false;
  for (u32 gap = 3; gap <= 10; ++gap)
    if (byte * 8 >= gap && ((before >> (17 - gap)) & 3u) == 0) possible = true;
  const u64 e = byte + 4 + n;
  if (!possible || ((body[e] >> 1) & 3u) != 1) return false;
  *endpoint = e;
  return true;
}

// Stored-run seed at body byte `byte`: a stored block of at least 1024 bytes
// whose LEN/NLEN start there and that another stored block follows.  Its
// endpoint (the next block's header, byte aligned) is a fast-path candidate,
// so that a long run of stored blocks splits into nodes of one block each;
// the reference's candidate rule seeds only stored blocks followed by a
// fixed one (stored_seed above), and its event count ignores these.
__device__ bool stored_chain(const u8* body, u64 bytes, u64 byte, u64* endpoint) {
  if (!byte || bytes - byte < 5) return false;
  const u32 n = u32(body[byte]) | (u32(body[byte + 1]) << 8);
  const u32 comp = u32(body[byte + 2]) | (u32(body[byte + 3]) << 8);
  if ((n ^ comp) != 0xffffu || n < 1024) return false;
  const u64 e = byte + 4 + n;
  if (e + 5 > bytes) return false;
  u32 before = u32(body[byte - 1]) << 8;
  if (byte >= 2) before |= body[byte - 2];
  bool possible = false;
  for (u32 gap = 3; gap <= 10; ++gap)
    if (byte * 8 >= gap && ((before >> (17 - gap)) & 3u) == 0) possible = true;
  if (!possible || ((body[e] >> 1) & 3u) != 0) return false;
  const u32 n2 = u32(body[e + 1]) | (u32(body[e + 2]) << 8);
  const u32 c2 = u32(body[e + 3]) | (u32(body[e + 4]) << 8);
  if ((n2 ^ c2) != 0xffffu) return false;
  *endpoint = e;
  return true;
}

constexpr u32 kDiscoverTile = 4096;     // body bytes per CTA step
constexpr u32 kDiscoverThreads = 256;
constexpr u32 kDiscoverWarps = kDiscoverThreads / 32;
// Tile bytes per warp, scanned in two rounds of 64 words (two per lane).
constexpr u32 kDiscoverWarpWords = kDiscoverTile / 4 / kDiscoverWarps;
// Offsets a round can pass: at most every other bit offset passes the BTYPE
// filter (bit b+1 clear and bit b+2 set), so 16 of a word's 32.
constexpr u32 kDiscoverPending = 2 * 32 * 16;

// Candidates of every body bit offset (discover, _decode_kernels.py:
// 998-1054): bit 0; offsets whose three header bits are BTYPE 2 and whose
// dynamic header is valid; stored-block endpoint seeds.  Sets bit b of
// bitmap[b >> 5] per candidate offset and adds the raw event count
// (duplicates included).  Per tile (staged in shared memory with a 32-byte
// halo), each lane filters the 32 offsets of a tile word at once with word
// operations (BTYPE 2, HLIT at most 29), the warp gathers the survivors, and
// then tests them 32 at a time, all lanes busy, for a complete code-length
// code (Kraft sums of three packed 3-bit lengths from a table).  The few
// offsets that pass go to a global queue, one atomic per warp batch, that
// validate_kernel works through one per thread, so the long validations of
// true headers run side by side across the GPU.  Offsets beyond the queue's
// capacity are validated here.
__global__ void __launch_bounds__(kDiscoverThreads)
discover_kernel(const u8* in, u64 in_size, u32* bitmap, u32* extra, u32* count, u32* queue,
                u32 queue_cap, u32* queued, const u32* gate) {
  __shared__ u32 tile[kDiscoverTile / 4 + 8];
  __shared__ u8 kraft3[512];
  __shared__ u16 pending[kDiscoverWarps][kDiscoverPending];  // tile bit offsets
  if (gate && *gate) return;
  if (in_size < 8) return;
  const u8* body = in + 2;
  const u64 bytes = in_size - 6;
  const u32 lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (u32 t = threadIdx.x; t < 512; t += blockDim.x) {
    u32 sum = 0;
    for (u32 k = 0; k < 3; ++k) {
      const u32 L = (t >> (3 * k)) & 7u;
      sum += L ? (128u >> L) : 0u;
    }
    kraft3[t] = u8(sum);
  }
  u8* const tile_bytes = reinterpret_cast<u8*>(tile);
  u32 events = 0;
  for (u64 base = u64(blockIdx.x) * kDiscoverTile; base < bytes;
       base += u64(gridDim.x) * kDiscoverTile) {
    __syncthreads();
    for (u32 j = threadIdx.x; j < kDiscoverTile + 32; j += blockDim.x)
      tile_bytes[j] = base + j < bytes ? body[base + j] : u8(0);
    __syncthreads();
    const u64 left = bytes - base;  // body bytes from the tile start (> 0)
    for (u32 round = 0; round < 2; ++round) {
      u32 masks[2];
      u32 mine = 0;
#pragma unroll
      for (u32 h = 0; h < 2; ++h) {
        const u32 wi = warp * kDiscoverWarpWords + round * 64 + h * 32 + lane;
        const u32 w0 = tile[wi], w1 = tile[wi + 1];
        const u64 x = u64(w0) | (u64(w1) << 32);
        // BTYPE 2 at offset b: bit b+1 clear, bit b+2 set; HLIT (bits
        // b+3..b+7) at most 29, i.e. not all of bits b+4..b+7 set.
        u64 all4 = x & (x >> 1);
        all4 &= all4 >> 2;
        u32 m = u32(~x >> 1) & u32(x >> 2) & ~u32(all4 >> 4);
        // Offsets at or past the body end are not candidates.
        const u64 first = u64(wi) * 4;
        if (first + 4 > left) m = first >= left ? 0u : m & ((1u << (8 * u32(left - first))) - 1u);
        if (base == 0 && wi == 0) {
          m &= ~1u;  // bit 0 is always a candidate
          ++events;
          atomicOr(&bitmap[0], 1u);
        }
        // Stored seed: LEN/NLEN complements at one of the word's bytes.
#pragma unroll
        for (u32 k = 0; k < 4; ++k) {
          const u32 v = __funnelshift_r(w0, w1, 8 * k);
          if (((v ^ (v >> 16)) & 0xffffu) == 0xffffu && first + k < left) {
            u64 e;
            if (stored_seed(body, bytes, base + first + k, &e)) {
              ++events;
              atomicOr(&bitmap[(e * 8) >> 5], 1u << ((e * 8) & 31));
            } else if (extra && stored_chain(body, bytes, base + first + k, &e)) {
              atomicOr(&extra[(e * 8) >> 5], 1u << ((e * 8) & 31));
            }
          }
        }
        masks[h] = m;
        mine += __popc(m);
      }
      // Gather the survivors of the warp's 64 words in order.
      u32 incl = mine;
#pragma unroll
      for (u32 o = 1; o < 32; o <<= 1) {
        const u32 v = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += v;
      }
      const u32 total = __shfl_sync(kFullMask, incl, 31);
      u32 at = incl - mine;
#pragma unroll
      for (u32 h = 0; h < 2; ++h) {
        const u32 bit0 = (warp * kDiscoverWarpWords + round * 64 + h * 32 + lane) * 32;
        u32 m = masks[h];
        while (m) {
          pending[warp][at++] = u16(bit0 + __ffs(m) - 1);
          m &= m - 1;
        }
      }
      __syncwarp();
      for (u32 batch = 0; batch < total; batch += 32) {
        const u32 i = batch + lane;
        bool pass = false;
        u32 p = 0;
        if (i < total) {
          p = pending[warp][i];
          // HCLEN and the code-length code lengths: 64 bits from p + 13.
          const u32 q = p + 13, wq = q >> 5, sh = q & 31;
          const u32 a = tile[wq], b = tile[wq + 1], c = tile[wq + 2];
          const u64 x = u64(__funnelshift_r(a, b, sh)) | (u64(__funnelshift_r(b, c, sh)) << 32);
          const u32 nc = u32(x & 15u) + 4;
          const u64 y = (x >> 4) & ((1ull << (3 * nc)) - 1);  // lengths beyond nc read as 0
          u32 kraft = 0;
#pragma unroll
          for (u32 g = 0; g < 7; ++g) kraft += kraft3[u32(y >> (9 * g)) & 511u];
          pass = kraft == 128;  // complete code-length code
        }
        const u32 ballot = __ballot_sync(kFullMask, pass);
        if (ballot) {
          u32 slot = 0;
          if (lane == 0) slot = atomicAdd(queued, u32(__popc(ballot)));
          slot = __shfl_sync(kFullMask, slot, 0) + __popc(ballot & ((1u << lane) - 1u));
          if (pass) {
            const u64 bit = base * 8 + p;
            if (slot < queue_cap) {
              queue[slot] = u32(bit);
            } else {
              u8 lut[128];  // queue full: validate here
              if (dynamic_header_valid(body, bytes, bit, lut)) {
                ++events;
                atomicOr(&bitmap[bit >> 5], 1u << (bit & 31));
              }
            }
          }
        }
      }
      __syncwarp();
    }
  }
  for (u32 o = 16; o; o >>= 1) events += __shfl_xor_sync(kFullMask, events, o);
  if ((threadIdx.x & 31) == 0 && events) atomicAdd(count, events);
}

// Full validation of the queued offsets.  Validations take from a few to a
// few hundred steps, so each lane holds its own offset and, whenever half
// of the warp has finished, the idle lanes take the next offsets together
// (one atomic on cursor[0] for the warp) and build their lookups side by
// side.  Lookup rows are padded by a word, so that lanes building or
// reading the same entry hit different banks.
constexpr u32 kLutStride = 132;
__global__ void __launch_bounds__(kDiscoverThreads)
validate_kernel(const u8* in, u64 in_size, const u32* queue, u32 queue_cap, const u32* queued,
                u32* bitmap, u32* count, const u32* gate) {
  __shared__ __align__(4) u8 cl_lut[kDiscoverThreads * kLutStride];
  if (gate && *gate) return;
  if (in_size < 8) return;
  const u8* body = in + 2;
  const u64 bytes = in_size - 6;
  const u32 n = min_u32(queued[0], queue_cap);
  u32* cursor = const_cast<u32*>(queued) + 1;
  const u32 lane = threadIdx.x & 31u;
  u8* lut = cl_lut + threadIdx.x * kLutStride;
  HeaderCheck h;
  u32 bit = 0, events = 0;
  bool busy = false, drained = false;
  for (;;) {
    const u32 idle = __ballot_sync(kFullMask, !busy);
    if (!drained && __popc(idle) >= 16) {
      // Refill the idle lanes.
      u32 base = 0;
      if (lane == __ffs(idle) - 1) base = atomicAdd(cursor, u32(__popc(idle)));
      base = __shfl_sync(kFullMask, base, __ffs(idle) - 1);
      if (base + __popc(idle) >= n) drained = true;
      if (!busy) {
        const u32 slot = base + __popc(idle & ((1u << lane) - 1u));
        if (slot < n) {
          bit = queue[slot];
          busy = header_init(h, body, bytes, bit, lut) == kHeaderMore;
        }
      }
    }
    if (!__any_sync(kFullMask, busy)) {
      if (drained) break;
      continue;
    }
    // Steps until half of the warp is idle again (or, once the queue is
    // drained, until every lane is).
    do {
      if (busy) {
        const u32 st = header_step(h, lut);
        if (st != kHeaderMore) {
          busy = false;
          if (st == kHeaderGood) {
            ++events;
            atomicOr(&bitmap[bit >> 5], 1u << (bit & 31));
          }
        }
      }
    } while (__popc(__ballot_sync(kFullMask, busy)) > (drained ? 0 : 16));
  }
  for (u32 o = 16; o; o >>= 1) events += __shfl_xor_sync(kFullMask, events, o);
  if ((threadIdx.x & 31) == 0 && events) atomicAdd(count, events);
}

// ---------------------------------------------------------------------------
// Exact general-route status (one thread)
// ---------------------------------------------------------------------------
// Serial table builder (same validation and layout as warp_build).
template <int Primary, int MaxSymbols, typename EntryFn>
__device__ u32 serial_build(Huffman<Primary, MaxSymbols>& t, const u8* lens, u32 n, bool empty_ok,
                            bool single_ok, EntryFn make) {
  u32 cnt[16];
  for (u32 l = 0; l < 16; ++l) cnt[l] = 0;
  u32 maximum = 0;
  for (u32 i = 0; i < n; ++i) {
    ++cnt[lens[i]];
    if (lens[i] > maximum) maximum = lens[i];
  }
  cnt[0] = 0;
  for (u32 l = 0; l < 16; ++l) t.count[l] = u16(cnt[l]);
  t.maxlen = maximum;
  if (!maximum) {
    for (u32 k = 0; k < (1u << Primary); ++k) t.lut[k] = make_entry(kEmpty, 0, 0, 0);
    return empty_ok ? 0u : u32(kBadTree);
  }
  int left = 1;
  for (u32 l = 1; l < 16; ++l) {
    left = (left << 1) - int(cnt[l]);
    if (left < 0) return kBadTree;
  }
  if (left && !(single_ok && maximum == 1 && cnt[1] == 1)) return kBadTree;
  u32 code = 0, offset = 0, cursor[16];
  for (u32 l = 1; l < 16; ++l) {
    code = (code + cnt[l - 1]) << 1;
    t.first[l] = code;
    t.offs[l] = u16(offset);
    cursor[l] = offset;
    offset += cnt[l];
  }
  for (u32 i = 0; i < n; ++i)
    if (lens[i]) t.symbols[cursor[lens[i]]++] = u16(i);
  for (u32 k = 0; k < (1u << Primary); ++k) {
    const u32 v = __brev(k) >> (32 - Primary);
    u32 entry = make_entry(maximum > u32(Primary) ? kLong : kHole, 0, 0, 0);
    const u32 top = maximum < u32(Primary) ? maximum : u32(Primary);
    for (u32 L = 1; L <= top; ++L) {
      const u32 i = (v >> (Primary - L)) - t.first[L];
      if (i < t.count[L]) { entry = make(t.symbols[t.offs[L] + i], L); break; }
    }
    t.lut[k] = entry;
  }
  return 0;
}

__device__ u32 serial_dynamic_header(BitCursor& c, Tables& t) {
  u32 err = 0;
  const u32 nl = c.take(5, &err) + 257, nd = c.take(5, &err) + 1, nc = c.take(4, &err) + 4;
  if (err) return err;
  if (nl > 286) return kBadTree;
  const u8 order[19] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};
  for (u32 i = 0; i < 19; ++i) t.lens[i] = 0;
  for (u32 i = 0; i < nc; ++i) t.lens[order[i]] = u8(c.take(3, &err));
  if (err) return err;
  err = serial_build(t.cl, t.lens, 19, false, false, CLFn());
  if (err) return err;
  u32 i = 0;
  while (i < nl + nd) {
    const u32 e = t.cl.lut[c.peek() & 127u];
    if (entry_len(e) > c.avail()) return kTruncated;
    c.skip(entry_len(e));
    const u32 sym = entry_value(e);
    if (sym < 16) { t.lens[i++] = u8(sym); continue; }
    u32 repeat, value;
    if (sym == 16) {
      if (!i) return kBadRepeat;
      repeat = c.take(2, &err) + 3;
      value = t.lens[i - 1];
    } else if (sym == 17) {
      repeat = c.take(3, &err) + 3;
      value = 0;
    } else {
      repeat = c.take(7, &err) + 11;
      value = 0;
    }
    if (err) return err;
    if (repeat > nl + nd - i) return kBadRepeat;
    for (u32 j = 0; j < repeat; ++j) t.lens[i++] = u8(value);
  }
  if (!t.lens[256]) return kBadTree;
  err = serial_build(t.ll, t.lens, nl, false, true, LLFn());
  if (err) return err;
  // Move the distance lengths to lens[288..): the ranges can overlap and the
  // destination is higher, so copy from the top down.
  for (u32 k = nd; k-- > 0;) t.lens[288 + k] = t.lens[nl + k];
  return serial_build(t.d, t.lens + 288, nd, true, true, DFn());
}

struct BlockInfo {
  u64 end;
  u32 size, final, status;
};

// parse_block<false> (_decode_kernels.py:683-781): no history, `limit`
// output bytes, window 32768, optional fixed budget (status 13).
__device__ BlockInfo parse_block(const u8* body, u64 bytes, u64 start, u32 limit, u32 budget,
                                 const Tables& fixed, Tables& dyn) {
  BitCursor c;
  c.init(body, bytes, start);
  BlockInfo b = {start, 0, 0, 0};
  u32 err = 0;
  b.final = c.take(1, &err);
  const u32 type = c.take(2, &err);
  if (err) { b.status = err; return b; }
  if (type == 3) { b.status = kReservedType; return b; }
  u32 produced = 0;
  if (type == 0) {
    c.seek((c.pos + 7) & ~7ull);
    const u32 n = c.take(16, &err), comp = c.take(16, &err);
    if (err) { b.status = err; return b; }
    if ((n ^ comp) != 0xffffu) { b.status = kBadSymbol; return b; }
    if (n > limit) { b.status = kOutputOverflow; return b; }
    if (c.pos > c.end || u64(n) * 8 > c.end - c.pos) { b.status = kTruncated; return b; }
    b.end = c.pos + u64(n) * 8;
    b.size = n;
    return b;
  }
  if (type == 2) {
    err = serial_dynamic_header(c, dyn);
    if (err) { b.status = err; return b; }
  }
  const Tables& t = type == 2 ? dyn : fixed;
  for (;;) {
    if (type == 1 && budget && (produced >= budget || c.pos - start >= u64(budget) * 8)) {
      err = kFixedTiles;
      break;
    }
    const Token tok = decode_token(c, t);
    if (tok.kind == kTokError) { err = tok.error; break; }
    c.skip(tok.bits);
    if (tok.kind == kTokEnd) break;
    if (tok.kind == kTokLiteral) {
      if (produced >= limit) { err = kOutputOverflow; break; }
      ++produced;
      continue;
    }
    if (tok.length > limit - produced) { err = kOutputOverflow; break; }
    if (tok.dist > 32768u) { err = kBadDistance; break; }
    produced += tok.length;
  }
  b.end = c.pos;
  b.size = produced;
  b.status = err;
  return b;
}

struct Summary {
  u64 end, first_end;
  u32 size, first_size, flags, status;
};

// scan_fixed_region (_decode_kernels.py:444-472), window checked in-token.
__device__ Summary scan_fixed(const u8* body, u64 bytes, u64 entry, u64 tile_end,
                              const Tables& fixed) {
  BitCursor c;
  c.init(body, bytes, entry);
  u32 err = entry >= bytes * 8 ? u32(kTruncated) : 0u;
  Summary s = {entry, ~0ull, 0, 0, 0, 0};
  u32 ended = 0, final = 2, kind = 0;
  while (c.pos < tile_end && !err) {
    const Token tok = decode_token(c, fixed);
    if (tok.kind == kTokError) { err = tok.error; break; }
    c.skip(tok.bits);
    if (tok.kind != kTokEnd) {
      s.size += tok.kind == kTokLiteral ? 1u : tok.length;
      continue;
    }
    if (s.first_end == ~0ull) { s.first_end = c.pos; s.first_size = s.size; }
    ++ended;
    if (final == 1) { kind = 2; break; }
    if (c.pos >= tile_end) { kind = 1; break; }
    const u64 header = c.pos;
    const u32 next_final = c.take(1, &err), type = c.take(2, &err);
    if (err) break;
    if (type != 1) { c.seek(header); kind = 1; break; }
    final = next_final;
  }
  s.end = c.pos;
  s.flags = kind | (final << 2) | (ended << 4);
  s.status = err;
  return s;
}

constexpr u64 kTileBits = 2048ull * 8;

// select_chain_impl (_decode_kernels.py:1226-1408); `tiles` selects the
// fixed-summary retry pass.
__device__ u32 chain_walk(const u8* body, u64 bytes, const u32* bitmap, u32 expected,
                          u32 max_blocks, bool tiles, const Tables& fixed, Tables& dyn) {
  const u64 bits = bytes * 8;
  u64 next = 0;
  u32 output = 0, n = 0, real_blocks = 0;
  for (;;) {
    if (n >= max_blocks) return kBlockLimit;
    BitCursor h;
    h.init(body, bytes, next);
    u32 err = 0;
    u32 final = h.take(1, &err);
    const u32 type = h.take(2, &err);
    if (err) return err;
    if (type == 3) return kReservedType;
    if (type == 1 && tiles) {
      u64 cursor = h.pos;
      for (;;) {
        if (cursor >= bits) return kTruncated;
        u64 tile_end = (cursor / kTileBits + 1) * kTileBits;
        if (tile_end > bits) tile_end = bits;
        Summary s = scan_fixed(body, bytes, cursor, tile_end, fixed);
        u32 kind = s.flags & 3u, ended = s.flags >> 4;
        if (final && s.first_end != ~0ull) {
          s.end = s.first_end;
          s.size = s.first_size;
          s.status = 0;
          kind = 2;
          ended = 1;
        }
        if (s.status) return s.status;
        if (s.end <= cursor || s.end > bits) return kExtentMismatch;
        if (s.size > expected - output) return kOutputOverflow;
        if (n >= max_blocks || ended > max_blocks - real_blocks) return kBlockLimit;
        output += s.size;
        real_blocks += ended;
        ++n;
        cursor = s.end;
        if (kind == 2) {
          if (output != expected) return kSizeMismatch;
          if ((cursor + 7) / 8 != bytes) return kExtentMismatch;
          return 0;
        }
        if (kind == 1) { next = cursor; break; }
        const u32 carried = (s.flags >> 2) & 3u;
        if (carried < 2) final = carried;
      }
      continue;
    }
    BlockInfo info;
    const bool candidate = (bitmap[next >> 5] >> (next & 31)) & 1u;
    if (candidate) {
      info = parse_block(body, bytes, next, expected, 65536, fixed, dyn);
    } else {
      if (type == 1) return kFixedTiles;
      if (type == 2) return kUndiscovered;
      info = parse_block(body, bytes, next, expected - output, 0, fixed, dyn);
    }
    if (info.status) return info.status;
    if (info.end <= next || info.end > bits) return kExtentMismatch;
    if (info.size > expected - output) return kOutputOverflow;
    if (real_blocks >= max_blocks) return kBlockLimit;
    output += info.size;
    ++real_blocks;
    ++n;
    next = info.end;
    if (info.final) {
      if (output != expected) return kSizeMismatch;
      if ((next + 7) / 8 != bytes) return kExtentMismatch;
      return 0;
    }
  }
}

// Emission history check on an accepted chain: any distance beyond the
// declared window or before the stream start is status 6.
__device__ u32 history_walk(const u8* body, u64 bytes, u32 window, const Tables& fixed,
                            Tables& dyn) {
  BitCursor c;
  c.init(body, bytes, 0);
  u64 produced = 0;
  for (;;) {
    u32 err = 0;
    const u32 final = c.take(1, &err);
    const u32 type = c.take(2, &err);
    if (err) return 0;  // cannot happen after an accepted chain
    if (type == 0) {
      c.seek((c.pos + 7) & ~7ull);
      const u32 n = c.take(16, &err);
      c.take(16, &err);
      produced += n;
      c.seek(c.pos + u64(n) * 8);
    } else {
      if (type == 2 && serial_dynamic_header(c, dyn)) return 0;
      const Tables& t = type == 2 ? dyn : fixed;
      for (;;) {
        const Token tok = decode_token(c, t);
        if (tok.kind == kTokError) return 0;
        c.skip(tok.bits);
        if (tok.kind == kTokEnd) break;
        if (tok.kind == kTokLiteral) { ++produced; continue; }
        if (tok.dist > window || tok.dist > produced) return kBadDistance;
        produced += tok.length;
      }
    }
    if (final) return 0;
  }
}

struct GeneralShared {
  Tables fixed;
  Tables dyn;
};

// meta[0] holds the fast path's status on entry.  count/bitmap come from
// discover_kernel.  Writes the reference route's status to meta[0].
__global__ void general_status_kernel(const u8* in, u64 in_size, u64 expected, u32 max_candidates,
                                      u32 max_blocks, const u32* bitmap, const u32* count,
                                      u32* meta) {
  __shared__ GeneralShared sh;
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const u32 fast = meta[0];
  u32 window = 0, wanted = 0;
  u32 status = zlib_framing(in, in_size, &window, &wanted);
  if (!status) {
    const u64 body_bytes = in_size - 6;
    const u64 capacity = min_u64(u64(max_candidates), body_bytes * 9 + 1);
    if (*count > capacity) status = kCandidateOverflow;
    else if (!*count) status = kInitialBlockMissing;
  }
  // A fast path that reached the checksum accepted the chain and its history
  // with the reference's checks (the trailer plays no part in them), so the
  // route's status is the checksum's: no replay.
  if (!status && fast == kAdlerMismatch) status = kAdlerMismatch;
  if (!status && fast) {
    const u8* body = in + 2;
    const u64 bytes = in_size - 6;
    for (u32 i = 0; i < 288; ++i) sh.fixed.lens[i] = i < 144 ? 8 : i < 256 ? 9 : i < 280 ? 7 : 8;
    serial_build(sh.fixed.ll, sh.fixed.lens, 288, false, true, LLFn());
    for (u32 i = 0; i < 32; ++i) sh.fixed.lens[i] = 5;
    serial_build(sh.fixed.d, sh.fixed.lens, 32, false, true, DFn());
    status = chain_walk(body, bytes, bitmap, u32(expected), max_blocks, false, sh.fixed, sh.dyn);
    if (status == kFixedTiles)
      status = chain_walk(body, bytes, bitmap, u32(expected), max_blocks, true, sh.fixed, sh.dyn);
    if (!status) status = history_walk(body, bytes, window, sh.fixed, sh.dyn);
    if (!status) status = fast;
  }
  meta[0] = status;
  meta[1] = 0;
}

// Zero a failed output (grid-stride).
__global__ void clear_on_failure_kernel(const u32* meta, u8* out, u64 n) {
  if (!meta[0]) return;
  const u64 stride = u64(gridDim.x) * blockDim.x;
  for (u64 i = u64(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = 0;
}

cudaError_t launch_discover(const u8* in, u64 in_size, u32* bitmap, u32* extra, u32* count,
                            u32* queue, u32 queue_cap, u32* queued, const u32* gate,
                            const DeviceInfo& dev, cudaStream_t stream) {
  if (in_size < 8) return cudaSuccess;
  const u64 bytes = in_size - 6;
  u64 blocks = (bytes + kDiscoverTile - 1) / kDiscoverTile;
  const u64 cap = u64(dev.sms) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  profile_begin("discover_kernel", stream);
  note_launch();
  discover_kernel<<<u32(blocks), kDiscoverThreads, 0, stream>>>(in, in_size, bitmap, extra, count,
                                                                queue, queue_cap, queued, gate);
  profile_end(stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  profile_begin("validate_kernel", stream);
  note_launch();
  validate_kernel<<<u32(dev.sms) * 8, kDiscoverThreads, 0, stream>>>(
      in, in_size, queue, queue_cap, queued, bitmap, count, gate);
  profile_end(stream);
  return cudaGetLastError();
}

// Queue of prefiltered offsets: generous for any stream (config-1 streams
// queue one offset per ~160 body bytes); overflow is validated in place.
u32 discover_queue_capacity(u64 in_size) {
  const u64 body = in_size > 6 ? in_size - 6 : 0;
  return u32(std::min<u64>(body / 16 + 4096, u64(1) << 26));
}

cudaError_t launch_general_status(const u8* in, u64 in_size, u64 expected, u32 max_candidates,
                                  u32 max_blocks, const u32* bitmap, const u32* count, u32* meta,
                                  u8* out, cudaStream_t stream) {
  note_launch();
  general_status_kernel<<<1, 32, 0, stream>>>(in, in_size, expected, max_candidates, max_blocks,
                                              bitmap, count, meta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_clear_on_failure(meta, out, expected, stream);
}

cudaError_t launch_clear_on_failure(const u32* meta, u8* out, u64 expected, cudaStream_t stream) {
  if (!expected) return cudaSuccess;
  u64 blocks = (expected + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  note_launch();
  clear_on_failure_kernel<<<u32(blocks), 256, 0, stream>>>(meta, out, expected);
  return cudaGetLastError();
}

}  // namespace cz
