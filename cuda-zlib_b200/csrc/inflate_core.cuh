// Device-side RFC 1951 decoding primitives shared by every inflate kernel.
//
//  * BitCursor: LSB-first bit reader over a byte stream of any alignment.  It
//    only issues 8-byte-aligned 64-bit loads (an unaligned wide global load
//    faults), keeps a three-word register window so the word needed two steps
//    ahead is already in flight, and never loads a word past the one holding
//    the stream's last byte.  A peek returns 64 bits, enough for any whole
//    token (at most 15+5+15+13 = 48 bits), so one peek serves one token.
//  * Huffman tables: canonical codes, built cooperatively by one warp into
//    shared memory.  Literal/length codes use a 9-bit primary table, distance
//    codes 8 bits, code-length codes a complete 7-bit table; codes longer than
//    the primary width decode canonically from the bit-reversed window.
//  * Token decode with the reference's exact status precedence
//    (Huffman::decode and fixed_token / SmallTokenRemainder,
//    src/cuda_zlib/_decode_kernels.py:199-232,398-421 and
//    src/cuda_zlib/native/batch_decode.cuh:44-69): a field that would extend
//    past the end of the Deflate body is status 1, an unusable code status 4,
//    reserved symbols status 4.
#pragma once

#include <cstddef>

#include "common.cuh"

namespace cz {

// ---------------------------------------------------------------------------
// Bit cursor
// ---------------------------------------------------------------------------
struct BitCursor {
  const u64* words;  // 8-byte aligned, at or below the first body byte
  u32 shift;         // bit offset of body bit 0 inside words[0]
  u64 last;          // index of the last word holding a body byte
  u64 end;           // body length in bits
  u64 pos;           // next unread body bit
  u64 idx;           // word index of w0
  u64 w0, w1, w2;

  __device__ __forceinline__ u64 load(u64 i) const { return i <= last ? __ldg(words + i) : 0ull; }

  __device__ __forceinline__ void init(const u8* body, u64 bytes, u64 start_bit) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(body);
    words = reinterpret_cast<const u64*>(a & ~uintptr_t(7));
    shift = u32(a & 7) * 8;
    end = bytes * 8;
    last = bytes ? (u64(shift) + end - 1) >> 6 : 0;
    seek(start_bit);
  }

  __device__ __forceinline__ void seek(u64 p) {
    pos = p;
    idx = (u64(shift) + p) >> 6;
    w0 = load(idx);
    w1 = load(idx + 1);
    w2 = load(idx + 2);
  }

  // 64 bits starting at pos; bits at or past `end` are unspecified.
  __device__ __forceinline__ u64 peek() const {
    const u32 o = u32((u64(shift) + pos) & 63);
    return o ? (w0 >> o) | (w1 << (64 - o)) : w0;
  }

  __device__ __forceinline__ u64 avail() const { return pos <= end ? end - pos : 0; }

  // Advance by n <= 64 bits.  The window moves at most one word.
  __device__ __forceinline__ void skip(u32 n) {
    pos += n;
    const u64 q = (u64(shift) + pos) >> 6;
    if (q != idx) {
      w0 = w1;
      w1 = w2;
      w2 = load(idx + 3);
      ++idx;
    }
  }

  // Bounded read of n <= 32 bits (BitReader::take semantics): a read that
  // does not fit before `end` sets *error = 1 and consumes nothing.
  __device__ __forceinline__ u32 take(u32 n, u32* error) {
    if (*error) return 0;
    if (pos > end || n > end - pos) { *error = kTruncated; return 0; }
    if (!n) return 0;
    const u32 v = u32(peek() & ((n == 32) ? 0xffffffffull : ((1ull << n) - 1)));
    skip(n);
    return v;
  }
};

// ---------------------------------------------------------------------------
// Bits: the hot-loop reader.  A 64-bit accumulator holds 33..64 unread bits
// after refill(), filled from 4-byte-aligned 32-bit words; positions are u32
// (a stream's body is below 2^29 bytes, so its bit offsets fit).  The token loops read
// fields straight from the low word of the accumulator.
// ---------------------------------------------------------------------------
struct Bits {
  const u32* words;  // 4-byte aligned, at or below the first body byte
  u32 shift;         // bit offset of body bit 0 inside words[0]
  u32 last;          // index of the last word holding a body byte
  u32 end;           // body length in bits
  u32 idx;           // next word to load
  u32 nbits;         // valid bits in (hi:lo)
  u32 lo, hi;        // 64-bit accumulator; lo holds the next bits

  __device__ __forceinline__ u32 load(u32 i) const { return i <= last ? __ldg(words + i) : 0u; }

  __device__ __forceinline__ void init(const u8* body, u32 bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(body);
    words = reinterpret_cast<const u32*>(a & ~uintptr_t(3));
    shift = u32(a & 3) * 8;
    end = bytes * 8;
    last = bytes ? (shift + end - 1) >> 5 : 0;
    seek(0);
  }
  // Absolute position of the next unread body bit.
  __device__ __forceinline__ u32 pos() const { return idx * 32 - nbits - shift; }
  __device__ __forceinline__ u32 avail() const {
    const u32 p = pos();
    return p <= end ? end - p : 0;
  }
  __device__ __forceinline__ void seek(u32 p) {
    const u32 a = shift + p;
    idx = a >> 5;
    const u32 off = a & 31;
    lo = load(idx) >> off;
    hi = 0;
    nbits = 32 - off;
    ++idx;
    refill();
  }
  // Append one 32-bit word at bit nbits (nbits <= 32).
  __device__ __forceinline__ void append(u32 w) {
    lo |= w << nbits;                      // shifts of 32 give 0
    hi |= __funnelshift_lc(w, 0u, nbits);  // high word of w << nbits
    nbits += 32;
  }
  __device__ __forceinline__ void refill() {
    if (nbits <= 32) {
      append(load(idx));
      ++idx;
    }
  }
  // Unguarded refill: only while idx < last is known (fast loops).
  __device__ __forceinline__ void refill_fast() {
    if (nbits <= 32) {
      append(__ldg(words + idx));
      ++idx;
    }
  }
  // Drop n < 32 bits.
  __device__ __forceinline__ void consume(u32 n) {
    lo = __funnelshift_r(lo, hi, n);
    hi >>= n;
    nbits -= n;
  }
  // Bounded read of n <= 16 bits (BitReader::take semantics).
  __device__ __forceinline__ u32 take(u32 n, u32* error) {
    if (*error) return 0;
    if (n > avail()) { *error = kTruncated; return 0; }
    refill();
    const u32 v = lo & ((1u << n) - 1u);
    consume(n);
    return v;
  }
};

// ---------------------------------------------------------------------------
// Huffman tables
// ---------------------------------------------------------------------------
// Entry layout: [value:16][kind:4][extra:4][length:8].
enum EntryKind : u32 {
  kLiteral = 0,   // literal byte (LL) / usable distance (D)
  kLength = 1,    // length symbol 257..285
  kEnd = 2,       // end of block (256)
  kReserved = 3,  // 286/287 or distance 30/31: a decodable code, status 4
  kLong = 4,      // code longer than the primary width
  kHole = 5,      // prefix of no code (incomplete single-code trees)
  kEmpty = 6,     // empty distance tree: any decode is status 4
};

__device__ __forceinline__ u32 entry_len(u32 e) { return e & 0xffu; }
__device__ __forceinline__ u32 entry_extra(u32 e) { return (e >> 8) & 0xfu; }
__device__ __forceinline__ u32 entry_kind(u32 e) { return (e >> 12) & 0xfu; }
__device__ __forceinline__ u32 entry_value(u32 e) { return e >> 16; }
__device__ __forceinline__ u32 make_entry(u32 kind, u32 len, u32 extra, u32 value) {
  return (value << 16) | (kind << 12) | (extra << 8) | len;
}

__device__ __forceinline__ u32 length_base(u32 index) {
  const u32 extra = index < 8 || index == 28 ? 0 : (index >> 2) - 1;
  return index < 8 ? index + 3 : index == 28 ? 258 : 3 + ((4 + (index & 3)) << extra);
}
__device__ __forceinline__ u32 length_extra(u32 index) {
  return index < 8 || index == 28 ? 0 : (index >> 2) - 1;
}
__device__ __forceinline__ u32 dist_base(u32 index) {
  const u32 extra = index < 4 ? 0 : (index >> 1) - 1;
  return index < 4 ? index + 1 : 1 + ((2 + (index & 1)) << extra);
}
__device__ __forceinline__ u32 dist_extra(u32 index) { return index < 4 ? 0 : (index >> 1) - 1; }

// Literal/length entry for symbol s with code length L.
__device__ __forceinline__ u32 ll_entry(u32 s, u32 L) {
  if (s < 256) return make_entry(kLiteral, L, 0, s);
  if (s == 256) return make_entry(kEnd, L, 0, 0);
  if (s <= 285) return make_entry(kLength, L, length_extra(s - 257), length_base(s - 257));
  return make_entry(kReserved, L, 0, 0);
}
__device__ __forceinline__ u32 d_entry(u32 s, u32 L) {
  if (s < 30) return make_entry(kLiteral, L, dist_extra(s), dist_base(s));
  return make_entry(kReserved, L, 0, 0);
}
__device__ __forceinline__ u32 cl_entry(u32 s, u32 L) { return make_entry(kLiteral, L, 0, s); }

template <int Primary, int MaxSymbols>
struct Huffman {
  u32 lut[1 << Primary];
  u16 symbols[MaxSymbols];  // sorted by (length, symbol)
  u16 count[16];
  u16 offs[16];
  u32 first[16];            // canonical first code of each length (MSB-first)
  u32 maxlen;
};

constexpr u32 kLLBits = 9;  // literal/length primary table width
constexpr u32 kLLMask = (1u << kLLBits) - 1u;
typedef Huffman<kLLBits, 288> LLTable;
typedef Huffman<8, 32> DTable;
typedef Huffman<7, 19> CLTable;

struct Tables {
  LLTable ll;
  DTable d;
  CLTable cl;
  u8 lens[320];
  u32 scratch[32];
};

__device__ __forceinline__ u32 lanemask_lt() {
  u32 m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Build table `t` from lens[0..n) (shared memory).  All 32 lanes of the warp
// must call it; every lane returns the same status.  Validation follows
// Huffman::build (_decode_kernels.py:143-196): over-subscription, an
// incomplete code other than one length-1 code (when single_ok), or an empty
// code (unless empty_ok) is status 3.
template <int Primary, int MaxSymbols, typename EntryFn>
__device__ u32 warp_build(Huffman<Primary, MaxSymbols>& t, const u8* lens, u32 n, bool empty_ok,
                          bool single_ok, u32* scratch, EntryFn make) {
  const u32 lane = threadIdx.x & 31u;
  if (lane < 16) scratch[lane] = 0;
  __syncwarp();
  for (u32 base = 0; base < n; base += 32) {
    const u32 s = base + lane;
    const u32 len = s < n ? lens[s] : 0u;
    const u32 group = __match_any_sync(kFullMask, len);
    if (s < n && len && (group & lanemask_lt()) == 0) atomicAdd(&scratch[len], __popc(group));
  }
  __syncwarp();
  u32 status = 0;
  if (lane == 0) {
    u32 maximum = 0;
    for (u32 l = 1; l < 16; ++l) {
      t.count[l] = u16(scratch[l]);
      if (scratch[l]) maximum = l;
    }
    t.count[0] = 0;
    t.maxlen = maximum;
    if (!maximum) {
      status = empty_ok ? 0u : u32(kBadTree);
    } else {
      int left = 1;
      for (u32 l = 1; l < 16; ++l) {
        left = (left << 1) - int(scratch[l]);
        if (left < 0) break;
      }
      if (left < 0 || (left && !(single_ok && maximum == 1 && scratch[1] == 1))) status = kBadTree;
    }
    u32 code = 0, offset = 0;
    for (u32 l = 1; l < 16; ++l) {
      code = (code + t.count[l - 1]) << 1;
      t.first[l] = code;
      t.offs[l] = u16(offset);
      scratch[16 + l] = offset;  // placement cursor
      offset += t.count[l];
    }
  }
  status = __shfl_sync(kFullMask, status, 0);
  __syncwarp();
  if (status) return status;
  // Stable placement of symbols by length.
  for (u32 base = 0; base < n; base += 32) {
    const u32 s = base + lane;
    const u32 len = s < n ? lens[s] : 0u;
    const u32 group = __match_any_sync(kFullMask, len);
    const u32 rank = __popc(group & lanemask_lt());
    if (s < n && len) t.symbols[scratch[16 + len] + rank] = u16(s);
    __syncwarp();
    if (s < n && len && rank == 0) scratch[16 + len] += __popc(group);
    __syncwarp();
  }
  // Primary table, one entry per lane at a time.
  const u32 maximum = t.maxlen;
  for (u32 k = lane; k < (1u << Primary); k += 32) {
    u32 entry;
    if (!maximum) {
      entry = make_entry(kEmpty, 0, 0, 0);
    } else {
      const u32 v = __brev(k) >> (32 - Primary);  // MSB-first code prefix
      entry = make_entry(maximum > u32(Primary) ? kLong : kHole, 0, 0, 0);
      const u32 top = maximum < u32(Primary) ? maximum : u32(Primary);
      for (u32 L = 1; L <= top; ++L) {
        const u32 c = v >> (Primary - L);
        const u32 i = c - t.first[L];
        if (i < t.count[L]) {
          entry = make(t.symbols[t.offs[L] + i], L);
          break;
        }
      }
    }
    t.lut[k] = entry;
  }
  __syncwarp();
  return 0;
}

// Canonical decode of a code longer than the primary width from `bits`
// (LSB-first stream order).  Returns the packed entry or a kHole entry.
template <int Primary, int MaxSymbols, typename EntryFn>
__device__ __forceinline__ u32 decode_long(const Huffman<Primary, MaxSymbols>& t, u64 bits,
                                           EntryFn make) {
  const u32 r = __brev(u32(bits & 0x7fffu)) >> 17;  // 15 bits, MSB-first
  for (u32 L = Primary + 1; L <= t.maxlen; ++L) {
    const u32 c = r >> (15 - L);
    const u32 i = c - t.first[L];
    if (i < t.count[L]) return make(t.symbols[t.offs[L] + i], L);
  }
  return make_entry(kHole, 0, 0, 0);
}

struct LLFn {
  __device__ __forceinline__ u32 operator()(u32 s, u32 L) const { return ll_entry(s, L); }
};
struct DFn {
  __device__ __forceinline__ u32 operator()(u32 s, u32 L) const { return d_entry(s, L); }
};
struct CLFn {
  __device__ __forceinline__ u32 operator()(u32 s, u32 L) const { return cl_entry(s, L); }
};

// Fixed Huffman tables (RFC 1951 3.2.6; fixed_tables, _decode_kernels.py:289-296).
__device__ inline void warp_build_fixed(Tables& t) {
  const u32 lane = threadIdx.x & 31u;
  for (u32 i = lane; i < 288; i += 32) t.lens[i] = i < 144 ? 8 : i < 256 ? 9 : i < 280 ? 7 : 8;
  __syncwarp();
  warp_build(t.ll, t.lens, 288, false, true, t.scratch, LLFn());
  for (u32 i = lane; i < 32; i += 32) t.lens[i] = 5;
  __syncwarp();
  warp_build(t.d, t.lens, 32, false, true, t.scratch, DFn());
}

// Rendezvous actions: lane 0 parses, then the whole warp performs one action.
enum Action : u32 {
  kNone = 0, kStored = 1, kCopy = 2, kDynamic = 3, kFlush = 4, kFixed = 5, kRound = 6
};

// Copy the decode part of the fixed tables (literal/length and distance)
// into a warp's shared-memory tables, so hot loops only read shared memory.
__device__ inline void warp_load_fixed(Tables& dst, const Tables& fixed) {
  const u32 lane = threadIdx.x & 31u;
  const u32* from = reinterpret_cast<const u32*>(&fixed);
  u32* to = reinterpret_cast<u32*>(&dst);
  const u32 words = (offsetof(Tables, cl) + 3) / 4;
  for (u32 i = lane; i < words; i += 32) to[i] = __ldg(from + i);
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Token decode
// ---------------------------------------------------------------------------
enum TokenKind : u32 { kTokLiteral = 0, kTokMatch = 1, kTokEnd = 2, kTokError = 3 };

struct Token {
  u32 kind;
  u32 value;   // literal byte
  u32 length;  // match length
  u32 dist;    // match distance
  u32 bits;    // bits consumed
  u32 error;   // status when kind == kTokError
};

// Decode one literal/length token (and its distance) at the cursor without
// consuming it.  Status precedence follows the reference decoders: the
// literal/length code (1 truncated, 4 unusable), reserved symbols 286/287
// (4), length extra bits (1), the distance code (1/4), reserved distances
// 30/31 (4), distance extra bits (1).  Window and history checks are the
// caller's, because the two reference routes order them differently.
__device__ __forceinline__ Token decode_token(const BitCursor& c, const Tables& t) {
  Token tok;
  tok.kind = kTokError;
  tok.value = tok.length = tok.dist = tok.bits = 0;
  tok.error = 0;
  const u64 v = c.peek();
  const u64 avail = c.avail();
  u32 e = t.ll.lut[v & kLLMask];
  u32 kind = entry_kind(e);
  if (kind == kLong) {
    e = decode_long(t.ll, v, LLFn());
    kind = entry_kind(e);
  }
  if (kind == kHole) {
    tok.error = avail >= t.ll.maxlen ? kBadSymbol : kTruncated;
    return tok;
  }
  const u32 L = entry_len(e);
  if (L > avail) { tok.error = kTruncated; return tok; }
  if (kind == kLiteral) {
    tok.kind = kTokLiteral;
    tok.value = entry_value(e);
    tok.bits = L;
    return tok;
  }
  if (kind == kEnd) {
    tok.kind = kTokEnd;
    tok.bits = L;
    return tok;
  }
  if (kind == kReserved) { tok.error = kBadSymbol; return tok; }
  const u32 E = entry_extra(e);
  if (L + E > avail) { tok.error = kTruncated; return tok; }
  tok.length = entry_value(e) + u32((v >> L) & ((1u << E) - 1u));
  const u32 at = L + E;
  u32 d = t.d.lut[(v >> at) & 255u];
  u32 dk = entry_kind(d);
  if (dk == kLong) {
    d = decode_long(t.d, v >> at, DFn());
    dk = entry_kind(d);
  }
  if (dk == kEmpty) { tok.error = kBadSymbol; return tok; }
  if (dk == kHole) {
    tok.error = avail - at >= t.d.maxlen ? kBadSymbol : kTruncated;
    return tok;
  }
  const u32 Ld = entry_len(d);
  if (at + Ld > avail) { tok.error = kTruncated; return tok; }
  if (dk == kReserved) { tok.error = kBadSymbol; return tok; }
  const u32 Ed = entry_extra(d);
  if (at + Ld + Ed > avail) { tok.error = kTruncated; return tok; }
  tok.dist = entry_value(d) + u32((v >> (at + Ld)) & ((1u << Ed) - 1u));
  tok.bits = at + Ld + Ed;
  tok.kind = kTokMatch;
  return tok;
}

// Exact token decode on Bits, consuming it.  Same status precedence as
// decode_token; after an error the reader state is unspecified (errors end
// the stream).
__device__ __forceinline__ Token take_token(Bits& b, const Tables& t) {
  Token tok;
  tok.kind = kTokError;
  tok.value = tok.length = tok.dist = tok.bits = 0;
  tok.error = 0;
  const u32 avail = b.avail();
  b.refill();
  u32 v = b.lo;
  u32 e = t.ll.lut[v & kLLMask];
  u32 kind = entry_kind(e);
  if (kind == kLong) {
    e = decode_long(t.ll, v, LLFn());
    kind = entry_kind(e);
  }
  if (kind == kHole) {
    tok.error = avail >= t.ll.maxlen ? kBadSymbol : kTruncated;
    return tok;
  }
  const u32 L = entry_len(e);
  if (L > avail) { tok.error = kTruncated; return tok; }
  if (kind == kLiteral || kind == kEnd) {
    tok.kind = kind == kLiteral ? kTokLiteral : kTokEnd;
    tok.value = entry_value(e);
    tok.bits = L;
    b.consume(L);
    return tok;
  }
  if (kind == kReserved) { tok.error = kBadSymbol; return tok; }
  const u32 E = entry_extra(e);
  if (L + E > avail) { tok.error = kTruncated; return tok; }
  tok.length = entry_value(e) + ((v >> L) & ((1u << E) - 1u));
  b.consume(L + E);
  const u32 left = avail - (L + E);
  b.refill();
  v = b.lo;
  u32 d = t.d.lut[v & 255u];
  u32 dk = entry_kind(d);
  if (dk == kLong) {
    d = decode_long(t.d, v, DFn());
    dk = entry_kind(d);
  }
  if (dk == kEmpty) { tok.error = kBadSymbol; return tok; }
  if (dk == kHole) {
    tok.error = left >= t.d.maxlen ? kBadSymbol : kTruncated;
    return tok;
  }
  const u32 Ld = entry_len(d);
  if (Ld > left) { tok.error = kTruncated; return tok; }
  if (dk == kReserved) { tok.error = kBadSymbol; return tok; }
  const u32 Ed = entry_extra(d);
  if (Ld + Ed > left) { tok.error = kTruncated; return tok; }
  tok.dist = entry_value(d) + ((v >> Ld) & ((1u << Ed) - 1u));
  b.consume(Ld + Ed);
  tok.bits = L + E + Ld + Ed;
  tok.kind = kTokMatch;
  return tok;
}

// Dynamic block header, lane 0 reading and the warp building tables
// (dynamic_tables, _decode_kernels.py:240-287).  All lanes call; lane 0's
// cursor is the one that advances.  Returns the status on every lane.
// One code-length symbol (complete 7-bit table); 1 if it does not fit.
__device__ __forceinline__ u32 cl_symbol(BitCursor& c, const Tables& t, u32* err) {
  const u32 e = t.cl.lut[c.peek() & 127u];
  if (entry_len(e) > c.avail()) { *err = kTruncated; return 0; }
  c.skip(entry_len(e));
  return entry_value(e);
}
__device__ __forceinline__ u32 cl_symbol(Bits& c, const Tables& t, u32* err) {
  const u32 avail = c.avail();
  c.refill();
  const u32 e = t.cl.lut[c.lo & 127u];
  if (entry_len(e) > avail) { *err = kTruncated; return 0; }
  c.consume(entry_len(e));
  return entry_value(e);
}

template <typename Reader>
__device__ u32 warp_dynamic_header(Reader& c, Tables& t) {
  const u32 lane = threadIdx.x & 31u;
  u32 err = 0, nl = 0, nd = 0, nc = 0;
  if (lane == 0) {
    nl = c.take(5, &err) + 257;
    nd = c.take(5, &err) + 1;
    nc = c.take(4, &err) + 4;
    if (!err && nl > 286) err = kBadTree;
    if (!err) {
      u8 clens[19];
      for (u32 i = 0; i < 19; ++i) clens[i] = 0;
      const u8 order[19] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};
      for (u32 i = 0; i < nc; ++i) clens[order[i]] = u8(c.take(3, &err));
      for (u32 i = 0; i < 19; ++i) t.lens[i] = clens[i];
    }
  }
  err = __shfl_sync(kFullMask, err, 0);
  if (err) return err;
  __syncwarp();
  err = warp_build(t.cl, t.lens, 19, false, false, t.scratch, CLFn());
  if (err) return err;
  nl = __shfl_sync(kFullMask, nl, 0);
  nd = __shfl_sync(kFullMask, nd, 0);
  if (lane == 0) {
    u32 i = 0;
    while (i < nl + nd) {
      const u32 sym = cl_symbol(c, t, &err);
      if (err) break;
      if (sym < 16) { t.lens[i++] = u8(sym); continue; }
      u32 repeat, value;
      if (sym == 16) {
        if (!i) { err = kBadRepeat; break; }
        repeat = c.take(2, &err) + 3;
        value = t.lens[i - 1];
      } else if (sym == 17) {
        repeat = c.take(3, &err) + 3;
        value = 0;
      } else {
        repeat = c.take(7, &err) + 11;
        value = 0;
      }
      if (err) break;
      if (repeat > nl + nd - i) { err = kBadRepeat; break; }
      for (u32 j = 0; j < repeat; ++j) t.lens[i++] = u8(value);
    }
    if (!err && !t.lens[256]) err = kBadTree;
  }
  err = __shfl_sync(kFullMask, err, 0);
  if (err) return err;
  __syncwarp();
  err = warp_build(t.ll, t.lens, nl, false, true, t.scratch, LLFn());
  if (err) return err;
  // Distance lengths follow the literal/length lengths; copy them down so
  // the builder reads a zero-based array.
  u8* dl = t.lens + 288;
  const u8 dv = lane < nd ? t.lens[nl + lane] : u8(0);  // nd <= 32: one per lane
  __syncwarp();
  if (lane < nd) dl[lane] = dv;
  __syncwarp();
  return warp_build(t.d, dl, nd, true, true, t.scratch, DFn());
}

}  // namespace cz
