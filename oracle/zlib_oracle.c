/*
 * zlib_oracle.c -- CPU restatement of xangma/cuda-zlib's codec semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped product links, loads or
 * calls this file: it is the checker that the CUDA path is compared against
 * (tests/, __graft_entry__.smoke(), and bench.py's cpu_baseline / reference
 * arm).  The product fails loudly when its CUDA library is missing; it never
 * falls back to this code.
 *
 * Parity pin: the encoder reproduces the 38 SHA-256-frozen streams of the
 * reference tests (tests/test_encode.py:52-70, tests/test_encode_match.py:26-57,
 * tests/test_encode_bounds.py:16-35); the decoder reproduces every status the
 * reference tests assert for hand-built streams (tests/test_decode.py,
 * tests/test_regressions.py).  Golden vectors live in tests/golden/.
 *
 * Citations are paths inside the reference project (src/cuda_zlib/...).
 * All arithmetic is integer; nothing here is floating point.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef uint8_t u8;
typedef uint16_t u16;
typedef uint32_t u32;
typedef uint64_t u64;

#define MAX_BYTES (1u << 28)        /* _codec.py:13, codec_ffi.cu:42 */
/* Single-stream bounds of this codec, a deliberate superset of the
 * reference's 2**28 (_codec.py:13,28,103): one stream may decode to 2**31
 * bytes from at most 2**29 - 2**16 compressed bytes (bit offsets stay below
 * 2**32), and compress up to 2**31 input bytes.  Batch calls keep 2**28. */
#define MAX_STREAM_BYTES (1u << 31)
#define MAX_STREAM_INPUT ((1u << 29) - (1u << 16))
/* Chunk sizes: the reference accepts [256, 65535] (_codec.py:158-159); this
 * codec also accepts chunks up to 2**18, whose stored fallback is split into
 * blocks of at most 65535 bytes. */
#define MAX_CHUNK_BYTES 262144u
#define STORED_MAX 65535u
#define MAX_CANDIDATES 262144u      /* _codec.py:14 */
#define MAX_BLOCKS 262144u          /* _codec.py:15 */

/* Status codes: 1..13 _decode_kernels.py:36-50; 14..23 codec_ffi.cu:51-62. */
enum {
  ST_OK = 0, ST_TRUNCATED = 1, ST_RESERVED_TYPE = 2, ST_BAD_TREE = 3,
  ST_BAD_SYMBOL = 4, ST_BAD_REPEAT = 5, ST_BAD_DISTANCE = 6,
  ST_OUTPUT_OVERFLOW = 7, ST_BLOCK_LIMIT = 9, ST_UNDISCOVERED = 10,
  ST_SIZE_MISMATCH = 11, ST_EXTENT_MISMATCH = 12, ST_FIXED_TILES = 13,
  ST_TRUNCATED_ZLIB = 14, ST_BAD_HEADER = 15, ST_GZIP = 16, ST_DICTIONARY = 17,
  ST_CANDIDATE_OVERFLOW = 18, ST_NO_INITIAL_BLOCK = 19, ST_DEPTH = 20,
  ST_ADLER = 21, ST_COMPRESSION_OVERFLOW = 22, ST_BOUNDS = 23
};

/* ------------------------------------------------------------------ */
/* Adler-32 (RFC 1950 section 8.2).                                    */
/* ------------------------------------------------------------------ */
u32 oracle_adler32(const u8* data, u64 n) {
  u64 a = 1, b = 0;
  u64 i = 0;
  while (i < n) {
    u64 stop = i + 4096 < n ? i + 4096 : n;
    for (; i < stop; ++i) { a += data[i]; b += a; }
    a %= 65521u;
    b %= 65521u;
  }
  return (u32)((b << 16) | a);
}

/* ------------------------------------------------------------------ */
/* Bounded LSB-first bit reader (follows BitReader,                    */
/* _decode_kernels.py:69-124: any read past `bits` sets error 1, a     */
/* zero-width read never fails).                                       */
/* ------------------------------------------------------------------ */
typedef struct {
  const u8* data;
  u64 bits;
  u64 pos;
  u32 error;
} Reader;

static u32 rd_take(Reader* r, u32 n) {
  if (r->error) return 0;
  if (r->pos > r->bits || n > r->bits - r->pos) { r->error = ST_TRUNCATED; return 0; }
  if (!n) return 0;
  /* n <= 16, so at most three bytes hold the field; all lie below `bits`. */
  u64 byte = r->pos >> 3;
  u32 skip = (u32)(r->pos & 7), need = (skip + n + 7) >> 3, w = 0;
  for (u32 i = 0; i < need; ++i) w |= (u32)r->data[byte + i] << (8 * i);
  r->pos += n;
  return (w >> skip) & ((1u << n) - 1u);
}

/* ------------------------------------------------------------------ */
/* Canonical Huffman code (follows Huffman<N,P>::build/decode,          */
/* _decode_kernels.py:135-232).  The reference's primary lookup table  */
/* is only a cache of this canonical decode, so the oracle decodes     */
/* bit by bit: identical symbols, identical error 1 / error 4 cases.   */
/* ------------------------------------------------------------------ */
#define LUT_BITS 10
typedef struct {
  u16 count[16];
  u16 symbols[320];
  u32 maximum;
  u16 lut[1u << LUT_BITS];  /* (length << 9) | symbol for codes <= LUT_BITS, else 0 */
} Code;

static u32 code_build(Code* c, const u8* lens, u32 n, int empty_ok, int single_ok,
                      u32 limit) {
  memset(c->count, 0, sizeof(c->count));
  c->maximum = 0;
  for (u32 i = 0; i < n; ++i) {
    if (lens[i] > limit) return ST_BAD_TREE;
    c->count[lens[i]]++;
    if (lens[i] > c->maximum) c->maximum = lens[i];
  }
  if (!c->maximum) return empty_ok ? 0 : ST_BAD_TREE;
  int left = 1;
  for (u32 l = 1; l <= limit; ++l) {
    left = (left << 1) - c->count[l];
    if (left < 0) return ST_BAD_TREE;  /* oversubscribed */
  }
  /* Incomplete codes are legal only as one code of length one. */
  if (left && !(single_ok && c->maximum == 1 && c->count[1] == 1)) return ST_BAD_TREE;
  u16 offset[16];
  offset[1] = 0;
  for (u32 l = 1; l < 15; ++l) offset[l + 1] = offset[l] + c->count[l];
  for (u32 i = 0; i < n; ++i)
    if (lens[i]) c->symbols[offset[lens[i]]++] = (u16)i;
  /* Lookup cache: canonical codes are assigned in (length, symbol) order. */
  memset(c->lut, 0, sizeof(c->lut));
  u32 code = 0, index = 0;
  for (u32 len = 1; len <= LUT_BITS; ++len) {
    for (u32 j = 0; j < c->count[len]; ++j) {
      u32 rev = 0, v = code + j;
      for (u32 b = 0; b < len; ++b) rev |= ((v >> b) & 1u) << (len - 1 - b);
      for (u32 k = rev; k < (1u << LUT_BITS); k += 1u << len)
        c->lut[k] = (u16)((len << 9) | c->symbols[index + j]);
    }
    index += c->count[len];
    code = (code + c->count[len]) << 1;
  }
  return 0;
}

static int code_decode(const Code* c, Reader* r) {
  if (!r->error && r->pos <= r->bits && r->bits - r->pos >= LUT_BITS) {
    u64 byte = r->pos >> 3;
    u32 skip = (u32)(r->pos & 7), need = (skip + LUT_BITS + 7) >> 3, w = 0;
    for (u32 i = 0; i < need; ++i) w |= (u32)r->data[byte + i] << (8 * i);
    u16 e = c->lut[(w >> skip) & ((1u << LUT_BITS) - 1u)];
    if (e) { r->pos += e >> 9; return e & 511; }
  }
  u32 code = 0, first = 0, index = 0;
  for (u32 len = 1; len <= c->maximum; ++len) {
    code |= rd_take(r, 1);
    if (r->error) return -1;
    if (code < first + c->count[len]) return (int)c->symbols[index + code - first];
    index += c->count[len];
    first = (first + c->count[len]) << 1;
    code <<= 1;
  }
  r->error = ST_BAD_SYMBOL;
  return -1;
}

typedef struct { Code ll, dd, cl; } Tables;

static const u8 kClOrder[19] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};

/* Dynamic header (follows dynamic_tables, _decode_kernels.py:240-287). */
static u32 dynamic_tables(Reader* r, Tables* t) {
  u32 nl = rd_take(r, 5) + 257;
  u32 nd = rd_take(r, 5) + 1;
  u32 nc = rd_take(r, 4) + 4;
  if (r->error) return r->error;
  if (nl > 286) return ST_BAD_TREE;
  u8 clens[19] = {0};
  for (u32 i = 0; i < nc; ++i) clens[kClOrder[i]] = (u8)rd_take(r, 3);
  if (r->error) return r->error;
  u32 err = code_build(&t->cl, clens, 19, 0, 0, 7);
  if (err) return err;
  u8 lens[320];
  u32 i = 0;
  while (i < nl + nd) {
    int sym = code_decode(&t->cl, r);
    if (r->error) return r->error;
    if (sym < 16) { lens[i++] = (u8)sym; continue; }
    u32 repeat, value;
    if (sym == 16) {
      if (!i) return ST_BAD_REPEAT;
      repeat = rd_take(r, 2) + 3;
      value = lens[i - 1];
    } else if (sym == 17) {
      repeat = rd_take(r, 3) + 3;
      value = 0;
    } else {
      repeat = rd_take(r, 7) + 11;
      value = 0;
    }
    if (r->error) return r->error;
    if (repeat > nl + nd - i) return ST_BAD_REPEAT;
    for (u32 j = 0; j < repeat; ++j) lens[i++] = (u8)value;
  }
  if (!lens[256]) return ST_BAD_TREE;
  u32 e = code_build(&t->ll, lens, nl, 0, 1, 15);
  if (e) return e;
  return code_build(&t->dd, lens + nl, nd, 1, 1, 15);
}

/* Fixed tables (fixed_tables, _decode_kernels.py:289-296). */
static u32 fixed_tables(Tables* t) {
  u8 lens[288];
  for (u32 i = 0; i < 288; ++i) lens[i] = i < 144 ? 8 : i < 256 ? 9 : i < 280 ? 7 : 8;
  u32 e = code_build(&t->ll, lens, 288, 0, 1, 15);
  for (u32 i = 0; i < 32; ++i) lens[i] = 5;
  return e ? e : code_build(&t->dd, lens, 32, 0, 1, 15);
}

static u32 length_base(u32 index) {
  u32 extra = index < 8 || index == 28 ? 0 : (index >> 2) - 1;
  return index < 8 ? index + 3 : index == 28 ? 258 : 3 + ((4 + (index & 3)) << extra);
}
static u32 length_extra(u32 index) { return index < 8 || index == 28 ? 0 : (index >> 2) - 1; }
static u32 dist_base(u32 index) {
  u32 extra = index < 4 ? 0 : (index >> 1) - 1;
  return index < 4 ? index + 1 : 1 + ((2 + (index & 1)) << extra);
}
static u32 dist_extra(u32 index) { return index < 4 ? 0 : (index >> 1) - 1; }

/* One token after its literal/length symbol.  `window_first` selects the
 * serial decoder's order (window check inside the token, before the output
 * bound: SmallTokenRemainder, batch_decode.cuh:44-69); otherwise the caller
 * checks the output bound first (parse_block, _decode_kernels.py:744-757). */
static int token_rest(Reader* r, const Tables* t, int sym, u32* size, u32* dist,
                      u32 window, int window_first) {
  *size = 0;
  *dist = 0;
  if (r->error || sym == 256) return sym;
  if (sym < 256) { *size = 1; return sym; }
  if (sym > 285) { r->error = ST_BAD_SYMBOL; return sym; }
  u32 idx = (u32)sym - 257;
  *size = length_base(idx) + rd_take(r, length_extra(idx));
  if (r->error) return sym;
  int ds = code_decode(&t->dd, r);
  if (r->error) return sym;
  if (ds < 0 || ds > 29) { r->error = ST_BAD_SYMBOL; return sym; }
  *dist = dist_base((u32)ds) + rd_take(r, dist_extra((u32)ds));
  if (window_first && !r->error && (!*dist || *dist > window)) r->error = ST_BAD_DISTANCE;
  return sym;
}

static u32 zlib_framing(const u8* in, u64 size, u32* window, u32* wanted) {
  if (size < 8) return ST_TRUNCATED_ZLIB;
  u32 cmf = in[0], flg = in[1];
  if (cmf == 0x1f && flg == 0x8b) return ST_GZIP;
  if ((cmf & 15) != 8 || (cmf >> 4) > 7 || (cmf * 256 + flg) % 31) return ST_BAD_HEADER;
  if (flg & 32) return ST_DICTIONARY;
  *window = 1u << ((cmf >> 4) + 8);
  *wanted = ((u32)in[size - 4] << 24) | ((u32)in[size - 3] << 16) |
            ((u32)in[size - 2] << 8) | (u32)in[size - 1];
  return 0;
}

/* ------------------------------------------------------------------ */
/* Serial route (follows DecodeOneFile, batch_decode.cuh:123-296): the  */
/* small single-stream route and every batch file.                     */
/* ------------------------------------------------------------------ */
u32 oracle_inflate_serial(const u8* in, u64 in_size, u8* out, u64 out_size, u32 max_blocks) {
  if (in_size > MAX_BYTES || out_size > MAX_BYTES || !max_blocks || max_blocks > MAX_BLOCKS)
    return ST_BOUNDS;
  memset(out, 0, out_size);
  u32 window = 0, wanted = 0;
  u32 err = zlib_framing(in, in_size, &window, &wanted);
  if (err) return err;
  Reader r = {in + 2, (in_size - 6) * 8, 0, 0};
  Tables* t = (Tables*)malloc(sizeof(Tables));
  u64 produced = 0;
  u32 final = 0, blocks = 0;
  int need_header = 1, complete = 0;
  while (!complete) {
    if (need_header) {
      if (blocks >= max_blocks) { err = ST_BLOCK_LIMIT; goto done; }
      ++blocks;
      final = rd_take(&r, 1);
      u32 type = rd_take(&r, 2);
      if (r.error) { err = r.error; goto done; }
      if (type == 3) { err = ST_RESERVED_TYPE; goto done; }
      if (type == 0) {
        r.pos = (r.pos + 7) & ~(u64)7;
        u32 n = rd_take(&r, 16), comp = rd_take(&r, 16);
        if (r.error) { err = r.error; goto done; }
        if ((n ^ comp) != 65535u) { err = ST_BAD_SYMBOL; goto done; }
        if (n > out_size - produced) { err = ST_OUTPUT_OVERFLOW; goto done; }
        if (r.pos > r.bits || (u64)n * 8 > r.bits - r.pos) { err = ST_TRUNCATED; goto done; }
        memcpy(out + produced, r.data + (r.pos >> 3), n);
        produced += n;
        r.pos += (u64)n * 8;
        complete = final != 0;
        continue;
      }
      err = type == 1 ? fixed_tables(t) : dynamic_tables(&r, t);
      need_header = 0;
      if (err) goto done;
    }
    u32 size, dist;
    int sym = code_decode(&t->ll, &r);
    sym = token_rest(&r, t, sym, &size, &dist, window, 1);
    if (r.error) { err = r.error; goto done; }
    if (sym == 256) { complete = final != 0; need_header = 1; continue; }
    if (size > out_size - produced) { err = ST_OUTPUT_OVERFLOW; goto done; }
    if (!dist) { out[produced++] = (u8)sym; continue; }
    if (dist > produced) { err = ST_BAD_DISTANCE; goto done; }
    for (u32 j = 0; j < size; ++j) out[produced + j] = out[produced + j - dist];
    produced += size;
  }
  if (produced != out_size) err = ST_SIZE_MISMATCH;
  else if ((r.pos + 7) / 8 != in_size - 6) err = ST_EXTENT_MISMATCH;
  else if (oracle_adler32(out, out_size) != wanted) err = ST_ADLER;
done:
  free(t);
  return err;
}

/* ------------------------------------------------------------------ */
/* General route (single streams outside the small route): speculative  */
/* candidate discovery, per-candidate description, exact chain walk     */
/* with fixed-tile retry, then emission history checks and Adler-32.    */
/* Follows codec_ffi.cu:662-950 and _decode_kernels.py:298-1447.        */
/* ------------------------------------------------------------------ */
typedef struct {
  u64 end;
  u32 size, final, status;
} Block;

/* parse_block<false> (_decode_kernels.py:683-781): no history, the given
 * output limit, window 32768, optional fixed budget (status 13). */
static Block parse_block(const u8* data, u32 bytes, u64 start, u32 limit, u32 fixed_budget,
                         Tables* t) {
  Reader r = {data, (u64)bytes * 8, start, 0};
  Block b = {start, 0, 0, 0};
  b.final = rd_take(&r, 1);
  u32 type = rd_take(&r, 2);
  if (r.error) { b.status = r.error; return b; }
  if (type == 3) { b.status = ST_RESERVED_TYPE; return b; }
  u32 produced = 0;
  if (type == 0) {
    r.pos = (r.pos + 7) & ~(u64)7;
    u32 n = rd_take(&r, 16), comp = rd_take(&r, 16);
    if (r.error) { b.status = r.error; return b; }
    if ((n ^ comp) != 65535u) { b.status = ST_BAD_SYMBOL; return b; }
    if (n > limit) { b.status = ST_OUTPUT_OVERFLOW; return b; }
    if (r.pos > r.bits || (u64)n * 8 > r.bits - r.pos) { b.status = ST_TRUNCATED; return b; }
    produced = n;
    r.pos += (u64)n * 8;
  } else {
    u32 err = type == 1 ? fixed_tables(t) : dynamic_tables(&r, t);
    if (err) { b.status = err; return b; }
    while (!r.error) {
      if (type == 1 && fixed_budget &&
          (produced >= fixed_budget || r.pos - start >= (u64)fixed_budget * 8)) {
        r.error = ST_FIXED_TILES;
        break;
      }
      u32 size, dist;
      int sym = code_decode(&t->ll, &r);
      if (r.error) break;
      if (sym == 256) break;
      if (sym < 256) {
        if (produced >= limit) { r.error = ST_OUTPUT_OVERFLOW; break; }
        ++produced;
        continue;
      }
      token_rest(&r, t, sym, &size, &dist, 32768, 0);
      if (r.error) break;
      if (size > limit - produced) { r.error = ST_OUTPUT_OVERFLOW; break; }
      if (!dist || dist > 32768) { r.error = ST_BAD_DISTANCE; break; }
      produced += size;
    }
  }
  b.end = r.pos;
  b.size = produced;
  b.status = r.error;
  return b;
}

/* Candidate rules of discover (_decode_kernels.py:998-1054). */
static int dynamic_valid(const u8* data, u32 bytes, u64 start, Tables* t) {
  Reader r = {data, (u64)bytes * 8, start, 0};
  u32 final = rd_take(&r, 1);
  u32 type = rd_take(&r, 2);
  (void)final;
  if (r.error || type != 2) return 0;
  return dynamic_tables(&r, t) == 0;
}

static int stored_seed_at(const u8* data, u32 bytes, u64 byte, u64* endpoint) {
  u64 available = (u64)bytes - byte;
  if (!byte || available < 5) return 0;
  u32 n = data[byte] | ((u32)data[byte + 1] << 8);
  u32 comp = data[byte + 2] | ((u32)data[byte + 3] << 8);
  if ((n ^ comp) != 65535u || (u64)n + 4 >= available) return 0;
  u32 before = (u32)data[byte - 1] << 8;
  if (byte >= 2) before |= data[byte - 2];
  int possible = 0;
  for (u32 gap = 3; gap <= 10; ++gap)
    if (byte * 8 >= gap && ((before >> (17 - gap)) & 3u) == 0) possible = 1;
  u64 e = byte + 4 + n;
  if (!possible || ((data[e] >> 1) & 3u) != 1) return 0;
  *endpoint = e;
  return 1;
}

/* Candidate set as a bitmap over bit offsets and the raw event count
 * (duplicates included, as the reference's atomic counter counts them). */
static u64 discover(const u8* data, u32 bytes, u8* bitmap, Tables* t) {
  u64 count = 0;
  for (u64 byte = 0; byte < bytes; ++byte) {
    u64 e;
    if (stored_seed_at(data, bytes, byte, &e)) {
      ++count;
      bitmap[e] |= 1;  /* seed at bit e*8 */
    }
    for (u32 bit = 0; bit < 8; ++bit) {
      u64 start = byte * 8 + bit;
      if (start == 0 || dynamic_valid(data, bytes, start, t)) {
        ++count;
        bitmap[byte] |= (u8)(1u << bit);
      }
    }
  }
  return count;
}

typedef struct {
  u64 end, first_end;
  u32 size, first_size, flags, status;
} Summary;

/* scan_fixed_region (_decode_kernels.py:444-472). */
static Summary scan_fixed(const u8* data, u32 bytes, u64 entry, u64 tile_end, const Tables* t) {
  Reader r = {data, (u64)bytes * 8, entry, entry >= (u64)bytes * 8 ? 1u : 0u};
  Summary s = {entry, ~(u64)0, 0, 0, 0, 0};
  u32 ended = 0, final = 2, kind = 0;
  while (r.pos < tile_end && !r.error) {
    u32 size, dist;
    int sym = code_decode(&t->ll, &r);
    sym = token_rest(&r, t, sym, &size, &dist, 32768, 1);
    if (r.error) break;
    if (sym != 256) { s.size += size; continue; }
    if (s.first_end == ~(u64)0) { s.first_end = r.pos; s.first_size = s.size; }
    ++ended;
    if (final == 1) { kind = 2; break; }
    if (r.pos >= tile_end) { kind = 1; break; }
    u64 header = r.pos;
    u32 next_final = rd_take(&r, 1), type = rd_take(&r, 2);
    if (r.error) break;
    if (type != 1) { r.pos = header; kind = 1; break; }
    final = next_final;
  }
  s.end = r.pos;
  s.flags = kind | (final << 2) | (ended << 4);
  s.status = r.error;
  return s;
}

#define TILE_BYTES 2048u  /* FIXED_TILE_BYTES, _decode_kernels.py:52 */

/* select_chain_impl (_decode_kernels.py:1226-1408) with both passes.
 * Records blocks (start, size, prefix) for emission. */
typedef struct {
  u64 start;       /* bit offset of the header, or of a fixed segment */
  u64 end;
  u32 prefix, size;
  int segment;     /* fixed-tile segment: starts after its header */
  int final;
} ChainEntry;

static u32 chain_walk(const u8* data, u32 bytes, const u8* bitmap, u32 expected,
                      u32 max_blocks, int tiles, Tables* t, Tables* ft,
                      ChainEntry* chain, u32* chain_len) {
  u64 bits = (u64)bytes * 8;
  u64 next = 0;
  u32 output = 0, n = 0, real_blocks = 0;
  *chain_len = 0;
  for (;;) {
    if (n >= max_blocks) return ST_BLOCK_LIMIT;
    Reader h = {data, bits, next, 0};
    u32 final = rd_take(&h, 1), type = rd_take(&h, 2);
    if (h.error) return h.error;
    if (type == 3) return ST_RESERVED_TYPE;
    if (type == 1 && tiles) {
      u64 cursor = h.pos, tile_bits = (u64)TILE_BYTES * 8;
      for (;;) {
        if (cursor >= bits) return ST_TRUNCATED;
        u64 tile = cursor / tile_bits, offset = cursor % tile_bits;
        u64 tile_end = (tile + 1) * tile_bits;
        if (tile_end > bits) tile_end = bits;
        /* Entries 0..31 come from the per-tile table; others scan from the
         * cursor.  Both scan the same bits, so one scan serves both. */
        (void)offset;
        Summary s = scan_fixed(data, bytes, cursor, tile_end, ft);
        u32 kind = s.flags & 3u, ended = s.flags >> 4;
        if (final && s.first_end != ~(u64)0) {
          s.end = s.first_end;
          s.size = s.first_size;
          s.status = 0;
          kind = 2;
          ended = 1;
        }
        if (s.status) return s.status;
        if (s.end <= cursor || s.end > bits) return ST_EXTENT_MISMATCH;
        if (s.size > expected - output) return ST_OUTPUT_OVERFLOW;
        if (n >= max_blocks || ended > max_blocks - real_blocks) return ST_BLOCK_LIMIT;
        chain[n].start = cursor;
        chain[n].end = s.end;
        chain[n].prefix = output;
        chain[n].size = s.size;
        chain[n].segment = 1;
        chain[n].final = final ? 1 : 0;
        output += s.size;
        real_blocks += ended;
        ++n;
        *chain_len = n;
        cursor = s.end;
        if (kind == 2) {
          if (output != expected) return ST_SIZE_MISMATCH;
          if ((cursor + 7) / 8 != bytes) return ST_EXTENT_MISMATCH;
          return 0;
        }
        if (kind == 1) { next = cursor; break; }
        u32 carried = (s.flags >> 2) & 3u;
        if (carried < 2) final = carried;
      }
      continue;
    }
    Block info;
    int candidate = (bitmap[next >> 3] >> (next & 7)) & 1;
    if (candidate) {
      info = parse_block(data, bytes, next, expected, 65536, t);
    } else {
      if (type == 1) return ST_FIXED_TILES;
      if (type == 2) return ST_UNDISCOVERED;
      info = parse_block(data, bytes, next, expected - output, 0, t);
    }
    if (info.status) return info.status;
    if (info.end <= next || info.end > bits) return ST_EXTENT_MISMATCH;
    if (info.size > expected - output) return ST_OUTPUT_OVERFLOW;
    if (real_blocks >= max_blocks) return ST_BLOCK_LIMIT;
    chain[n].start = next;
    chain[n].end = info.end;
    chain[n].prefix = output;
    chain[n].size = info.size;
    chain[n].segment = 0;
    chain[n].final = info.final ? 1 : 0;
    output += info.size;
    ++real_blocks;
    ++n;
    *chain_len = n;
    next = info.end;
    if (info.final) {
      if (output != expected) return ST_SIZE_MISMATCH;
      if ((next + 7) / 8 != bytes) return ST_EXTENT_MISMATCH;
      return 0;
    }
  }
}

/* Emission with history (emit_blocks / emit_fixed_segment / emit_stored,
 * _decode_kernels.py:474-680,1449-1687): decodes every accepted chain
 * entry at its absolute output prefix; a distance beyond the declared
 * window or before the stream start is status 6 (EmissionStatus takes
 * the maximum over blocks, codec_ffi.cu:405-435, and 6 is the only
 * status emission can add after an accepted chain). */
static u32 emit_chain(const u8* data, u32 bytes, const ChainEntry* chain, u32 count,
                      u32 window, u8* out, Tables* t, Tables* ft) {
  u32 status = 0;
  u64 bits = (u64)bytes * 8;
  for (u32 k = 0; k < count; ++k) {
    const ChainEntry* c = &chain[k];
    Reader r = {data, bits, c->start, 0};
    u32 produced = 0;
    const Tables* tab;
    u32 type = 1;
    if (!c->segment) {
      rd_take(&r, 1);
      type = rd_take(&r, 2);
    }
    if (type == 0) {
      r.pos = (r.pos + 7) & ~(u64)7;
      u32 n = rd_take(&r, 16);
      rd_take(&r, 16);
      memcpy(out + c->prefix, data + (r.pos >> 3), n);
      continue;
    }
    if (type == 2) {
      dynamic_tables(&r, t);
      tab = t;
    } else {
      tab = ft;
    }
    while (r.pos < c->end || !c->segment) {
      u32 size, dist;
      int sym = code_decode(&tab->ll, &r);
      sym = token_rest(&r, tab, sym, &size, &dist, 32768, 0);
      if (r.error) break;
      if (sym == 256) {
        if (!c->segment || r.pos == c->end) break;
        rd_take(&r, 3);  /* next fixed header inside a tile segment */
        continue;
      }
      u64 at = (u64)c->prefix + produced;
      if (!dist) {
        out[at] = (u8)sym;
      } else {
        if (dist > window || dist > at) { status = ST_BAD_DISTANCE; break; }
        for (u32 j = 0; j < size; ++j) out[at + j] = out[at + j - dist];
      }
      produced += size;
    }
  }
  return status;
}

u32 oracle_inflate_general(const u8* in, u64 in_size, u8* out, u64 out_size,
                           u32 max_candidates, u32 max_blocks) {
  if (out_size > MAX_STREAM_BYTES) return ST_BOUNDS;
  memset(out, 0, out_size);
  if (in_size > MAX_STREAM_INPUT || max_candidates < 1 || max_candidates > MAX_CANDIDATES ||
      max_blocks < 1 || max_blocks > MAX_BLOCKS)
    return ST_BOUNDS;
  u32 window = 0, wanted = 0;
  u32 err = zlib_framing(in, in_size, &window, &wanted);
  if (err) return err;
  const u8* data = in + 2;
  u32 bytes = (u32)(in_size - 6);
  u32 expected = (u32)out_size;
  Tables* t = (Tables*)malloc(sizeof(Tables));
  Tables* ft = (Tables*)malloc(sizeof(Tables));
  fixed_tables(ft);
  u8* bitmap = (u8*)calloc((size_t)bytes + 1, 1);
  ChainEntry* chain = NULL;
  u64 count = discover(data, bytes, bitmap, t);
  u64 capacity = (u64)bytes * 9 + 1;
  if (capacity > max_candidates) capacity = max_candidates;
  if (count > capacity) { err = ST_CANDIDATE_OVERFLOW; goto done; }
  if (!count) { err = ST_NO_INITIAL_BLOCK; goto done; }
  /* A chain entry consumes at least three bits, and tile segments at least
   * one bit of a 2 KiB tile; max_blocks bounds both. */
  chain = (ChainEntry*)malloc(sizeof(ChainEntry) * ((size_t)max_blocks + 1));
  u32 chain_len = 0;
  err = chain_walk(data, bytes, bitmap, expected, max_blocks, 0, t, ft, chain, &chain_len);
  if (err == ST_FIXED_TILES)
    err = chain_walk(data, bytes, bitmap, expected, max_blocks, 1, t, ft, chain, &chain_len);
  if (err) goto done;
  err = emit_chain(data, bytes, chain, chain_len, window, out, t, ft);
  if (err) goto done;
  if (oracle_adler32(out, out_size) != wanted) err = ST_ADLER;
done:
  if (err) memset(out, 0, out_size);
  free(chain);
  free(bitmap);
  free(t);
  free(ft);
  return err;
}

/* Route selection of Decompress (codec_ffi.cu:662-700): the small route
 * (output <= 64 KiB, input <= 128 KiB, default limits) decodes serially;
 * every other stream reports general-route statuses.  The stored and medium
 * fast routes only ever publish success, which the general route shares. */
u32 oracle_decompress(const u8* in, u64 in_size, u8* out, u64 out_size,
                      u32 max_candidates, u32 max_blocks) {
  if (out_size > MAX_STREAM_BYTES) return ST_BOUNDS;
  if (in_size > MAX_STREAM_INPUT || max_candidates < 1 || max_candidates > MAX_CANDIDATES ||
      max_blocks < 1 || max_blocks > MAX_BLOCKS) {
    memset(out, 0, out_size);
    return ST_BOUNDS;
  }
  if (in_size < 8) { memset(out, 0, out_size); return ST_TRUNCATED_ZLIB; }
  if (out_size <= 65536 && in_size <= 131072 && max_candidates == MAX_CANDIDATES &&
      max_blocks == MAX_BLOCKS) {
    u32 s = oracle_inflate_serial(in, in_size, out, out_size, max_blocks);
    if (s) memset(out, 0, out_size);
    return s;
  }
  return oracle_inflate_general(in, in_size, out, out_size, max_candidates, max_blocks);
}

/* ------------------------------------------------------------------ */
/* Encoder (follows encode_chunk, _encode_kernels.py:283-400, and the   */
/* finish steps, batch_encode.cuh:39-112 / codec_ffi.cu:551-612).       */
/* ------------------------------------------------------------------ */
static const u32 kLenBase[29] = {3, 4, 5, 6, 7, 8, 9, 10, 11, 13, 15, 17, 19, 23, 27, 31,
                                 35, 43, 51, 59, 67, 83, 99, 115, 131, 163, 195, 227, 258};
static const u32 kLenExtra[29] = {0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2,
                                  2, 3, 3, 3, 3, 4, 4, 4, 4, 5, 5, 5, 5, 0};
static const u32 kDistBase[30] = {1, 2, 3, 4, 5, 7, 9, 13, 17, 25, 33, 49, 65, 97, 129,
                                  193, 257, 385, 513, 769, 1025, 1537, 2049, 3073, 4097,
                                  6145, 8193, 12289, 16385, 24577};
static const u32 kDistExtra[30] = {0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6,
                                   6, 7, 7, 8, 8, 9, 9, 10, 10, 11, 11, 12, 12, 13, 13};

typedef struct {
  u8* data;
  u32 size, capacity, cache, bits, error;
} Writer;

static void w_byte(Writer* w, u32 v) {
  if (w->size >= w->capacity) { w->error = 1; return; }
  w->data[w->size++] = (u8)v;
}
static void w_put(Writer* w, u32 v, u32 n) {
  w->cache |= v << w->bits;
  w->bits += n;
  while (w->bits >= 8) { w_byte(w, w->cache & 255u); w->cache >>= 8; w->bits -= 8; }
}
static void w_align(Writer* w) {
  if (w->bits) { w_byte(w, w->cache & 255u); w->cache = 0; w->bits = 0; }
}
static u32 reverse_bits(u32 x, u32 n) {
  u32 r = 0;
  for (u32 i = 0; i < n; ++i) { r = (r << 1) | (x & 1u); x >>= 1; }
  return r;
}
static void fixed_put(Writer* w, u32 sym) {
  u32 code, bits;
  if (sym <= 143) { code = 0x30u + sym; bits = 8; }
  else if (sym <= 255) { code = 0x190u + sym - 144u; bits = 9; }
  else if (sym <= 279) { code = sym - 256u; bits = 7; }
  else { code = 0xc0u + sym - 280u; bits = 8; }
  w_put(w, reverse_bits(code, bits), bits);
}

/* enc_hash (_encode_kernels.py:47-51): 13-bit multiplicative hash. */
static u32 hash3(const u8* d, u32 p) {
  u32 v = (u32)d[p] | ((u32)d[p + 1] << 8) | ((u32)d[p + 2] << 16);
  return (v * 2654435761u) >> 19;
}

/* Heap-based Huffman tree with (weight, node) ordering and positive
 * frequency flattening retries (enc_tree, _encode_kernels.py:65-157). */
typedef struct {
  u32 weight[571];
  u16 parent[571];
  u16 heap[286];
} TreeScratch;

static int tless(u32 a, u32 b, const u32* w) { return w[a] < w[b] || (w[a] == w[b] && a < b); }
static void heap_push(u32 node, u16* heap, u32* count, const u32* w) {
  u32 i = (*count)++;
  while (i) {
    u32 p = (i - 1) >> 1;
    if (!tless(node, heap[p], w)) break;
    heap[i] = heap[p];
    i = p;
  }
  heap[i] = (u16)node;
}
static void heap_sift(u32 node, u16* heap, u32 count, const u32* w) {
  u32 i = 0;
  while (2 * i + 1 < count) {
    u32 c = 2 * i + 1;
    if (c + 1 < count && tless(heap[c + 1], heap[c], w)) ++c;
    if (!tless(heap[c], node, w)) break;
    heap[i] = heap[c];
    i = c;
  }
  heap[i] = (u16)node;
}

static int build_tree(const u32* freq, u32 alphabet, u32 limit, u8* lengths, u16* codes,
                      TreeScratch* s) {
  for (u32 shift = 0; shift <= 16; ++shift) {
    u32 hs = 0;
    u32* w = s->weight;
    for (u32 i = 0; i < alphabet; ++i) {
      lengths[i] = 0;
      codes[i] = 0;
      w[i] = freq[i] ? ((freq[i] + (1u << shift) - 1u) >> shift) : 0;
      if (w[i]) heap_push(i, s->heap, &hs, w);
    }
    if (!hs) { w[0] = 1; heap_push(0, s->heap, &hs, w); }
    if (hs == 1) {
      u32 dummy = s->heap[0] ? 0u : 1u;
      w[dummy] = 1;
      heap_push(dummy, s->heap, &hs, w);
    }
    u32 next = alphabet;
    while (hs > 1) {
      u32 a = s->heap[0];
      u32 last = s->heap[--hs];
      if (hs) heap_sift(last, s->heap, hs, w);
      u32 b = s->heap[0];
      w[next] = w[a] + w[b];
      s->parent[a] = (u16)next;
      s->parent[b] = (u16)next;
      heap_sift(next++, s->heap, hs, w);
    }
    s->parent[next - 1] = 65535u;
    u32 count[16] = {0}, first[16] = {0};
    int overlong = 0;
    for (u32 i = 0; i < alphabet; ++i) {
      if (!w[i]) continue;
      u32 node = i, depth = 0;
      while (s->parent[node] != 65535u) {
        node = s->parent[node];
        if (++depth > limit) { overlong = 1; break; }
      }
      if (depth <= limit) { lengths[i] = (u8)depth; ++count[depth]; }
    }
    if (overlong) continue;
    u32 code = 0;
    for (u32 b = 1; b <= limit; ++b) { code = (code + count[b - 1]) << 1; first[b] = code; }
    for (u32 i = 0; i < alphabet; ++i)
      if (lengths[i]) codes[i] = (u16)reverse_bits(first[lengths[i]]++, lengths[i]);
    return 1;
  }
  return 0;
}

static u32 extent_of(u32 bits, int final) { return final ? (bits + 7) / 8 : (bits + 3 + 7) / 8 + 4; }

/* Stored blocks of an n-byte chunk's stored fallback: one for chunks within
 * the reference's bound (n <= 65535), else ceil(n / 65535). */
static u32 stored_blocks(u32 n) { return n ? (n + STORED_MAX - 1) / STORED_MAX : 1u; }

/* Worst-case stream layout of n bytes at `chunk` (both a multiple of nothing
 * in particular): stored blocks of every chunk's fallback, which size the
 * padded capacity n + 5 * stored + 6 (compress_zlib_padded, _codec.py:
 * 151-177, where every chunk has one), and the most Deflate blocks the
 * stream can hold (2 * chunks - 1 for chunks <= 65535). */
static void stream_layout(u64 n, u32 chunk, u64* chunks_out, u64* stored_out, u64* blocks_out) {
  u64 chunks = n ? (n + chunk - 1) / chunk : 1;
  u32 last = (u32)(n - (chunks - 1) * chunk);
  u64 full = stored_blocks(chunk), tail = stored_blocks(last);
  *chunks_out = chunks;
  *stored_out = (chunks - 1) * full + tail;
  *blocks_out = (chunks - 1) * (full > 2 ? full : 2) + tail;
}

/* Opt-in level 2 (no reference counterpart; the GPU encoder's restated
 * parse).  Every position below n - 2 has its hash chain: prev[p] = 1 + the
 * last earlier position with its hash, or 0.  A position's best match is the
 * longest of its first L2_CHAIN chain candidates within 32768 bytes (the
 * nearest among equal lengths; the search stops at L2_NICE bytes or the end
 * of the chunk), a length-3 match farther than L2_TOO_FAR bytes counts as
 * none, and the token at p is a literal when p's best match is shorter than
 * L2_LAZY and p + 1 has a longer one (one-step lazy evaluation).  The token
 * at p is a function of the data alone, which the GPU's speculative walks
 * need. */
#ifndef L2_CHAIN
#define L2_CHAIN 32u
#endif
#ifndef L2_LAZY
#define L2_LAZY 32u
#endif
#ifndef L2_NICE
#define L2_NICE 258u
#endif
#define L2_TOO_FAR 4096u

static u32 l2_best(const u8* d, u32 n, const u32* prev, u32 p, u32* where) {
  if (n < 3 || p >= n - 2) return 0;
  const u32 limit = n - p < 258 ? n - p : 258;
  u32 best = 0, at = 0, c = prev[p];
  for (u32 step = 0; c && step < L2_CHAIN; ++step) {
    const u32 q = c - 1;
    if (p - q > 32768u) break;
    if (d[q] == d[p] && d[q + 1] == d[p + 1] && d[q + 2] == d[p + 2]) {
      u32 m = 3;
      while (m < limit && d[q + m] == d[p + m]) ++m;
      if (m > best) {
        best = m;
        at = q;
        if (m >= limit || m >= L2_NICE) break;
      }
    }
    c = prev[q];
  }
  if (best == 3 && p - at > L2_TOO_FAR) best = 0;
  *where = at;
  return best;
}

static u32 l2_token(const u8* d, u32 n, const u32* prev, u32 p, u32* where) {
  const u32 m = l2_best(d, n, prev, p, where);
  if (!m || m >= L2_LAZY) return m;
  u32 next = 0;
  return l2_best(d, n, prev, p + 1, &next) > m ? 0u : m;
}

/* Encodes one chunk into `slot`; returns the status (0 ok).  `size` gets
 * the encoded byte count.  level 1 is the reference's parse, level 2 the
 * parse above. */
static u32 encode_chunk(const u8* data, u32 n, int final, u8* slot, u32 slot_bytes, u32* size,
                        u32 level) {
  u32* last = (u32*)calloc(8192, sizeof(u32));
  u32* tokens = (u32*)malloc(sizeof(u32) * (n ? n : 1));
  u32 freq[335];
  u8 lengths[335];
  u16 codes[335];
  u8 rle_sym[316], rle_extra[316];
  TreeScratch ts;
  memset(freq, 0, sizeof(freq));
  memset(lengths, 0, sizeof(lengths));
  memset(codes, 0, sizeof(codes));
  u32 extra_bits = 0, count = 0, pos = 0;
  if (level == 2) {
    u32* prev = (u32*)calloc(n ? n : 1, sizeof(u32));
    for (u32 p = 0; n >= 3 && p < n - 2; ++p) {
      const u32 h = hash3(data, p);
      prev[p] = last[h];
      last[h] = p + 1;
    }
    while (pos < n) {
      u32 earlier = 0;
      const u32 match = l2_token(data, n, prev, pos, &earlier);
      if (!match) {
        freq[data[pos]]++;
        tokens[count++] = data[pos++];
        continue;
      }
      u32 dist = pos - earlier, li = 0, di = 0;
      while (li < 28 && match >= kLenBase[li + 1]) ++li;
      while (di < 29 && dist >= kDistBase[di + 1]) ++di;
      freq[257 + li]++;
      freq[286 + di]++;
      extra_bits += kLenExtra[li] + kDistExtra[di];
      tokens[count++] = 0x80000000u | li | (di << 5) | ((match - kLenBase[li]) << 10) |
                        ((dist - kDistBase[di]) << 15);
      pos += match;
    }
    free(prev);
  }
  /* Greedy one-candidate parse.  Every position is inserted in order, so the
   * candidate of a position is the last earlier position with its hash. */
  for (; level != 2;) {
    u32 earlier = 0;
    int candidate = 0;
    while (pos < n) {
      candidate = 0;
      if (n - pos >= 3) {
        u32 h = hash3(data, pos), prev = last[h];
        last[h] = pos + 1;
        if (prev) {
          earlier = prev - 1;
          u32 dist = pos - earlier;
          candidate = dist && dist <= 32768u && data[earlier] == data[pos] &&
                      data[earlier + 1] == data[pos + 1] && data[earlier + 2] == data[pos + 2];
        }
      }
      if (candidate) break;
      freq[data[pos]]++;
      tokens[count++] = data[pos++];
    }
    if (pos == n) break;
    u32 limit = n - pos < 258 ? n - pos : 258;
    u32 match = limit;
    for (u32 o = 3; o < limit; ++o)
      if (data[earlier + o] != data[pos + o]) { match = o; break; }
    for (u32 j = 1; j < match && n - (pos + j) >= 3; ++j) last[hash3(data, pos + j)] = pos + j + 1;
    u32 dist = pos - earlier, li = 0, di = 0;
    while (li < 28 && match >= kLenBase[li + 1]) ++li;
    while (di < 29 && dist >= kDistBase[di + 1]) ++di;
    freq[257 + li]++;
    freq[286 + di]++;
    extra_bits += kLenExtra[li] + kDistExtra[di];
    tokens[count++] = 0x80000000u | li | (di << 5) | ((match - kLenBase[li]) << 10) |
                      ((dist - kDistBase[di]) << 15);
    pos += match;
  }
  freq[256]++;

  /* Exact stored / fixed / dynamic extents (encode_chunk, :312-356); the
   * stored fallback of a chunk above 65535 bytes takes several blocks. */
  const u32 nstored = stored_blocks(n);
  u32 mode = 0, extent = n + 5 * nstored, status = 0;
  u32 fixed_bits = 3 + extra_bits, dist_tokens = 0;
  for (u32 i = 0; i < 286; ++i)
    fixed_bits += freq[i] * (i <= 143 ? 8u : i <= 255 ? 9u : i <= 279 ? 7u : 8u);
  for (u32 i = 0; i < 30; ++i) { dist_tokens += freq[286 + i]; fixed_bits += freq[286 + i] * 5; }
  u32 fixed_extent = extent_of(fixed_bits, final);
  if (fixed_extent < extent) { extent = fixed_extent; mode = 1; }
  int trees = 1;
  u32 ll_bits = 0, nll = 286, ndist = 30, ncl = 19, rle_size = 0;
  int dyn = extent_of(29 + extra_bits + count + 1 + dist_tokens, final) < extent;
  if (dyn) {
    trees = build_tree(freq, 286, 15, lengths, codes, &ts);
    for (u32 i = 0; i < 286; ++i) ll_bits += freq[i] * lengths[i];
    dyn = extent_of(29 + extra_bits + ll_bits + dist_tokens, final) < extent;
  }
  if (trees && dyn) {
    trees = build_tree(freq + 286, 30, 15, lengths + 286, codes + 286, &ts);
    while (nll > 257 && !lengths[nll - 1]) --nll;
    while (ndist > 1 && !lengths[286 + ndist - 1]) --ndist;
    /* Run-length code the concatenated code lengths (enc_rle, :163-191). */
    u32 total = nll + ndist, i = 0;
    while (i < total) {
      u32 value = i < nll ? lengths[i] : lengths[286 + i - nll], run = 1;
      while (i + run < total && (i + run < nll ? lengths[i + run] : lengths[286 + i + run - nll]) == value)
        ++run;
      i += run;
      if (value) {
        rle_sym[rle_size] = (u8)value; rle_extra[rle_size++] = 0; freq[316 + value]++; --run;
        while (run >= 3) {
          u32 take = run < 6 ? run : 6;
          rle_sym[rle_size] = 16; rle_extra[rle_size++] = (u8)(take - 3); freq[316 + 16]++; run -= take;
        }
      } else {
        while (run >= 11) {
          u32 take = run < 138 ? run : 138;
          rle_sym[rle_size] = 18; rle_extra[rle_size++] = (u8)(take - 11); freq[316 + 18]++; run -= take;
        }
        if (run >= 3) {
          rle_sym[rle_size] = 17; rle_extra[rle_size++] = (u8)(run - 3); freq[316 + 17]++; run = 0;
        }
      }
      while (run) { rle_sym[rle_size] = (u8)value; rle_extra[rle_size++] = 0; freq[316 + value]++; --run; }
    }
    trees = trees && build_tree(freq + 316, 19, 7, lengths + 316, codes + 316, &ts);
    while (ncl > 4 && !lengths[316 + kClOrder[ncl - 1]]) --ncl;
  }
  if (!trees) {
    mode = 3;
    status = 1;
  } else if (dyn) {
    u32 dbits = 17 + 3 * ncl + extra_bits + ll_bits;
    for (u32 i = 0; i < 30; ++i) dbits += freq[286 + i] * lengths[286 + i];
    for (u32 i = 0; i < 19; ++i)
      dbits += freq[316 + i] * (lengths[316 + i] + (i == 16 ? 2u : i == 17 ? 3u : i == 18 ? 7u : 0u));
    u32 dext = extent_of(dbits, final);
    if (dext < extent) { extent = dext; mode = 2; }
  }
  *size = 0;
  if (mode == 3) goto out;
  if (mode == 0) {
    /* Blocks of 65535 bytes, the last one shorter; only the stream's very
     * last block carries BFINAL. */
    u32 at = 0;
    for (u32 k = 0; k < nstored; ++k) {
      u32 len = n - k * STORED_MAX < STORED_MAX ? n - k * STORED_MAX : STORED_MAX;
      slot[at] = (final && k + 1 == nstored) ? 1 : 0;
      slot[at + 1] = (u8)len; slot[at + 2] = (u8)(len >> 8);
      u32 c = len ^ 65535u;
      slot[at + 3] = (u8)c; slot[at + 4] = (u8)(c >> 8);
      memcpy(slot + at + 5, data + k * STORED_MAX, len);
      at += 5 + len;
    }
    *size = extent;
    goto out;
  }
  {
    Writer w = {slot, 0, slot_bytes, 0, 0, 0};
    int dynamic = mode == 2;
    w_put(&w, (final ? 1u : 0u) | (dynamic ? 4u : 2u), 3);
    if (dynamic) {
      w_put(&w, nll - 257, 5);
      w_put(&w, ndist - 1, 5);
      w_put(&w, ncl - 4, 4);
      for (u32 i = 0; i < ncl; ++i) w_put(&w, lengths[316 + kClOrder[i]], 3);
      for (u32 i = 0; i < rle_size; ++i) {
        u32 s = rle_sym[i];
        w_put(&w, codes[316 + s], lengths[316 + s]);
        if (s >= 16) w_put(&w, rle_extra[i], s == 16 ? 2 : s == 17 ? 3 : 7);
      }
    }
    for (u32 i = 0; i < count; ++i) {
      u32 tk = tokens[i];
      if (tk & 0x80000000u) {
        u32 li = tk & 31u, di = (tk >> 5) & 31u;
        if (dynamic) w_put(&w, codes[257 + li], lengths[257 + li]);
        else fixed_put(&w, 257 + li);
        w_put(&w, (tk >> 10) & 31u, kLenExtra[li]);
        if (dynamic) w_put(&w, codes[286 + di], lengths[286 + di]);
        else w_put(&w, reverse_bits(di, 5), 5);
        w_put(&w, (tk >> 15) & 8191u, kDistExtra[di]);
      } else {
        if (dynamic) w_put(&w, codes[tk], lengths[tk]);
        else fixed_put(&w, tk);
      }
    }
    if (dynamic) w_put(&w, codes[256], lengths[256]);
    else fixed_put(&w, 256);
    if (!final) {
      w_put(&w, 0, 3);  /* empty stored block re-aligns the next chunk */
      w_align(&w);
      w_byte(&w, 0); w_byte(&w, 0); w_byte(&w, 255); w_byte(&w, 255);
    } else {
      w_align(&w);
    }
    if (w.error || w.size != extent) status = 1;
    else *size = w.size;
  }
out:
  free(last);
  free(tokens);
  return status;
}

/* Whole-stream compression: metadata = [encoded_length, status].  The
 * capacity must be n + 5 * stored_blocks + 6, i.e. n + 5*chunks + 6 for
 * chunks <= 65535 (compress_zlib_padded, _codec.py:151-177). */
u32 oracle_compress_level(const u8* in, u64 n, u32 chunk_bytes, u32 level, u8* out,
                          u64 capacity, u32* meta) {
  meta[0] = 0;
  meta[1] = 0;
  memset(out, 0, capacity);
  if (n > MAX_STREAM_BYTES || chunk_bytes < 256 || chunk_bytes > MAX_CHUNK_BYTES) {
    meta[1] = ST_BOUNDS;
    return ST_BOUNDS;
  }
  u64 chunks, stored, blocks;
  stream_layout(n, chunk_bytes, &chunks, &stored, &blocks);
  if (blocks > MAX_BLOCKS || capacity != n + stored * 5 + 6) {
    meta[1] = ST_BOUNDS;
    return ST_BOUNDS;
  }
  u32 slot_bytes = (chunk_bytes * 9 + 7) / 8 + 16 + 5 * stored_blocks(chunk_bytes);
  u8* slot = (u8*)malloc(slot_bytes);
  u64 total = 2;
  out[0] = 0x78;
  out[1] = 0x01;
  for (u64 c = 0; c < chunks; ++c) {
    u64 start = c * chunk_bytes;
    u32 len = (u32)(n - start < chunk_bytes ? n - start : chunk_bytes);
    u32 size = 0;
    u32 st = encode_chunk(in + start, len, c + 1 == chunks, slot, slot_bytes, &size, level);
    if (st || size > slot_bytes || total + size + 4 > capacity) {
      free(slot);
      memset(out, 0, capacity);
      meta[1] = ST_COMPRESSION_OVERFLOW;
      return ST_COMPRESSION_OVERFLOW;
    }
    memcpy(out + total, slot, size);
    total += size;
  }
  free(slot);
  u32 a = oracle_adler32(in, n);
  out[total] = (u8)(a >> 24);
  out[total + 1] = (u8)(a >> 16);
  out[total + 2] = (u8)(a >> 8);
  out[total + 3] = (u8)a;
  total += 4;
  meta[0] = (u32)total;
  return 0;
}

u32 oracle_compress(const u8* in, u64 n, u32 chunk_bytes, u8* out, u64 capacity, u32* meta) {
  return oracle_compress_level(in, n, chunk_bytes, 1, out, capacity, meta);
}

/* Compress a chunk range [first, first+count) of one stream into the
 * caller's slots (used for a multi-threaded CPU baseline; each chunk is
 * independent).  Returns the number of failed chunks. */
u32 oracle_compress_chunks_level(const u8* in, u64 n, u32 chunk_bytes, u32 level, u64 first,
                                 u64 count, u8* slots, u32 slot_bytes, u32* sizes) {
  u64 chunks = (n + chunk_bytes - 1) / chunk_bytes;
  if (!chunks) chunks = 1;
  u32 failed = 0;
  for (u64 c = first; c < first + count && c < chunks; ++c) {
    u64 start = c * chunk_bytes;
    u32 len = (u32)(n - start < chunk_bytes ? n - start : chunk_bytes);
    failed += encode_chunk(in + start, len, c + 1 == chunks, slots + (c - first) * slot_bytes,
                           slot_bytes, &sizes[c - first], level) != 0;
  }
  return failed;
}

u32 oracle_compress_chunks(const u8* in, u64 n, u32 chunk_bytes, u64 first, u64 count,
                           u8* slots, u32 slot_bytes, u32* sizes) {
  return oracle_compress_chunks_level(in, n, chunk_bytes, 1, first, count, slots, slot_bytes,
                                      sizes);
}
