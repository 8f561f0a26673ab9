// Block-parallel inflate of one large zlib stream.
//
// A Deflate stream is serial inside a block but its blocks can be decoded
// independently once their start bits and output offsets are known, except
// for back-references that reach into earlier blocks.  The pipeline:
//
//   candidates  the reference's candidate rule (bit 0, every bit offset that
//               parses as a valid dynamic header, stored-block endpoint
//               seeds; discover_kernel) compacted into a sorted list;
//   describe    one warp per candidate decodes without output from the
//               candidate through any following stored/fixed blocks up to
//               the next dynamic header ("node"): end bit, output size,
//               block count, final flag.  Every valid dynamic header is a
//               candidate, so the true chain is a path of nodes;
//   chain       one CTA links each node to the candidate at its end bit and
//               extracts the path from bit 0 by pointer doubling, with
//               output prefixes, extent and block-count checks;
//   emit        one warp per path node decodes into a shared-memory ring of
//               u16 symbols: a byte, or 256 + k for "the byte k+1 positions
//               before this node's start" (a reference into an earlier
//               node; copies propagate the marker).  Flushes write bytes to
//               the output and, for markers, the absolute source position
//               plus a bit in an unresolved-position bitmap;
//   resolve     each unresolved position follows source positions until it
//               reaches a byte decoded directly (positions strictly
//               decrease, so every chase ends);
//   adler       a segmented reduction over the output, then the checksum
//               and status.
//
// This is the marker method of published parallel gzip decoders (pugz,
// rapidgzip) applied with the chain known exactly, so no speculation is
// ever wrong: the output is exact or the stream is reported failed.  Any
// failure hands over to general_status_kernel, which reports the status
// the reference's route reports.
#include "kernels.h"
#include "inflate_core.cuh"

namespace cz {

constexpr u32 kNodeWarps = 4;      // warps per CTA in describe
constexpr u32 kExpandWarps = 4;    // warps per CTA in expand
constexpr u32 kLaneTokens = 4;     // consecutive tokens per lane in an expand chunk
constexpr u32 kChunkTokens = 32 * kLaneTokens;
// Ring entry of a copy byte not yet known: kPending | r, the symbol r
// positions back (r < 8192; bytes are below 256, markers below 33024).
constexpr u32 kPending = 0xe000u;
// Token flag, in the chunk's shared copy only: the copy reads nothing the
// chunk writes.
constexpr u32 kOwnFlag = 0x20000000u;
constexpr u32 kEmitRing = 4096;    // u16 history entries per emitting warp
constexpr u32 kEmitMask = kEmitRing - 1;
constexpr u32 kEmitFlush = 2048;   // pending symbols that trigger a flush
// Node facts (infos[]): the node decoded cleanly (ok), ended the stream
// (final), ran out of arena pages (spilled), ended on a fixed-region seed
// (fixed stop; the next node is that seed's), and whether the block in
// progress at its end is the final one (exit final).
constexpr u32 kInfoFinal = 1u, kInfoOk = 2u, kInfoSpilled = 4u, kInfoFixedStop = 8u,
              kInfoExitFinal = 16u;
constexpr u32 kPageWords = 1024;   // token words per arena page
constexpr u32 kNoPage = 0xffffffffu;
constexpr u32 kPassPages = 40;     // pages one pass can reach (32 Ki tokens)
constexpr u32 kSeedTileBits = 1u << 18;  // body bits per fixed-region seed probe (32 KiB)
constexpr u32 kSeedProbeBits = 1024;     // bits a probe decodes before its seed

// ---------------------------------------------------------------------------
// Lane-parallel rounds over a Huffman block body.
// ---------------------------------------------------------------------------
// A round gives lane j the window [start + jW, start + (j+1)W) of the body.
// Lane 0 starts on the true token chain; the others start at an arbitrary
// bit and decode speculatively (phase 1), marking where their tokens start.
// Huffman decoding resynchronizes: a lane that runs on past its window
// (phase 2) soon lands on a position some later lane marked, and from there
// that lane's chain is its own.  Lane 0 links the lanes in order from the
// true start, which gives each lane a region between two boundaries known to
// be on the true chain; phase 3 writes every region's tokens, copied from
// the tokens the lane kept while decoding (or decoded again when it kept too
// many to hold).  A
// code the exact decoder must judge (or too few bits left) ends the round at
// that token, and the serial decoder carries on from there, so statuses
// stay the serial decoder's.  On config-1 streams half the lanes resynchronize
// within 64 bits and the share left halves every further 64 bits, so a
// whole window of marks almost never runs out.
constexpr u32 kRoundWindow = 1024;  // body bits per lane per round
constexpr u32 kMarkWords = kRoundWindow / 32;
// Tokens a lane keeps from phases 1 and 2 of a round (a config-1 window
// holds about 150).  Phase 3 copies a region's tokens from there instead of
// decoding them again, unless the lane decoded more than this.
constexpr u32 kStash = 256;

enum LaneEnd : u32 {
  kLaneWindow = 0,     // reached the window end / a boundary past the round
  kLaneBlockEnd = 1,   // end-of-block code at the recorded position
  kLaneIrregular = 2,  // a token for the serial decoder at the recorded position
  kLaneMerged = 3,     // landed on a later lane's mark
  kLaneFixedStop = 4,  // reached the round's fixed-region seed (a token starts there)
};
enum RoundOutcome : u32 {
  kRoundMore = 0, kRoundBlockEnd = 1, kRoundFallback = 2, kRoundFixedStop = 3
};

// Mark rows are padded by a word: lanes work through their windows in near
// lockstep, and rows 32 words apart would put them all in one bank.
struct RoundShared {
  u32 marks[32][kMarkWords + 1];
  u32 stop[32];      // phase 1: kLaneWindow or where and why it stopped early
  u32 stop_at[32];
  u32 link[32];      // phase 2: kLaneMerged / kLaneWindow (past the round) / stop
  u32 link_at[32];   // position reached
  u32 link_to[32];   // lane merged with
  u32 region_from[32], region_to[32], region_end[32];  // set by the walk
  // Where the pass's tokens go (set by lane 0 before phase 3): pages[k] holds
  // tokens fill0 + [1024k, 1024(k+1)) of the pass, or `word` is the first
  // contiguous word; `drop` when there is no room.
  u32 pages[kPassPages];
  u32 fill0, word, drop;
};

// Where a node's tokens go: nowhere (count only), one contiguous run (the
// layout by path token prefixes), or a chain of arena pages allocated as the
// node grows (describe, before the path is known).  Lane 0 owns the state.
struct SymbolSink {
  enum Mode : u32 { kNoWrite = 0, kContiguous = 1, kPages = 2 };
  u32 mode;
  u32* pool;       // arena words (page k at pool + k * kPageWords)
  u32 room;        // contiguous: words available at pool
  u32* next;       // pages: next page of a chain (kNoPage ends it)
  u32* used;       // pages: words used per page
  u32* cursor;     // pages: next free page
  u32 npages;
  u32 page, fill;  // current page (kNoPage before the first) and its words
  u32 first;       // the node's first page
  u32 written;     // words appended
  u32 spilled;     // a word could not be stored

  __device__ void new_page() {
    const u32 idx = atomicAdd(cursor, 1u);
    if (idx >= npages) {
      spilled = 1;
      return;
    }
    if (page == kNoPage) first = idx;
    else { used[page] = fill; next[page] = idx; }
    page = idx;
    fill = 0;
  }
  // Lane 0: append one word, or two that stay on one page.
  __device__ void put(u32 word) {
    if (mode == kContiguous) {
      if (written < room) pool[written] = word;
      else spilled = 1;
    } else if (mode == kPages && !spilled) {
      if (page == kNoPage || fill == kPageWords) new_page();
      if (!spilled) pool[u64(page) * kPageWords + fill++] = word;
    }
    ++written;
  }
  __device__ void put_pair(u32 a, u32 b) {
    if (mode == kPages && !spilled && (page == kNoPage || fill + 2 > kPageWords)) new_page();
    put(a);
    put(b);
  }
  // Lane 0: room for a pass's `count` words, described in r for the lanes.
  __device__ void reserve(u32 count, RoundShared& r) {
    r.drop = 0;
    if (mode == kContiguous) {
      r.word = written;
      if (written + count > room) { r.drop = 1; spilled = 1; }
    } else if (mode == kPages) {
      if (!spilled && count && (page == kNoPage || fill == kPageWords)) new_page();
      r.fill0 = fill;
      u32 k = 0, left = count;
      if (!spilled) {
        r.pages[k++] = page;
        u32 space = kPageWords - fill;
        while (left > space && !spilled && k < kPassPages) {
          left -= space;
          fill = kPageWords;
          new_page();
          if (!spilled) r.pages[k++] = page;
          space = kPageWords;
        }
        if (left > space) spilled = 1;
        else fill += left;
      }
      r.drop = spilled;
    }
    written += count;
  }
  // Address of word g of the current pass (after reserve), or nullptr.
  __device__ __forceinline__ u32* slot(const RoundShared& r, u32 g) const {
    if (mode == kContiguous) return pool + r.word + g;
    const u32 a = r.fill0 + g;
    return pool + u64(r.pages[a / kPageWords]) * kPageWords + a % kPageWords;
  }
  __device__ void finish() {
    if (mode == kPages && page != kNoPage) {
      used[page] = fill;
      next[page] = kNoPage;
    }
  }
};

// A node's tokens as the decoder writes them: a literal byte;
// kMatchFlag | distance << 9 | length; or kStoredFlag | length followed by a
// word with the stored bytes' body offset.  Empty stored blocks write none.
constexpr u32 kMatchFlag = 0x80000000u;
constexpr u32 kStoredFlag = 0x40000000u;

struct RoundResult {
  u32 pos, bytes, tokens, outcome;
};

// Token bits of a match.
__device__ __forceinline__ u32 match_symbol(u32 length, u32 dist) {
  return kMatchFlag | (dist << 9) | length;
}

// Bit reader of the passes: Bits with the next word already requested, so a
// refill does not wait for a load it could have issued a word earlier.
struct AheadBits {
  const u32* words;  // 4-byte aligned, at or below the first body byte
  u32 shift, last, end;  // as in Bits
  u32 idx;           // index of `next`, the word appended at the next refill
  u32 nbits, lo, hi, next;

  __device__ __forceinline__ u32 load(u32 i) const { return i <= last ? __ldg(words + i) : 0u; }
  __device__ __forceinline__ void init(const u8* body, u32 bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(body);
    words = reinterpret_cast<const u32*>(a & ~uintptr_t(3));
    shift = u32(a & 3) * 8;
    end = bytes * 8;
    last = bytes ? (shift + end - 1) >> 5 : 0;
  }
  __device__ __forceinline__ u32 pos() const { return idx * 32 - nbits - shift; }
  __device__ __forceinline__ u32 avail() const {
    const u32 p = pos();
    return p <= end ? end - p : 0;
  }
  __device__ __forceinline__ void seek(u32 p) {
    const u32 a = shift + p;
    idx = (a >> 5) + 1;
    lo = load(idx - 1) >> (a & 31);
    hi = 0;
    nbits = 32 - (a & 31);
    next = load(idx);
    refill();
  }
  __device__ __forceinline__ void refill() {
    if (nbits <= 32) {
      lo |= next << nbits;                      // shifts of 32 give 0
      hi |= __funnelshift_lc(next, 0u, nbits);  // high word of next << nbits
      nbits += 32;
      next = load(++idx);
    }
  }
  __device__ __forceinline__ void consume(u32 n) {
    lo = __funnelshift_r(lo, hi, n);
    hi >>= n;
    nbits -= n;
  }
};

// One token.  Returns kLaneWindow (decoded: *bytes output bytes, *sym its
// symbol word), kLaneBlockEnd (end-of-block code, consumed) or
// kLaneIrregular (a code the serial decoder must judge, a distance beyond
// the window, or fewer than 48 body bits left, so every token taken here
// lies wholly inside the body).  kChecked = false skips the 48-bit check
// for callers that know the token starts at least 48 bits before the end.
template <bool kChecked = true, typename Reader>
__device__ __forceinline__ u32 symbol_token(Reader& c, const Tables& t, u32 window, u32* bytes,
                                            u32* sym) {
  if (kChecked && c.avail() < 48) return kLaneIrregular;
  c.refill();
  u32 v = c.lo;
  u32 e = t.ll.lut[v & kLLMask];
  u32 kind = entry_kind(e);
  if (kind == kLong) {
    e = decode_long(t.ll, v, LLFn());
    kind = entry_kind(e);
  }
  if (kind == kLiteral) {
    c.consume(entry_len(e));
    *bytes = 1;
    *sym = entry_value(e);
    return kLaneWindow;
  }
  if (kind == kEnd) {
    c.consume(entry_len(e));
    return kLaneBlockEnd;
  }
  if (kind != kLength) return kLaneIrregular;
  const u32 L = entry_len(e), E = entry_extra(e);
  const u32 length = entry_value(e) + ((v >> L) & ((1u << E) - 1u));
  c.consume(L + E);
  c.refill();
  v = c.lo;
  u32 d = t.d.lut[v & 255u];
  u32 dk = entry_kind(d);
  if (dk == kLong) {
    d = decode_long(t.d, v, DFn());
    dk = entry_kind(d);
  }
  if (dk != kLiteral) return kLaneIrregular;
  const u32 Ld = entry_len(d), Ed = entry_extra(d);
  const u32 span = entry_value(d) + ((v >> Ld) & ((1u << Ed) - 1u));
  if (span > window) return kLaneIrregular;
  c.consume(Ld + Ed);
  *bytes = length;
  *sym = match_symbol(length, span);
  return kLaneWindow;
}

// Marks of one lane's row in [a, b) (bit offsets within its window).
__device__ __forceinline__ u32 marks_between(const u32* row, u32 a, u32 b) {
  u32 n = 0;
  for (u32 k = a >> 5; k < kMarkWords && (k << 5) < b; ++k) {
    u32 w = row[k];
    const u32 lo = k << 5;
    if (lo < a) w &= ~0u << (a - lo);
    if (b - lo < 32) w &= (1u << (b - lo)) - 1u;
    n += __popc(w);
  }
  return n;
}

// Phase 1 of a round on one lane: decode its window from s, marking token
// starts and keeping the tokens; stop/stop_at say where and why it ended.
// The mark word being filled stays in a register until the tokens move past
// it.  kChecked = false when the window ends 48 bits or more before the
// body end, so no token needs the end check.
template <bool kChecked>
__device__ __forceinline__ void window_pass(AheadBits& c, const Tables& t, u32 window, u32 s,
                                            u32 wend, u32 fixed_stop, u32* my_marks,
                                            u32* kept_at, u32& kept, u32& stop, u32& stop_at,
                                            u32& block_end) {
  u32 mark_index = 0, mark_word = 0, bytes = 0, sym = 0;
  for (;;) {
    const u32 p = c.pos();
    if (p >= wend) {
      stop = kLaneWindow;
      stop_at = p;
      break;
    }
    if (p == fixed_stop) {
      stop = kLaneFixedStop;
      stop_at = p;
      break;
    }
    const u32 off = p - s;
    if ((off >> 5) != mark_index) {
      my_marks[mark_index] = mark_word;
      mark_index = off >> 5;
      mark_word = 0;
    }
    mark_word |= 1u << (off & 31);
    const u32 st = symbol_token<kChecked>(c, t, window, &bytes, &sym);
    if (st != kLaneWindow) {
      stop = st;
      stop_at = p;
      if (st == kLaneBlockEnd) block_end = c.pos();
      break;
    }
    if (kept_at && kept < kStash) kept_at[kept * 32] = sym;
    ++kept;
  }
  my_marks[mark_index] = mark_word;
}

// Phase 2 on one lane: decode on past the window until landing on a later
// lane's mark, passing the round's end, or stopping; link/link_at/link_to
// say which.  kChecked as for window_pass, over the whole round.
template <bool kChecked>
__device__ __forceinline__ void run_on(AheadBits& c, const Tables& t, u32 window, u32 start,
                                       u32 round_end, u32 fixed_stop, const RoundShared& r,
                                       u32* kept_at, u32& kept, u32& cont_tokens, u32& link,
                                       u32& link_at, u32& link_to, u32& block_end) {
  u32 bytes = 0, sym = 0;
  for (;;) {
    const u32 p = c.pos();
    if (p >= round_end) {
      link = kLaneWindow;
      link_at = p;
      break;
    }
    if (p == fixed_stop) {
      link = kLaneFixedStop;
      link_at = p;
      break;
    }
    const u32 to = (p - start) / kRoundWindow, off = p - (start + to * kRoundWindow);
    if ((r.marks[to][off >> 5] >> (off & 31)) & 1u) {
      link = kLaneMerged;
      link_at = p;
      link_to = to;
      break;
    }
    const u32 st = symbol_token<kChecked>(c, t, window, &bytes, &sym);
    if (st != kLaneWindow) {
      link = st;
      link_at = p;
      if (st == kLaneBlockEnd) block_end = c.pos();
      break;
    }
    if (kept_at && kept < kStash) kept_at[kept * 32] = sym;
    ++kept;
    ++cont_tokens;
  }
}

// One round from the token boundary `start` (the same on every lane).  On
// every lane: the committed position, the output bytes and tokens before
// it, and whether the block continues, ended (position after its
// end-of-block code) or goes to the serial decoder at that position.  With
// kWrite, the round's tokens go to the sink in order: each lane's region
// holds as many tokens as it marked after its entry plus those it decoded
// past its window, so a warp scan places every lane's tokens before phase 3
// writes them.  `stash` (the warp's kStash * 32 words, or null) keeps every
// lane's decoded tokens, token k of lane i at word 32 k + i, so that the
// stores of one loop step are coalesced; phase 3 copies a region from there,
// starting at the token its entry mark counts to.
// fixed_stop: a position inside a fixed-Huffman block at which the node
// must end if its token chain starts a token there (~0u for none); the
// round then ends there with kRoundFixedStop.
template <bool kWrite>
__device__ RoundResult warp_round(const u8* body, u32 body_bytes, u32 start, u32 window,
                                  u32 fixed_stop, const Tables& t, RoundShared& r,
                                  SymbolSink& sink, u32* stash) {
  const u32 lane = threadIdx.x & 31u;
  u32* const kept_at = stash ? stash + lane : nullptr;
  u32 kept = 0;         // tokens decoded in phases 1 and 2
  u32 block_end = 0;    // position after an end-of-block code either phase met
  const u32 s = start + lane * kRoundWindow, wend = s + kRoundWindow;
  const u32 round_end = start + 32 * kRoundWindow;
  u32* my_marks = r.marks[lane];
  for (u32 k = 0; k < kMarkWords; ++k) my_marks[k] = 0;
  AheadBits c;
  c.init(body, body_bytes);
  u32 bytes = 0, sym = 0;
  // Phase 1: speculative decode of the window, marking token starts.  The
  // mark word being filled stays in a register until the tokens move past
  // it; windows ending 48 bits or more before the body end skip the
  // per-token end check.
  u32 stop = kLaneIrregular, stop_at = s;
  if (s < c.end) {
    c.seek(s);
    if (wend + 48 <= c.end)
      window_pass<false>(c, t, window, s, wend, fixed_stop, my_marks, kept_at, kept, stop,
                         stop_at, block_end);
    else
      window_pass<true>(c, t, window, s, wend, fixed_stop, my_marks, kept_at, kept, stop,
                        stop_at, block_end);
  }
  __syncwarp();
  // Phase 2: run on until landing on a later lane's mark (or past the round).
  u32 link = stop, link_at = stop_at, link_to = lane, cont_tokens = 0;
  if (stop == kLaneWindow) {
    if (round_end + 48 <= c.end)
      run_on<false>(c, t, window, start, round_end, fixed_stop, r, kept_at, kept, cont_tokens,
                    link, link_at, link_to, block_end);
    else
      run_on<true>(c, t, window, start, round_end, fixed_stop, r, kept_at, kept, cont_tokens,
                   link, link_at, link_to, block_end);
  }
  r.link[lane] = link;
  r.link_at[lane] = link_at;
  r.link_to[lane] = link_to;
  r.region_to[lane] = 0;
  r.region_end[lane] = kLaneIrregular;
  r.region_from[lane] = 1;  // empty region (from > to)
  __syncwarp();
  // Walk: the true chain from lane 0, lane to lane (always to higher lanes).
  if (lane == 0) {
    u32 j = 0, from = start;
    for (;;) {
      r.region_from[j] = from;
      const u32 kind = r.link[j];
      r.region_to[j] = r.link_at[j];
      r.region_end[j] = kind;
      if (kind != kLaneMerged) break;
      from = r.link_at[j];
      j = r.link_to[j];
    }
  }
  __syncwarp();
  const u32 from = r.region_from[lane], to = r.region_to[lane], end = r.region_end[lane];
  const bool visited = from <= to;
  // Tokens of the region: marks from the entry on (up to the early stop when
  // phase 1 ended the region), plus the tokens phase 2 decoded.
  u32 expect = 0;
  if (visited) {
    expect = stop == kLaneWindow ? marks_between(my_marks, from - s, kRoundWindow) + cont_tokens
                                 : marks_between(my_marks, from - s, stop_at - s);
  }
  u32 before = expect;
  for (u32 o = 1; o < 32; o <<= 1) {
    const u32 v = __shfl_up_sync(kFullMask, before, o);
    if (lane >= o) before += v;
  }
  before -= expect;
  if (kWrite) {
    const u32 all = __shfl_sync(kFullMask, before + expect, 31);
    if (lane == 0) sink.reserve(all, r);
    __syncwarp();
  }
  const bool drop = kWrite && r.drop;
  // Phase 3: the region's tokens, copied from the stash when the lane kept
  // them all (its tokens before the entry are the marks before it), else
  // decoded again.
  u32 total = 0, tokens = 0, finish = to, broken = 0;
  const u32 entry = visited && kept_at ? marks_between(my_marks, 0, from - s) : 0u;
  if (visited && kept_at && kept <= kStash) {
    // Loads in groups of eight, ahead of the stores, so the copy waits on
    // memory once per group rather than once per token.
    constexpr u32 kGroup = 8;
    for (; tokens + kGroup <= expect; tokens += kGroup) {
      u32 word[kGroup];
#pragma unroll
      for (u32 g = 0; g < kGroup; ++g) word[g] = kept_at[(entry + tokens + g) * 32];
#pragma unroll
      for (u32 g = 0; g < kGroup; ++g) {
        if (kWrite && !drop) *sink.slot(r, before + tokens + g) = word[g];
        total += word[g] & kMatchFlag ? word[g] & 511u : 1u;
      }
    }
    for (; tokens < expect; ++tokens) {
      const u32 word = kept_at[(entry + tokens) * 32];
      if (kWrite && !drop) *sink.slot(r, before + tokens) = word;
      total += word & kMatchFlag ? word & 511u : 1u;
    }
    if (end == kLaneBlockEnd) finish = block_end;
  } else if (visited) {
    c.seek(from);
    // The same tokens phases 1 and 2 took; any other answer would be a
    // decoder fault, and the round is then dropped.
    while (c.pos() < to) {
      if (symbol_token(c, t, window, &bytes, &sym) != kLaneWindow || tokens == expect) {
        broken = 1;
        break;
      }
      if (kWrite && !drop) *sink.slot(r, before + tokens) = sym;
      ++tokens;
      total += bytes;
    }
    if (!broken && (c.pos() != to || tokens != expect)) broken = 1;
    if (!broken && end == kLaneBlockEnd) {
      if (symbol_token(c, t, window, &bytes, &sym) != kLaneBlockEnd) broken = 1;
      finish = c.pos();
    }
  }
  u32 count = tokens;
  for (u32 o = 16; o; o >>= 1) {
    total += __shfl_xor_sync(kFullMask, total, o);
    count += __shfl_xor_sync(kFullMask, count, o);
  }
  // The lane whose region ends the walk holds the round's end.
  const u32 enders = __ballot_sync(kFullMask, visited && end != kLaneMerged);
  RoundResult out{start, 0, 0, kRoundFallback};
  if (enders && !__any_sync(kFullMask, broken)) {
    const u32 who = __ffs(enders) - 1;
    const u32 outcome_end = __shfl_sync(kFullMask, end, who);
    out.pos = __shfl_sync(kFullMask, finish, who);
    out.bytes = total;
    out.tokens = count;
    out.outcome = outcome_end == kLaneWindow ? kRoundMore
                : outcome_end == kLaneBlockEnd ? kRoundBlockEnd
                : outcome_end == kLaneFixedStop ? kRoundFixedStop : kRoundFallback;
  }
  __syncwarp();
  return out;
}

struct NodeShared {
  Tables dyn[kNodeWarps];
  RoundShared round[kNodeWarps];
};
struct ExpandShared {
  __align__(16) u16 ring[kExpandWarps][kEmitRing];
  u32 token[kExpandWarps][kChunkTokens];  // the chunk's tokens and output offsets
  u32 at[kExpandWarps][kChunkTokens];
};

// ---------------------------------------------------------------------------
// Candidate compaction: bitmap over body bit offsets -> sorted u32 list.
// ---------------------------------------------------------------------------
constexpr u32 kCompactWords = 4096;  // bitmap words per CTA (131072 offsets)

// The fast path's candidates are the reference rule's (bitmap) and the
// fast-only stored-run seeds (extra), one bit per body bit offset each.
__global__ void cand_count_kernel(const u32* bitmap, const u32* extra, u32 words,
                                  u32* block_counts) {
  __shared__ u32 warp_sum[8];
  const u32 base = blockIdx.x * kCompactWords;
  u32 count = 0;
  for (u32 i = threadIdx.x; i < kCompactWords && base + i < words; i += blockDim.x)
    count += __popc(bitmap[base + i] | extra[base + i]);
  for (u32 o = 16; o; o >>= 1) count += __shfl_xor_sync(kFullMask, count, o);
  if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = count;
  __syncthreads();
  if (threadIdx.x == 0) {
    u32 total = 0;
    for (u32 w = 0; w < blockDim.x / 32; ++w) total += warp_sum[w];
    block_counts[blockIdx.x] = total;
  }
}

// extra |= bitmap, grid-stride: the candidate headers nodes stop at.
__global__ void bitmap_or_kernel(const u32* bitmap, u32* extra, u32 words) {
  for (u32 i = blockIdx.x * blockDim.x + threadIdx.x; i < words; i += gridDim.x * blockDim.x)
    extra[i] |= bitmap[i];
}

// Exclusive scan of block_counts in place (one CTA); total -> *total.
__global__ void cand_scan_kernel(u32* block_counts, u32 blocks, u32* total) {
  __shared__ u32 carry;
  __shared__ u32 warp_sum[32];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (u32 base = 0; base < blocks; base += blockDim.x) {
    const u32 i = base + threadIdx.x;
    const u32 v = i < blocks ? block_counts[i] : 0;
    u32 incl = v;
    for (u32 o = 1; o < 32; o <<= 1) {
      const u32 t = __shfl_up_sync(kFullMask, incl, o);
      if ((threadIdx.x & 31) >= o) incl += t;
    }
    if ((threadIdx.x & 31) == 31) warp_sum[threadIdx.x >> 5] = incl;
    __syncthreads();
    if (threadIdx.x < 32) {
      u32 w = threadIdx.x < blockDim.x / 32 ? warp_sum[threadIdx.x] : 0;
      for (u32 o = 1; o < 32; o <<= 1) {
        const u32 t = __shfl_up_sync(kFullMask, w, o);
        if (threadIdx.x >= o) w += t;
      }
      warp_sum[threadIdx.x] = w;  // inclusive per warp
    }
    __syncthreads();
    const u32 warp = threadIdx.x >> 5;
    const u32 before = carry + (warp ? warp_sum[warp - 1] : 0) + incl - v;
    if (i < blocks) block_counts[i] = before;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = before + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

__global__ void cand_write_kernel(const u32* bitmap, const u32* extra, u32 words,
                                  const u32* block_offsets, u32* cands, u32 capacity) {
  __shared__ u32 warp_sum[8];
  const u32 base = blockIdx.x * kCompactWords;
  const u32 per = kCompactWords / blockDim.x;  // contiguous words per thread
  const u32 first = base + threadIdx.x * per;
  u32 count = 0;
  for (u32 k = 0; k < per; ++k)
    if (first + k < words) count += __popc(bitmap[first + k] | extra[first + k]);
  u32 incl = count;
  for (u32 o = 1; o < 32; o <<= 1) {
    const u32 t = __shfl_up_sync(kFullMask, incl, o);
    if ((threadIdx.x & 31) >= o) incl += t;
  }
  if ((threadIdx.x & 31) == 31) warp_sum[threadIdx.x >> 5] = incl;
  __syncthreads();
  u32 before = block_offsets[blockIdx.x] + incl - count;
  for (u32 w = 0; w < (threadIdx.x >> 5); ++w) before += warp_sum[w];
  for (u32 k = 0; k < per; ++k) {
    if (first + k >= words) break;
    u32 bits = bitmap[first + k] | extra[first + k];
    while (bits) {
      const u32 b = __ffs(bits) - 1;
      bits &= bits - 1;
      if (before < capacity) cands[before] = (first + k) * 32 + b;
      ++before;
    }
  }
}

// ---------------------------------------------------------------------------
// Node walk: decode from a candidate through any following stored/fixed
// blocks up to the next dynamic header.  Describe counts; the symbols
// kernel also writes the node's tokens to `syms` (room for `room` words).
// ---------------------------------------------------------------------------
struct NodeResult {
  u32 end, size, blocks, info, tokens;
  // First end-of-block code of a node that starts inside a fixed block:
  // where the node ends if that block is the stream's final one.
  u32 has_eob, eob_end, eob_size, eob_tokens;
};

// Where nodes stop besides the stream end: at a block header that is a
// candidate (header_bits: one bit per body bit offset), and, while inside a
// fixed-Huffman block, exactly at a fixed-region seed (sorted positions).
struct NodeStops {
  const u32* header_bits;
  const u32* fixed;
  u32 fixed_count;
};

__device__ __forceinline__ bool bit_set(const u32* bits, u32 p) {
  return (__ldg(bits + (p >> 5)) >> (p & 31)) & 1u;
}

// First fixed seed strictly after p, or ~0u.
__device__ __forceinline__ u32 seed_after(const NodeStops& stops, u32 p) {
  u32 lo = 0, hi = stops.fixed_count;
  while (lo < hi) {
    const u32 mid = (lo + hi) >> 1;
    if (__ldg(stops.fixed + mid) <= p) lo = mid + 1;
    else hi = mid;
  }
  return lo < stops.fixed_count ? __ldg(stops.fixed + lo) : ~0u;
}

// Decode one node.  A node starts at a header candidate, or (fixed_entry)
// at a fixed-region seed inside a fixed-Huffman block whose final flag is
// entry_final; it runs through blocks until the stream ends, the next block
// header is a candidate, or, inside a fixed block, its token chain starts a
// token exactly at a fixed seed.
template <bool kWrite>
__device__ NodeResult warp_node(const u8* body, u32 bytes, u32 start, bool fixed_entry,
                                u32 entry_final, u32 expected, u32 window, const NodeStops& stops,
                                const Tables& fixed, Tables& dyn, RoundShared& rounds,
                                SymbolSink& sink, u32* stash) {
  const u32 lane = threadIdx.x & 31u;
  NodeResult r{start, 0, 0, 0, 0, 0, 0, 0, 0};
  Bits c;
  u32 produced = 0, tokens = 0, final = entry_final, blocks = 0, full_words = 0;
  u32 fail = 0, stop = 0, ended_final = 0, fixed_hit = 0;
  u32 has_eob = 0, eob_end = 0, eob_size = 0, eob_tokens = 0;
  bool need_header = !fixed_entry;
  bool parallel = fixed_entry;  // this block's body goes through lane-parallel rounds
  bool in_fixed = fixed_entry;  // inside a fixed-Huffman block body
  u32 next_stop = ~0u;          // first fixed seed past the position (inside fixed blocks)
  if (fixed_entry) warp_load_fixed(dyn, fixed);
  if (lane == 0) {
    c.init(body, bytes);
    c.seek(start);
    full_words = (c.shift + c.end) >> 5;
    if (fixed_entry) next_stop = seed_after(stops, start);
  }
  const u32 limit = expected;  // output bound of a node
  // Lane 0 appends one symbol word.
  auto put = [&](u32 word) {
    if (kWrite) sink.put(word);
    ++tokens;
  };
  // Lane 0, at a token boundary p inside a fixed block: is p the next seed?
  // (Seeds the chain jumps over are skipped.)
  auto at_seed = [&](u32 p) -> bool {
    if (p < next_stop) return false;
    if (p == next_stop) return true;
    next_stop = seed_after(stops, p - 1);
    return p == next_stop;
  };
  // Lane 0, after an end-of-block code: the first one is kept for the
  // final-block reading of a fixed-entry node.
  auto block_end = [&]() {
    need_header = true;
    in_fixed = false;
    next_stop = ~0u;
    if (fixed_entry && !has_eob) {
      has_eob = 1;
      eob_end = c.pos();
      eob_size = produced;
      eob_tokens = tokens;
    }
    if (final) {
      stop = 1;
      ended_final = 1;
    }
  };
  for (;;) {
    u32 action = kNone;
    if (lane == 0) {
      while (!fail && !stop) {
        if (need_header) {
          const u32 header = c.pos();
          if (header != start && bit_set(stops.header_bits, header)) {
            stop = 1;  // the next node starts at this candidate
            break;
          }
          u32 err = 0;
          const u32 f = c.take(1, &err), type = c.take(2, &err);
          if (err || type == 3) { fail = 1; break; }
          final = f;
          ++blocks;
          if (type == 0) {
            c.seek((c.pos() + 7) & ~7u);
            const u32 n = c.take(16, &err), comp = c.take(16, &err);
            const u32 at = c.pos();
            if (err || (n ^ comp) != 0xffffu || n > limit - produced || at > c.end ||
                n * 8 > c.end - at) { fail = 1; break; }
            if (n) {
              if (kWrite) sink.put_pair(kStoredFlag | n, at >> 3);
              tokens += 2;
            }
            produced += n;
            c.seek(at + n * 8);
            if (final) {
              stop = 1;
              ended_final = 1;
            }
            continue;
          }
          action = type == 2 ? kDynamic : kFixed;
          break;
        }
        if (parallel) {
          action = kRound;
          break;
        }
        if (in_fixed && at_seed(c.pos())) {
          stop = 1;
          fixed_hit = 1;
          break;
        }
        const Tables& t = dyn;
        // One bound for the fast loop: room for a maximal match.
        const u32 stop_at = limit >= 258 ? limit - 258 : 0;
        const u32 idx_limit = full_words >= 2 ? full_words - 1 : 0;
        bool seed = false;
        while (c.idx < idx_limit && produced < stop_at) {
          if (in_fixed && at_seed(c.pos())) {
            seed = true;
            break;
          }
          c.refill_fast();
          const u32 v = c.lo;
          const u32 e = t.ll.lut[v & kLLMask];
          const u32 kind = entry_kind(e);
          if (kind == kLiteral) {
            c.consume(entry_len(e));
            put(entry_value(e));
            ++produced;
            continue;
          }
          if (kind != kLength) break;
          const u32 saved_lo = c.lo, saved_hi = c.hi;
          const u32 saved_bits = c.nbits, saved_idx = c.idx;
          const u32 L = entry_len(e), E = entry_extra(e);
          const u32 length = entry_value(e) + ((v >> L) & ((1u << E) - 1u));
          c.consume(L + E);
          c.refill_fast();
          const u32 w = c.lo;
          const u32 d = t.d.lut[w & 255u];
          const u32 Ld = entry_len(d), Ed = entry_extra(d);
          const u32 span = entry_value(d) + ((w >> Ld) & ((1u << Ed) - 1u));
          if (entry_kind(d) != kLiteral || span > window) {
            c.lo = saved_lo;
            c.hi = saved_hi;
            c.nbits = saved_bits;
            c.idx = saved_idx;
            break;
          }
          c.consume(Ld + Ed);
          put(match_symbol(length, span));
          produced += length;
        }
        if (seed) {
          stop = 1;
          fixed_hit = 1;
          break;
        }
        if (fail) break;
        if (in_fixed && at_seed(c.pos())) {
          stop = 1;
          fixed_hit = 1;
          break;
        }
        const Token tok = take_token(c, t);
        if (tok.kind == kTokError) { fail = 1; break; }
        if (tok.kind == kTokEnd) {
          block_end();
          continue;
        }
        const u32 size = tok.kind == kTokLiteral ? 1u : tok.length;
        if (size > limit - produced) { fail = 1; break; }
        if (tok.kind == kTokLiteral) {
          put(tok.value);
          ++produced;
          continue;
        }
        if (tok.dist > window) { fail = 1; break; }
        put(match_symbol(tok.length, tok.dist));
        produced += tok.length;
      }
    }
    fail = __shfl_sync(kFullMask, fail, 0);
    if (fail) break;
    action = __shfl_sync(kFullMask, action, 0);
    const bool done = __shfl_sync(kFullMask, stop, 0) != 0;
    if (action == kDynamic) {
      const u32 st = warp_dynamic_header(c, dyn);
      if (st) { fail = 1; break; }
      if (lane == 0) {
        need_header = false;
        parallel = true;
        in_fixed = false;
        next_stop = ~0u;
      }
    } else if (action == kFixed) {
      warp_load_fixed(dyn, fixed);
      if (lane == 0) {
        need_header = false;
        parallel = true;
        in_fixed = true;
        next_stop = seed_after(stops, c.pos() - 1);
      }
    } else if (action == kRound) {
      u32 from = 0, seed = ~0u;
      if (lane == 0) {
        from = c.pos();
        if (in_fixed) {
          if (from > next_stop) next_stop = seed_after(stops, from - 1);
          seed = next_stop;
        }
      }
      from = __shfl_sync(kFullMask, from, 0);
      seed = __shfl_sync(kFullMask, seed, 0);
      const RoundResult rr = warp_round<kWrite>(body, bytes, from, window, seed, dyn, rounds,
                                                sink, stash);
      if (lane == 0) {
        if (rr.bytes > limit - produced) {
          // The round would pass the output bound: the serial decoder takes
          // the block from the round's start and reports it exactly.
          parallel = false;
        } else {
          produced += rr.bytes;
          tokens += rr.tokens;
          c.seek(rr.pos);
          if (rr.outcome == kRoundFallback) {
            // The serial decoder takes the rest of the block from the last
            // boundary known to be on the true chain.
            parallel = false;
          } else if (rr.outcome == kRoundBlockEnd) {
            parallel = false;
            block_end();
          } else if (rr.outcome == kRoundFixedStop) {
            stop = 1;
            fixed_hit = 1;
          }
        }
      }
    }
    __syncwarp();
    if (done || __shfl_sync(kFullMask, stop, 0)) break;
  }
  if (kWrite && lane == 0) sink.finish();
  r.end = __shfl_sync(kFullMask, c.pos(), 0);
  r.size = __shfl_sync(kFullMask, produced, 0);
  r.blocks = __shfl_sync(kFullMask, blocks, 0);
  r.tokens = __shfl_sync(kFullMask, tokens, 0);
  r.has_eob = __shfl_sync(kFullMask, has_eob, 0);
  r.eob_end = __shfl_sync(kFullMask, eob_end, 0);
  r.eob_size = __shfl_sync(kFullMask, eob_size, 0);
  r.eob_tokens = __shfl_sync(kFullMask, eob_tokens, 0);
  const u32 spilled = kWrite ? __shfl_sync(kFullMask, sink.spilled, 0) : 0u;
  const u32 hit = __shfl_sync(kFullMask, fixed_hit, 0);
  r.info = (fail ? 0u : kInfoOk) | (__shfl_sync(kFullMask, ended_final, 0) ? kInfoFinal : 0u) |
           (spilled ? kInfoSpilled : 0u) | (hit ? kInfoFixedStop : 0u) |
           (hit && __shfl_sync(kFullMask, final, 0) ? kInfoExitFinal : 0u);
  return r;
}

// Node ids: header candidates 0 .. K-1 (K = min(total, capacity)), then two
// per fixed seed j: K + 2j (the seed's block is not the final one) and
// K + 2j + 1 (it is).
struct NodeSpace {
  u32 headers, seeds;
  __device__ __forceinline__ u32 count() const { return headers + 2 * seeds; }
};
__device__ __forceinline__ NodeSpace node_space(const u32* total, u32 capacity,
                                                const u32* fixed_total, u32 fixed_capacity) {
  return NodeSpace{min_u32(*total, capacity), min_u32(*fixed_total, fixed_capacity)};
}

// Describe every candidate and fixed seed (warp per item, work stealing).
// A seed is decoded once, for the non-final reading; its final-block
// reading ends at the first end-of-block code, or, without one, where the
// other ends.
__global__ void __launch_bounds__(kNodeWarps * 32)
describe_kernel(const u8* in, u32 in_size, u64 expected, const u32* cands, const u32* total,
                u32 capacity, const u32* fixed, const u32* fixed_total, u32 fixed_capacity,
                const u32* header_bits, u32* next_item, u32* ends, u32* sizes, u32* blocks,
                u32* infos, u32* tokens, u32* first_page, u32* pool, u32* page_next,
                u32* page_used, u32* page_cursor, u32 npages, const Tables* fixed_tables,
                u32* stash) {
  __shared__ NodeShared sh;
  const u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  u32* const warp_stash = stash + (u64(blockIdx.x) * kNodeWarps + warp) * (32 * kStash);
  u32 window = 0, wanted = 0;
  if (zlib_framing(in, in_size, &window, &wanted)) return;
  const NodeSpace ns = node_space(total, capacity, fixed_total, fixed_capacity);
  const NodeStops stops{header_bits, fixed, ns.seeds};
  for (;;) {
    u32 item = 0;
    if (lane == 0) item = atomicAdd(next_item, 1u);
    item = __shfl_sync(kFullMask, item, 0);
    if (item >= ns.headers + ns.seeds) break;
    const bool seed = item >= ns.headers;
    const u32 node = seed ? ns.headers + 2 * (item - ns.headers) : item;
    const u32 start = seed ? fixed[item - ns.headers] : cands[item];
    SymbolSink sink{SymbolSink::kPages, pool, 0, page_next, page_used, page_cursor, npages,
                    kNoPage, 0, kNoPage, 0, 0};
    const NodeResult r = warp_node<true>(in + 2, in_size - 6, start, seed, 0u, u32(expected),
                                         window, stops, *fixed_tables, sh.dyn[warp],
                                         sh.round[warp], sink, warp_stash);
    if (lane == 0) {
      first_page[node] = sink.first;
      ends[node] = r.end;
      sizes[node] = r.size;
      blocks[node] = r.blocks;
      infos[node] = r.info;
      tokens[node] = r.tokens;
      if (seed) {
        const u32 v = node + 1;
        first_page[v] = sink.first;
        if (r.has_eob) {
          ends[v] = r.eob_end;
          sizes[v] = r.eob_size;
          blocks[v] = 0;
          infos[v] = kInfoOk | kInfoFinal | (r.info & kInfoSpilled);
          tokens[v] = r.eob_tokens;
        } else {
          ends[v] = r.end;
          sizes[v] = r.size;
          blocks[v] = r.blocks;
          infos[v] = r.info | ((r.info & kInfoFixedStop) ? kInfoExitFinal : 0u);
          tokens[v] = r.tokens;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Chain: successor links, pointer doubling from bit 0, prefixes and checks.
// One CTA.  state[0] = path length, state[1] = chain ok, state[2] = some path
// node spilled its tokens (use the contiguous layout).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
chain_kernel(const u8* in, u32 in_size, u64 expected, u32 max_blocks, const u32* cands,
             const u32* total, u32 capacity, const u32* fixed, const u32* fixed_total,
             u32 fixed_capacity, const u32* ends, const u32* sizes, const u32* blocks,
             const u32* infos, const u32* tokens, u32* jump, u32 levels, u32* path, u32* prefix,
             u32* tprefix, u32* state) {
  __shared__ u32 warp_sum[32], warp_tsum[32];
  __shared__ u32 s_len, s_ok, s_carry, s_tcarry, s_blocks;
  const u32 tid = threadIdx.x;
  u32 window = 0, wanted = 0;
  const NodeSpace ns = node_space(total, capacity, fixed_total, fixed_capacity);
  if (zlib_framing(in, in_size, &window, &wanted) || *total > capacity || !ns.headers ||
      cands[0] != 0) {
    if (tid == 0) { state[0] = 0; state[1] = 0; state[2] = 0; }
    return;
  }
  const u32 count = ns.count();
  const u32 end_node = count, bad_node = count + 1, nodes = count + 2;
  // Level 0: successors.  A node that ended on a fixed seed continues at that
  // seed's node for the final flag of the block in progress; any other
  // ending position must be a header candidate.
  for (u32 i = tid; i < nodes; i += blockDim.x) {
    u32 next = bad_node;
    if (i == end_node) next = end_node;
    else if (i < count) {
      const u32 info = infos[i];
      if (info & kInfoOk) {
        if (info & kInfoFinal) {
          next = end_node;
        } else {
          const u32 target = ends[i];
          const bool to_seed = (info & kInfoFixedStop) != 0;
          const u32* list = to_seed ? fixed : cands;
          const u32 n = to_seed ? ns.seeds : ns.headers;
          u32 lo = 0, hi = n;
          while (lo < hi) {
            const u32 mid = (lo + hi) >> 1;
            if (list[mid] < target) lo = mid + 1;
            else hi = mid;
          }
          if (lo < n && list[lo] == target)
            next = to_seed ? ns.headers + 2 * lo + ((info & kInfoExitFinal) ? 1u : 0u) : lo;
        }
      }
    }
    jump[i] = next;
  }
  __syncthreads();
  for (u32 k = 1; k < levels; ++k) {
    const u32* prev = jump + u64(k - 1) * nodes;
    u32* cur = jump + u64(k) * nodes;
    for (u32 i = tid; i < nodes; i += blockDim.x) cur[i] = prev[prev[i]];
    __syncthreads();
  }
  if (tid == 0) {
    // Nodes on the path from node 0 (bit 0), excluding the terminal sink.
    u32 node = 0, len = 1;
    for (u32 k = levels; k-- > 0;) {
      const u32 n = jump[u64(k) * nodes + node];
      if (n < count) {
        node = n;
        len += 1u << k;
      }
    }
    const u32 terminal = jump[node];
    s_len = len;
    s_ok = terminal == end_node;
    s_carry = 0;
    s_tcarry = 0;
    s_blocks = 0;
  }
  __syncthreads();
  const u32 len = s_len;
  if (!s_ok) {
    if (tid == 0) { state[0] = 0; state[1] = 0; state[2] = 0; }
    return;
  }
  for (u32 base = 0; base < len; base += blockDim.x) {
    const u32 m = base + tid;
    u32 node = 0, size = 0, nb = 0, nt = 0;
    if (m < len) {
      for (u32 k = 0; k < levels; ++k)
        if ((m >> k) & 1u) node = jump[u64(k) * nodes + node];
      path[m] = node;
      size = sizes[node];
      nb = blocks[node];
      nt = tokens[node];
    }
    u32 incl = size, bincl = nb, tincl = nt;
    for (u32 o = 1; o < 32; o <<= 1) {
      const u32 t = __shfl_up_sync(kFullMask, incl, o);
      const u32 tb = __shfl_up_sync(kFullMask, bincl, o);
      const u32 tt = __shfl_up_sync(kFullMask, tincl, o);
      if ((tid & 31) >= o) { incl += t; bincl += tb; tincl += tt; }
    }
    if ((tid & 31) == 31) {
      warp_sum[tid >> 5] = incl;
      warp_tsum[tid >> 5] = tincl;
    }
    __syncthreads();
    u32 before = s_carry + incl - size, tbefore = s_tcarry + tincl - nt;
    for (u32 w = 0; w < (tid >> 5); ++w) {
      before += warp_sum[w];
      tbefore += warp_tsum[w];
    }
    if (m < len) {
      prefix[m] = before;
      tprefix[m] = tbefore;
    }
    if ((tid & 31) == 31) atomicAdd(&s_blocks, bincl);
    __syncthreads();
    if (tid == blockDim.x - 1 || m == len - 1) {
      s_carry = before + size;
      s_tcarry = tbefore + nt;
    }
    __syncthreads();
  }
  if (tid == 0) {
    const u32 last = path[len - 1];
    const u32 body = in_size - 6;
    const bool ok = u64(s_carry) == expected && (ends[last] + 7) / 8 == body &&
                    s_blocks <= max_blocks;
    state[0] = ok ? len : 0;
    state[1] = ok ? 1u : 0u;
  }
  // Any path node whose tokens did not all fit the page arena sends the whole
  // stream through the contiguous layout (symbols_kernel decodes again).
  if (tid == 0) state[2] = 0;
  __syncthreads();
  for (u32 m = tid; m < len; m += blockDim.x)
    if (infos[path[m]] & kInfoSpilled) state[2] = 1;
}

// Decode every path node again, writing its tokens at its place in the
// symbol arena (warp per node, work stealing).
__global__ void __launch_bounds__(kNodeWarps * 32)
symbols_kernel(const u8* in, u32 in_size, u64 expected, const u32* cands, const u32* total,
               u32 capacity, const u32* fixed, const u32* fixed_total, u32 fixed_capacity,
               const u32* header_bits, const u32* path, const u32* tprefix, const u32* sizes,
               const u32* tokens, const u32* state, u32* next_item, u32* syms, u32* fail_flag,
               const Tables* fixed_tables, u32* stash) {
  __shared__ NodeShared sh;
  const u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  u32* const warp_stash = stash + (u64(blockIdx.x) * kNodeWarps + warp) * (32 * kStash);
  if (!state[1] || !state[2]) return;
  const u32 len = state[0];
  u32 window = 0, wanted = 0;
  zlib_framing(in, in_size, &window, &wanted);
  const NodeSpace ns = node_space(total, capacity, fixed_total, fixed_capacity);
  const NodeStops stops{header_bits, fixed, ns.seeds};
  for (;;) {
    u32 item = 0;
    if (lane == 0) item = atomicAdd(next_item, 1u);
    item = __shfl_sync(kFullMask, item, 0);
    if (item >= len) break;
    const u32 node = path[item];
    const bool seed = node >= ns.headers;
    const u32 start = seed ? fixed[(node - ns.headers) >> 1] : cands[node];
    const u32 entry_final = seed ? (node - ns.headers) & 1u : 0u;
    SymbolSink sink{SymbolSink::kContiguous, syms + tprefix[item], tokens[node], nullptr, nullptr,
                    nullptr, 0, kNoPage, 0, kNoPage, 0, 0};
    const NodeResult r = warp_node<true>(in + 2, in_size - 6, start, seed, entry_final,
                                         u32(expected), window, stops, *fixed_tables,
                                         sh.dyn[warp], sh.round[warp], sink, warp_stash);
    if (lane == 0 && (!(r.info & kInfoOk) || (r.info & kInfoSpilled) || r.size != sizes[node] ||
                      r.tokens != tokens[node]))
      atomicOr(fail_flag, 1u);
  }
}

// Flush ring symbols [from, to) of a node whose output starts at `prefix`:
// bytes to `out`, markers to `source` + the `unresolved` bitmap.
__device__ void flush_symbols(const u16* ring, u8* out, u32* source, u32* unresolved, u32 prefix,
                              u32 from, u32 to) {
  const u32 lane = threadIdx.x & 31u;
  for (u32 p = from + lane; p < to; p += 32) {
    const u32 v = ring[p & kEmitMask];
    const u32 at = prefix + p;
    if (v < 256) {
      out[at] = u8(v);
    } else {
      out[at] = 0;
      source[at] = prefix - 1 - (v - 256);
      atomicOr(&unresolved[at >> 5], 1u << (at & 31));
    }
  }
}

// Symbol of node-local position q (already flushed) from global memory.
__device__ __forceinline__ u32 flushed_symbol(const u8* out, const u32* source,
                                              const u32* unresolved, u32 prefix, u32 q) {
  const u32 at = prefix + q;
  const u32 word = unresolved[at >> 5];
  const u32 byte = out[at];  // issued alongside the bitmap load
  if ((word >> (at & 31)) & 1u) return 256 + (prefix - 1 - source[at]);
  return byte;
}

// Expansion units.  A path node is expanded in units of about 2^unit_shift
// output bytes, cut at token boundaries, so that nodes much longer than the
// window (long fixed or stored runs, zeros, highly compressible data) still
// spread over many warps.  A unit starts with an empty history like a node:
// its references before its own start become markers, so every hop of a
// marker chase moves at least one unit back and the staged resolution runs
// over units.  Unit j of a node ends after the first token that reaches
// (j + 1) << unit_shift node bytes; a stored block's two words stay together.
// The unit is at least kUnitBytes and grows with the stream, so that large
// streams, whose nodes already fill the GPU, are not cut into more markers.
constexpr u32 kUnitBytes = 32768;
constexpr u32 kUnitsPerSm = 32;  // units a stream aims for per SM
constexpr u32 kPlanTokens = 8;   // token words per lane per step of the unit planner

u32 unit_shift_for(u64 expected, u32 sms) {
  u32 shift = 15;  // kUnitBytes
  while ((u64(1) << shift) * sms * kUnitsPerSm < expected && shift < 31) ++shift;
  return shift;
}

// Bytes of token word t whose preceding word is `prev` (a stored block's
// source word follows its header and takes no bytes).
__device__ __forceinline__ u32 token_bytes(u32 t, u32 prev, bool has_prev) {
  if (has_prev && (prev & kStoredFlag) && !(prev & kMatchFlag)) return 0;
  if (t & kMatchFlag) return t & 511u;
  if (t & kStoredFlag) return t & 0xffffu;
  return 1;
}

// Warp per path item: walk the node's tokens in order.  Count pass (units ==
// nullptr): units per item into `counts` and the node size check.  Write
// pass: the item's units at item_units[item] onwards.
__global__ void __launch_bounds__(256)
unit_plan_kernel(const u32* state, const u32* path, const u32* prefix, const u32* tprefix,
                 const u32* sizes, const u32* tokens, const u32* syms, const u32* first_page,
                 const u32* page_next, const u32* page_used, u32 npages, u32 unit_shift,
                 u32* counts, const u32* item_units, u32* unit_item, u32* unit_page,
                 u32* unit_first, u32* unit_tokens, u32* unit_start, u32* unit_bytes,
                 u32* fail_flag) {
  if (!state[1] || *fail_flag) return;
  const u32 len = state[0];
  const bool contiguous = state[2] != 0;
  const bool write = unit_item != nullptr;
  const u32 lane = threadIdx.x & 31u;
  const u32 warps = gridDim.x * (blockDim.x >> 5);
  for (u32 item = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; item < len; item += warps) {
    const u32 node = path[item], node_tokens = tokens[node];
    u32 left = node_tokens;
    u32 page = contiguous ? kNoPage : first_page[node];
    u64 bytes = 0;          // node bytes before the current word
    u32 units = 1, token_index = 0, bad = 0;
    u32 open_page = page, open_first = 0, open_token = 0;
    u64 open_bytes = 0;
    auto close_unit = [&](u32 end_token, u64 end_bytes, u32 next_page, u32 next_first) {
      if (write && lane == 0) {
        const u32 u = item_units[item] + units - 1;
        unit_item[u] = item;
        unit_page[u] = open_page;
        unit_first[u] = open_first;
        unit_tokens[u] = end_token - open_token;
        unit_start[u] = prefix[item] + u32(open_bytes);
        unit_bytes[u] = u32(end_bytes - open_bytes);
      }
      open_page = next_page;
      open_first = next_first;
      open_token = end_token;
      open_bytes = end_bytes;
    };
    // A node of at most one unit's bytes is one unit (no token can reach a
    // multiple of the unit before its last), so only longer nodes are
    // walked.
    if ((u64(sizes[node]) >> unit_shift) == 0 || sizes[node] == (1u << unit_shift)) {
      left = 0;
      token_index = node_tokens;
      bytes = sizes[node];
    }
    for (bool first_run = true; left && !bad; first_run = false) {
      const u32* sy;
      u32 n;
      if (contiguous) {
        sy = syms + tprefix[item];
        n = left;
      } else {
        if (page == kNoPage || page >= npages || page_used[page] > kPageWords) {
          bad = 1;
          break;
        }
        sy = syms + u64(page) * kPageWords;
        n = min_u32(page_used[page], left);
      }
      u32 carry = 0;  // the page's previous word (pairs never cross pages)
      // kPlanTokens consecutive words per lane a step; the next step's words
      // are loaded while this step's are scanned.
      u32 ahead[kPlanTokens];
#pragma unroll
      for (u32 k = 0; k < kPlanTokens; ++k) {
        const u32 i = kPlanTokens * lane + k;
        ahead[k] = i < n ? sy[i] : 0u;
      }
      for (u32 base = 0; base < n; base += 32 * kPlanTokens) {
        const u32 i0 = base + kPlanTokens * lane;
        u32 t[kPlanTokens], size[kPlanTokens];
#pragma unroll
        for (u32 k = 0; k < kPlanTokens; ++k) {
          t[k] = ahead[k];
          const u32 i = i0 + 32 * kPlanTokens + k;
          ahead[k] = i < n ? sy[i] : 0u;
        }
        u32 prev = __shfl_up_sync(kFullMask, t[kPlanTokens - 1], 1);
        if (lane == 0) prev = carry;
        u32 lane_bytes = 0;
#pragma unroll
        for (u32 k = 0; k < kPlanTokens; ++k) {
          size[k] = i0 + k < n ? token_bytes(t[k], k ? t[k - 1] : prev, i0 + k > 0) : 0u;
          lane_bytes += size[k];
        }
        u64 incl = lane_bytes;
        for (u32 o = 1; o < 32; o <<= 1) {
          const u64 v = __shfl_up_sync(kFullMask, incl, o);
          if (lane >= o) incl += v;
        }
        // A token reaching a multiple of kUnitBytes ends its unit; the next
        // unit starts after it (after a stored block's source word).
        u64 before = bytes + incl - lane_bytes;
        u32 ends = 0;
#pragma unroll
        for (u32 k = 0; k < kPlanTokens; ++k) {
          const u64 after = before + size[k];
          if (size[k] && (after >> unit_shift) > (before >> unit_shift)) ends |= 1u << k;
          before = after;
        }
        for (u32 ballot = __ballot_sync(kFullMask, ends != 0); ballot; ballot &= ballot - 1) {
          const u32 l = __ffs(ballot) - 1;
          u32 lane_ends = __shfl_sync(kFullMask, ends, l);
          u64 at = __shfl_sync(kFullMask, bytes + incl - lane_bytes, l);
#pragma unroll
          for (u32 k = 0; k < kPlanTokens; ++k) {
            const u32 tk = __shfl_sync(kFullMask, t[k], l);
            at += __shfl_sync(kFullMask, size[k], l);
            if (!((lane_ends >> k) & 1u)) continue;
            const bool header = (tk & kStoredFlag) && !(tk & kMatchFlag);
            const u32 next = base + kPlanTokens * l + k + (header ? 2u : 1u);
            if (token_index + next < node_tokens) {
              // A next unit that starts on the following page starts at
              // that page's word 0.
              const bool on_next = next >= n && !contiguous;
              close_unit(token_index + next, at, on_next ? page_next[page] : page,
                         on_next ? 0u : next);
              ++units;
            }
          }
        }
        bytes += __shfl_sync(kFullMask, incl, 31);
        carry = __shfl_sync(kFullMask, t[kPlanTokens - 1], 31);
      }
      token_index += n;
      left -= n;
      if (contiguous) break;
      page = page_next[page];
    }
    if (!bad) {
      close_unit(token_index, bytes, kNoPage, 0);
      if (bytes != sizes[node]) bad = 1;
    }
    if (lane == 0) {
      if (bad) atomicOr(fail_flag, 1u);
      if (!write) counts[item] = units;
    }
  }
}

// Exclusive prefix of the units per item (one CTA); item_units[len] is the
// total.
__global__ void unit_scan_kernel(const u32* state, const u32* counts, u32* item_units) {
  __shared__ u32 warp_total[32];
  __shared__ u32 carry;
  if (!state[1]) return;
  const u32 len = state[0];
  const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    carry = 0;
    if (!len) item_units[0] = 0;
  }
  __syncthreads();
  for (u32 base = 0; base < len; base += blockDim.x) {
    const u32 i = base + threadIdx.x;
    const u32 v = i < len ? counts[i] : 0u;
    u32 incl = v;
    for (u32 o = 1; o < 32; o <<= 1) {
      const u32 t = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_total[warp] = incl;
    __syncthreads();
    u32 before = carry;
    for (u32 w = 0; w < warp; ++w) before += warp_total[w];
    if (i < len) item_units[i] = before + incl - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) {
      carry = before + incl;
      if (base + blockDim.x >= len) item_units[len] = carry;
    }
    __syncthreads();
  }
}

// Expand every path node's tokens into the output (warp per node, work
// stealing).  The warp takes kChunkTokens tokens at a time, kLaneTokens
// consecutive ones per lane: a scan of their sizes places them, then every
// output byte of the chunk is written in parallel, copies that read the
// chunk's own output through pending entries resolved in a second pass.  The ring holds the node's recent output as u16
// symbols: a byte, or 256 + k for the byte k + 1 positions before the node
// start (a reference into an earlier node; copies propagate it); full
// stretches of the ring flush to the output, markers as source positions in
// `source` plus a bit in `unresolved`.
__global__ void __launch_bounds__(kExpandWarps * 32)
expand_kernel(const u8* in, u32 in_size, const u32* tprefix, const u32* state,
              const u32* syms, const u32* page_next, const u32* page_used, u32 npages,
              const u32* item_units, const u32* unit_item, const u32* unit_page,
              const u32* unit_first, const u32* unit_tokens, const u32* unit_start,
              const u32* unit_bytes, u32* next_item, u8* out, u32* source, u32* unresolved,
              u32* fail_flag) {
  __shared__ ExpandShared sh;
  const u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  // A failed chain or symbol pass leaves nothing to expand (the status path
  // reports the stream).
  if (!state[1] || *fail_flag) return;
  const u32 units = item_units[state[0]];
  const u8* body = in + 2;
  u16* ring = sh.ring[warp];
  for (;;) {
    u32 unit = 0;
    if (lane == 0) unit = atomicAdd(next_item, 1u);
    unit = __shfl_sync(kFullMask, unit, 0);
    if (unit >= units) break;
    const u32 item = unit_item[unit], start = unit_start[unit];
    // The unit's tokens: a stretch of the node's contiguous run, or of its
    // chain of arena pages (allocated in order, so page numbers strictly
    // increase along it), from word `skip` of its first page.
    const bool contiguous = state[2] != 0;
    u32 page = unit_page[unit], last_page = 0, skip = unit_first[unit];
    u32 pos = 0, flushed = 0, bad = 0;
    u32 left = unit_tokens[unit];
    for (bool first_run = true;; first_run = false) {
    const u32* sy = syms + tprefix[item] + skip;
    u32 n = left;
    if (!contiguous) {
      if (page == kNoPage || !left) break;
      if (page >= npages || (!first_run && page <= last_page) || page_used[page] > kPageWords ||
          (first_run && skip > page_used[page])) {
        bad = 1;
        break;
      }
      const u32 from = first_run ? skip : 0u;
      sy = syms + u64(page) * kPageWords + from;
      n = min_u32(page_used[page] - from, left);
      left -= n;
      last_page = page;
    }
    // Tokens of the chunk after the current one are loaded while the current
    // one is expanded (chunks usually take kChunkTokens tokens).
    auto load_tokens = [&](u32* t, u32 from) {
#pragma unroll
      for (u32 k = 0; k < kLaneTokens; ++k) {
        const u32 i = from + kLaneTokens * lane + k;
        t[k] = i < n ? sy[i] : kStoredFlag;
      }
    };
    u32 ahead[kLaneTokens];
    u32 ahead_at = 0;
    load_tokens(ahead, 0);
    for (u32 first = 0; first < n && !bad;) {
      if (pos - flushed >= kEmitFlush) {
        flush_symbols(ring, out, source, unresolved, start, flushed, pos);
        flushed = pos;
      }
      u32 tk[kLaneTokens];
      if (first == ahead_at) {
#pragma unroll
        for (u32 k = 0; k < kLaneTokens; ++k) tk[k] = ahead[k];
      } else {
        load_tokens(tk, first);
      }
      ahead_at = first + kChunkTokens;
      load_tokens(ahead, ahead_at);
      const u32 head = __shfl_sync(kFullMask, tk[0], 0);
      if (head & kStoredFlag && !(head & kMatchFlag)) {
        // Stored bytes: flush, then copy straight from the input.
        const u32 count = head & 0xffffu, src = sy[first + 1];
        flush_symbols(ring, out, source, unresolved, start, flushed, pos);
        // Eight independent loads per lane before the stores; only the last
        // kEmitRing bytes can still be read through the ring.
        constexpr u32 kUnroll = 8;
        const u32 ring_from = count > kEmitRing ? count - kEmitRing : 0u;
        for (u32 base = 0; base < count; base += 32 * kUnroll) {
          u8 v[kUnroll];
#pragma unroll
          for (u32 k = 0; k < kUnroll; ++k) {
            const u32 j = base + 32 * k + lane;
            v[k] = j < count ? body[src + j] : u8(0);
          }
#pragma unroll
          for (u32 k = 0; k < kUnroll; ++k) {
            const u32 j = base + 32 * k + lane;
            if (j < count) {
              out[start + pos + j] = v[k];
              if (j >= ring_from) ring[(pos + j) & kEmitMask] = v[k];
            }
          }
        }
        pos += count;
        flushed = pos;
        first += 2;
        __syncwarp();
        continue;
      }
      // The chunk's tokens stop before a stored block: lane i holds tokens
      // first + kLaneTokens i + k, valid up to the first stored one.
      u32 mine = kLaneTokens;
#pragma unroll
      for (u32 k = kLaneTokens; k-- > 0;)
        if ((tk[k] & kStoredFlag) && !(tk[k] & kMatchFlag)) mine = k;
      const u32 stops = __ballot_sync(kFullMask, mine < kLaneTokens);
      const u32 stop_lane = stops ? __ffs(stops) - 1 : 32u;
      const u32 valid = lane < stop_lane ? kLaneTokens : lane == stop_lane ? mine : 0u;
      // Output offsets: the lane's own prefix, then a warp scan.
      u32 size[kLaneTokens], lane_bytes = 0;
#pragma unroll
      for (u32 k = 0; k < kLaneTokens; ++k) {
        size[k] = k >= valid ? 0u : (tk[k] & kMatchFlag) ? (tk[k] & 511u) : 1u;
        lane_bytes += size[k];
      }
      u32 incl = lane_bytes;
#pragma unroll
      for (u32 o = 1; o < 32; o <<= 1) {
        const u32 v = __shfl_up_sync(kFullMask, incl, o);
        if (lane >= o) incl += v;
      }
      // Tokens whose output fits without wrapping onto unflushed entries
      // (a prefix of the chunk: ends only grow).
      const u32 budget = kEmitRing - (pos - flushed);
      u32 at[kLaneTokens], taken = 0, end = incl - lane_bytes, last_end = 0;
#pragma unroll
      for (u32 k = 0; k < kLaneTokens; ++k) {
        at[k] = pos + end;
        end += size[k];
        if (k < valid && end <= budget) {
          taken = k + 1;
          last_end = end;
        }
      }
      const u32 chunk_end = pos + __reduce_max_sync(kFullMask, last_end);
      const u32 m = __reduce_add_sync(kFullMask, taken);
      // The chunk's tokens for the byte pass, copies flagged when they read
      // nothing the chunk writes (their source ends before the chunk, or,
      // overlapping themselves, their period lies before it).
      bool broken = false, outside = false;
#pragma unroll
      for (u32 k = 0; k < kLaneTokens; ++k) {
        if (k >= taken) continue;
        u32 t = tk[k];
        if (t & kMatchFlag) {
          const u32 length = t & 511u, dist = (t >> 9) & 0xffffu;
          if (dist > start + at[k]) broken = true;
          if (length <= dist ? at[k] + length <= pos + dist : at[k] == pos) t |= kOwnFlag;
          else outside = true;
        }
        sh.token[warp][kLaneTokens * lane + k] = t;
        sh.at[warp][kLaneTokens * lane + k] = at[k];
      }
      if (__any_sync(kFullMask, broken)) {
        bad = 1;
        break;
      }
      const bool waits = __any_sync(kFullMask, outside);
      __syncwarp();
      // Symbol of node position dst + j - dist for a copy: a marker before
      // the node start, the ring while the entry is still there (nothing at
      // or past chunk_end is written), else the output.
      auto source_symbol = [&](u32 dst, u32 dist, u32 j) -> u32 {
        if (dist > dst + j) return 256 + (dist - dst - j - 1);
        const u32 q = dst + j - dist;
        if (q + kEmitRing >= chunk_end) return ring[q & kEmitMask];
        return flushed_symbol(out, source, unresolved, start, q);
      };
      // Output-byte parallel pass: lane b takes chunk bytes 32 w + b.  The
      // token covering a byte is the last one starting at or before it: the
      // lanes OR their tokens' start bits of the window into one word, whose
      // popcount below the byte adds to the starts of earlier windows.  A
      // copy that reads the chunk's own output leaves a pending entry,
      // kPending | r, whose r reaches past the copy (a periodic copy points
      // into its seed period).
      const u32 total = chunk_end - pos;
      u32 starts = 0;
      for (u32 w = 0; w * 32 < total; ++w) {
        u32 mine_bits = 0;
#pragma unroll
        for (u32 k = 0; k < kLaneTokens; ++k) {
          const u32 o = at[k] - pos;
          if (k < taken && (o >> 5) == w) mine_bits |= 1u << (o & 31);
        }
        const u32 word = __reduce_or_sync(kFullMask, mine_bits);
        const u32 t = starts + __popc(word & ((2u << lane) - 1u)) - 1;
        starts += __popc(word);
        const u32 b = w * 32 + lane;
        if (b < total) {
          const u32 tw = sh.token[warp][t];
          u32 v;
          if (!(tw & kMatchFlag)) {
            v = tw & 255u;
          } else {
            const u32 t_len = tw & 511u, t_dist = (tw >> 9) & 0xffffu;
            const u32 j = pos + b - sh.at[warp][t];
            if (tw & kOwnFlag) v = source_symbol(pos + b - j, t_dist, t_len <= t_dist ? j : j % t_dist);
            else v = kPending | (t_len <= t_dist ? t_dist : t_dist * (j / t_dist + 1));
          }
          ring[(pos + b) & kEmitMask] = u16(v);
        }
      }
      if (waits) {
        // Pending entries to symbols: each follows its chain, which only
        // steps back and leaves a copy at every step.  An entry another lane
        // resolves at the same time reads as either form; both lead to the
        // same symbol.
        __syncwarp();
        for (u32 b = lane; b < total; b += 32) {
          u32 x = pos + b;
          u32 v = ring[x & kEmitMask];
          if (v < kPending) continue;
          u32 r = v - kPending;
          for (;;) {
            if (r > x) { v = 256 + (r - x - 1); break; }  // before the node start
            const u32 q = x - r;
            if (q + kEmitRing < chunk_end) { v = flushed_symbol(out, source, unresolved, start, q); break; }
            v = ring[q & kEmitMask];
            if (v < kPending) break;
            x = q;
            r = v - kPending;
          }
          ring[(pos + b) & kEmitMask] = u16(v);
        }
      }
      __syncwarp();
      pos = chunk_end;
      first += m;
    }
    if (contiguous || bad) break;
    page = page_next[page];
    }
    if (!bad) flush_symbols(ring, out, source, unresolved, start, flushed, pos);
    __syncwarp();
    if (lane == 0 && (bad || pos != unit_bytes[unit])) atomicOr(fail_flag, 1u);
  }
}

// Resolve unresolved positions by chasing source positions.  Markers come
// in runs (a node's first window reads the node before it), so a warp takes
// 32 bitmap words and resolves the positions of up to four nonzero words at
// once, one lane per bit position, the four chases interleaved so their
// loads overlap.
constexpr u32 kResolveWays = 4;
// Hops a chase may take.  A marker's source lies before its own expansion
// unit, so every hop moves at least one unit back.  Data whose every byte copies
// from the previous record (long runs of records, zero padding) chains each
// marker through every earlier node; such a chase stops here, records the
// position it reached (at least kResolveHops nodes back) in source[], sets
// its bit in `longs` and raises *deep for the staged pass below.
constexpr u32 kResolveHops = 32;
__global__ void resolve_kernel(const u32* state, u32 words, const u32* unresolved, u32* source,
                               u8* out, u32* longs, u32* deep) {
  if (!state[1]) return;
  const u32 lane = threadIdx.x & 31u;
  const u64 warp = (u64(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const u64 warps = (u64(gridDim.x) * blockDim.x) >> 5;
  auto marked = [&](u32 q) { return ((unresolved[q >> 5] >> (q & 31)) & 1u) != 0; };
  for (u64 w0 = warp * 32; w0 < words; w0 += warps * 32) {
    const u32 mine = w0 + lane < words ? unresolved[w0 + lane] : 0u;
    if (w0 + lane < words && !mine) longs[w0 + lane] = 0;
    for (u32 nonzero = __ballot_sync(kFullMask, mine != 0); nonzero;) {
      u32 at[kResolveWays], q[kResolveWays], word[kResolveWays];
      bool live[kResolveWays], has[kResolveWays];
#pragma unroll
      for (u32 k = 0; k < kResolveWays; ++k) {
        const u32 i = nonzero ? __ffs(nonzero) - 1 : 0u;
        const u32 bits = __shfl_sync(kFullMask, mine, i);
        has[k] = nonzero != 0;
        live[k] = has[k] && ((bits >> lane) & 1u);
        nonzero &= nonzero - 1;
        word[k] = u32(w0) + i;
        at[k] = word[k] * 32 + lane;
        q[k] = live[k] ? source[at[k]] : 0u;
      }
      // Sources strictly decrease along a chase, so each ends at a position
      // that emission wrote directly, unless it runs out of hops.
      bool more = true;
      for (u32 hop = 0; more && hop < kResolveHops; ++hop) {
        bool step[kResolveWays];
#pragma unroll
        for (u32 k = 0; k < kResolveWays; ++k) step[k] = live[k] && marked(q[k]);
        more = false;
#pragma unroll
        for (u32 k = 0; k < kResolveWays; ++k) {
          if (step[k]) {
            q[k] = source[q[k]];
            more = true;
          }
        }
      }
      // A chase reading source[] while another warp shortens it follows
      // either value: both are positions of the same chain.
      bool any_long = false;
#pragma unroll
      for (u32 k = 0; k < kResolveWays; ++k) {
        const bool is_long = live[k] && marked(q[k]);
        if (is_long) source[at[k]] = q[k];
        else if (live[k]) out[at[k]] = out[q[k]];
        const u32 ballot = __ballot_sync(kFullMask, is_long);
        if (has[k] && lane == 0) longs[word[k]] = ballot;
        any_long |= ballot != 0;
      }
      if (any_long && lane == 0) atomicOr(deep, 1u);
    }
  }
}

// After resolve_kernel raised *deep: the long markers, in stages of
// kResolveHops consecutive expansion units.  A long marker of unit i reads
// source[] = a position in unit i - kResolveHops or earlier, which is either
// final since resolve_kernel or a long marker of an earlier stage, so the
// markers of one stage resolve in parallel once every earlier stage is done.
// CTAs take (stage, tile) tickets in order; a tile waits for its previous
// stage's kStageTiles tiles.  Every earlier ticket belongs to a running CTA
// that waits only on even earlier ones, so the waits end; each is bounded
// anyway and sets *fail when it gives up.  Output bytes written in this
// kernel are read with L2-coherent loads (ld.global.cg).
constexpr u32 kStageThreads = 256;
constexpr u32 kStageWaitLimit = 1u << 22;  // polls of ~256 ns: about a second
__global__ void __launch_bounds__(kStageThreads)
stage_resolve_kernel(const u32* state, const u32* item_units, const u32* unit_start,
                     u32 expected, const u32* longs, const u32* source, u8* out,
                     u32 tiles_per_stage, u32* stage_done, u32* ticket, u32* fail,
                     const u32* deep) {
  __shared__ u32 s_ticket, s_go;
  if (!state[1] || !*deep) return;
  const u32 len = item_units[state[0]];  // expansion units, in output order
  const u32 stages = (len + kResolveHops - 1) / kResolveHops;
  const u64 total = u64(stages) * tiles_per_stage;
  const bool vec = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  for (;;) {
    if (threadIdx.x == 0) {
      const u32 t = atomicAdd(ticket, 1u);
      u32 go = t < total;
      if (go && t >= tiles_per_stage) {
        const u32* done = stage_done + (t / tiles_per_stage - 1);
        for (u32 polls = 0;; ++polls) {
          if (*reinterpret_cast<volatile const u32*>(done) >= tiles_per_stage) break;
          if (*reinterpret_cast<volatile const u32*>(fail) || polls >= kStageWaitLimit) {
            atomicOr(fail, 1u);
            go = 0;
            break;
          }
          __nanosleep(256);
        }
        __threadfence();
      }
      s_ticket = t;
      s_go = go;
    }
    __syncthreads();
    const u32 t = s_ticket;
    if (!s_go) return;
    const u32 stage = t / tiles_per_stage, tile = t % tiles_per_stage;
    const u32 first = stage * kResolveHops, last = first + kResolveHops;
    const u32 lo = unit_start[first], hi = last < len ? unit_start[last] : expected;
    if (hi > lo) {
      const u32 w_lo = lo >> 5, w_hi = (hi - 1) / 32 + 1;
      const u32 per = (w_hi - w_lo + tiles_per_stage - 1) / tiles_per_stage;
      const u32 a = w_lo + tile * per, b = min_u32(w_hi, a + per);
      for (u32 w = a + threadIdx.x; w < b; w += kStageThreads) {
        u32 bits = longs[w];
        const u32 base = w * 32;
        if (base < lo) bits &= ~0u << (lo - base);
        if (hi - base < 32) bits &= (1u << (hi - base)) - 1u;
        if (!bits) continue;
        if (vec && base + 32 <= expected) {
          // The word's 32 bytes in two 16-byte halves: read, patch the
          // long markers, write back (bytes outside the stage are final or
          // rewritten unchanged; nothing else writes them meanwhile).
          const uint4 h0 = __ldcg(reinterpret_cast<const uint4*>(out + base));
          const uint4 h1 = __ldcg(reinterpret_cast<const uint4*>(out + base + 16));
          u32 v[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
          for (u32 i = 0; i < 32; ++i) {
            if ((bits >> i) & 1u) {
              const u32 byte = __ldcg(reinterpret_cast<const unsigned char*>(out + source[base + i]));
              const u32 shift = 8 * (i & 3);
              v[i >> 2] = (v[i >> 2] & ~(0xffu << shift)) | (byte << shift);
            }
          }
          reinterpret_cast<uint4*>(out + base)[0] = make_uint4(v[0], v[1], v[2], v[3]);
          reinterpret_cast<uint4*>(out + base)[1] = make_uint4(v[4], v[5], v[6], v[7]);
        } else {
          for (u32 m = bits; m; m &= m - 1) {
            const u32 i = __ffs(m) - 1;
            out[base + i] = u8(__ldcg(reinterpret_cast<const unsigned char*>(out + source[base + i])));
          }
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(stage_done + stage, 1u);
    }
  }
}

// Adler-32 partials over 64 KiB segments: (s1, s2 with segment-local weights).
constexpr u32 kAdlerSegment = 65536;

__global__ void adler_parts_kernel(const u32* state, const u8* out, u32 n, u64* parts) {
  if (!state[1]) return;
  __shared__ u64 a1[8], a2[8];
  const u32 seg = blockIdx.x;
  const u32 base = seg * kAdlerSegment;
  const u32 len = min_u32(kAdlerSegment, n - base);
  u64 s1 = 0, s2 = 0;
  const bool vec = (reinterpret_cast<uintptr_t>(out + base) & 15u) == 0;
  if (vec) {
    for (u32 p = threadIdx.x * 16; p + 16 <= len; p += blockDim.x * 16) {
      const uint4 v = *reinterpret_cast<const uint4*>(out + base + p);
      const u32 words[4] = {v.x, v.y, v.z, v.w};
      for (u32 k = 0; k < 4; ++k) {
        const u32 w = words[k];
        const u32 b0 = w & 255u, b1 = (w >> 8) & 255u, b2 = (w >> 16) & 255u, b3 = w >> 24;
        const u32 sum = b0 + b1 + b2 + b3;
        const u32 weight = len - p - 4 * k;
        s1 += sum;
        s2 += u64(weight) * sum - (b1 + 2 * b2 + 3 * b3);
      }
    }
    for (u32 p = (len & ~15u) + threadIdx.x; p < len; p += blockDim.x) {
      const u32 x = out[base + p];
      s1 += x;
      s2 += u64(len - p) * x;
    }
  } else {
    for (u32 p = threadIdx.x; p < len; p += blockDim.x) {
      const u32 x = out[base + p];
      s1 += x;
      s2 += u64(len - p) * x;
    }
  }
  for (u32 o = 16; o; o >>= 1) {
    s1 += __shfl_xor_sync(kFullMask, s1, o);
    s2 += __shfl_xor_sync(kFullMask, s2, o);
  }
  if ((threadIdx.x & 31) == 0) { a1[threadIdx.x >> 5] = s1; a2[threadIdx.x >> 5] = s2; }
  __syncthreads();
  if (threadIdx.x == 0) {
    u64 t1 = 0, t2 = 0;
    for (u32 w = 0; w < blockDim.x / 32; ++w) { t1 += a1[w]; t2 += a2[w]; }
    parts[2 * seg] = t1 % kAdlerMod;
    parts[2 * seg + 1] = t2 % kAdlerMod;
  }
}

// Fast-path verdict into meta[0] (0 or 1), for general_status_kernel.
__global__ void parallel_finish_kernel(const u8* in, u32 in_size, const u32* state,
                                       const u32* fail_flag, const u64* parts, u32 segments,
                                       u32 n, u32 checksum, u32* meta) {
  __shared__ u64 a1[32], a2[32];
  u32 window = 0, wanted = 0;
  const bool framed = zlib_framing(in, in_size, &window, &wanted) == 0;
  const bool ok = framed && state[1] && !*fail_flag;
  u64 s1 = 0, s2 = 0;
  if (ok && checksum) {
    for (u32 s = threadIdx.x; s < segments; s += blockDim.x) {
      const u32 end = min_u32((s + 1) * kAdlerSegment, n);
      const u64 after = (n - end) % kAdlerMod;
      s1 += parts[2 * s];
      s2 += (parts[2 * s + 1] + parts[2 * s] * after) % kAdlerMod;
    }
    s1 %= kAdlerMod;
    s2 %= kAdlerMod;
  }
  for (u32 o = 16; o; o >>= 1) {
    s1 += __shfl_xor_sync(kFullMask, s1, o);
    s2 += __shfl_xor_sync(kFullMask, s2, o);
  }
  if ((threadIdx.x & 31) == 0) { a1[threadIdx.x >> 5] = s1; a2[threadIdx.x >> 5] = s2; }
  __syncthreads();
  if (threadIdx.x == 0) {
    u64 t1 = 0, t2 = 0;
    for (u32 w = 0; w < blockDim.x / 32; ++w) { t1 += a1[w]; t2 += a2[w]; }
    u32 status = 1;
    if (ok) status = !checksum || adler_finish(t1, t2, n) == wanted ? 0u : u32(kAdlerMismatch);
    meta[0] = status;
    meta[1] = 0;
  }
}

// ---------------------------------------------------------------------------
// Fixed-region seeds.  A fixed-Huffman block has no header to discover, so a
// long run of fixed blocks (a Z_FIXED stream) would be one node decoded by
// one warp.  Instead, every tile of kSeedTileBits body bits gets one thread
// that decodes with the fixed tables from the tile start, through further
// fixed blocks, for kSeedProbeBits bits; if every token is valid, the first
// token start past that is a seed.  Huffman decoding resynchronises within a
// few tokens, so the probe's chain has almost surely joined the true chain
// there when the tile lies inside fixed blocks.  Nothing depends on that: a
// node stops at a seed only if its own (true) chain starts a token exactly
// there, and a seed no true chain reaches is a node no path visits.
// ---------------------------------------------------------------------------
__global__ void seed_probe_kernel(const u8* in, u64 in_size, const Tables* fixed, u32 tiles,
                                  u32* raw) {
  const u32 k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= tiles) return;
  u32 seed = ~0u;
  if (k > 0 && in_size >= 8) {
    const u8* body = in + 2;
    const u64 bytes = in_size - 6;
    const u64 start = u64(k) * kSeedTileBits, goal = start + kSeedProbeBits;
    if (goal + 64 < bytes * 8) {
      BitCursor c;
      c.init(body, bytes, start);
      bool valid = true;
      while (valid && c.pos < goal) {
        const Token tok = decode_token(c, *fixed);
        if (tok.kind == kTokError) {
          valid = false;
          break;
        }
        c.skip(tok.bits);
        if (tok.kind == kTokEnd) {  // the next block must be fixed-Huffman too
          u32 err = 0;
          c.take(1, &err);
          const u32 type = c.take(2, &err);
          valid = !err && type == 1;
        }
      }
      if (valid && c.pos >= goal && c.pos < bytes * 8) seed = u32(c.pos);
    }
  }
  raw[k] = seed;
}

// Sorted seeds from the per-tile probe results (one CTA).
__global__ void __launch_bounds__(1024)
seed_compact_kernel(const u32* raw, u32 tiles, u32* seeds, u32* total) {
  __shared__ u32 warp_sum[32];
  const u32 per = (tiles + blockDim.x - 1) / blockDim.x;
  const u32 first = min_u32(threadIdx.x * per, tiles), last = min_u32(first + per, tiles);
  u32 count = 0;
  for (u32 k = first; k < last; ++k) count += raw[k] != ~0u ? 1u : 0u;
  u32 incl = count;
  for (u32 o = 1; o < 32; o <<= 1) {
    const u32 v = __shfl_up_sync(kFullMask, incl, o);
    if ((threadIdx.x & 31) >= o) incl += v;
  }
  if ((threadIdx.x & 31) == 31) warp_sum[threadIdx.x >> 5] = incl;
  __syncthreads();
  if (threadIdx.x < 32) {
    u32 w = threadIdx.x < blockDim.x / 32 ? warp_sum[threadIdx.x] : 0u;
    for (u32 o = 1; o < 32; o <<= 1) {
      const u32 v = __shfl_up_sync(kFullMask, w, o);
      if (threadIdx.x >= o) w += v;
    }
    warp_sum[threadIdx.x] = w;
  }
  __syncthreads();
  const u32 warp = threadIdx.x >> 5;
  u32 at = (warp ? warp_sum[warp - 1] : 0u) + incl - count;
  for (u32 k = first; k < last; ++k)
    if (raw[k] != ~0u) seeds[at++] = raw[k];
  if (threadIdx.x == blockDim.x - 1) *total = at;
}

// The fixed Huffman tables, built once per device into global memory.
__global__ void build_fixed_kernel(Tables* fixed) { warp_build_fixed(*fixed); }

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

cudaError_t build_fixed_tables(void** out) {
  Tables* fixed = nullptr;
  cudaError_t e = cudaMalloc(&fixed, sizeof(Tables));
  if (e != cudaSuccess) return e;
  note_launch();
  build_fixed_kernel<<<1, 32>>>(fixed);
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  *out = fixed;
  return cudaSuccess;
}

cudaError_t configure_parallel_inflate(int* emit_per_sm) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(emit_per_sm, expand_kernel,
                                                       kExpandWarps * 32, 0);
}

u32 chain_levels(u32 capacity) {
  u32 levels = 1;
  while ((1ull << (levels - 1)) < u64(capacity) + 2) ++levels;
  return levels;
}

ParallelScratch parallel_scratch_layout(u64 in_size, u64 expected, u32 capacity,
                                        u64 arena_slack) {
  ParallelScratch s{};
  const u64 body = in_size - 6;
  s.bitmap_words = (body * 8 + 31) / 32 + 1;
  s.compact_blocks = u32((s.bitmap_words + kCompactWords - 1) / kCompactWords);
  // Candidates: the reference rule's (at most `capacity`, else the stream
  // fails as the reference's does) plus the stored-run seeds, at most one per
  // 1029 body bytes (each ends a stored block of at least 1024 bytes).
  s.capacity = capacity + u32(body / 1024) + 64;
  s.tiles = u32((body * 8 + kSeedTileBits - 1) / kSeedTileBits);
  s.node_capacity = s.capacity + 2 * s.tiles;
  s.levels = chain_levels(s.node_capacity);
  s.out_words = (expected + 31) / 32 + 1;
  // Units: at most one per node plus one per kUnitBytes of output.
  s.max_units = u32(expected / kUnitBytes) + s.node_capacity + 2;
  s.stages = (s.max_units + kResolveHops - 1) / kResolveHops + 1;
  s.segments = u32((expected + kAdlerSegment - 1) / kAdlerSegment);
  // Path tokens of a chain that passes its checks: at most one per output
  // byte, plus two words per stored block (at most kMaxBlocks blocks).
  s.symbol_words = expected + 2 * u64(kMaxBlocks) + 64;
  // The page arena holds every candidate's tokens before the path is known:
  // the path's words plus `arena_slack` words for partial last pages and the
  // few tokens false candidates decode.  It also serves as the contiguous
  // layout, so it is never smaller than that.
  s.pages = u32((s.symbol_words + arena_slack + kPageWords - 1) / kPageWords);
  return s;
}

// CTAs of describe_kernel and symbols_kernel, and the stash their warps use.
static u32 node_ctas(const DeviceInfo& dev) { return u32(dev.sms) * 4; }
u64 round_stash_words(const DeviceInfo& dev) {
  return u64(node_ctas(dev)) * kNodeWarps * 32 * kStash;
}

cudaError_t launch_parallel_inflate(const u8* in, u64 in_size, u8* out, u64 expected,
                                    u32 max_blocks, const ParallelScratch& s,
                                    const ParallelBuffers& b, u32* meta, const DeviceInfo& dev,
                                    cudaStream_t stream, bool checksum) {
  const Tables* fixed = static_cast<const Tables*>(dev.fixed_tables);
  note_launch();
  seed_probe_kernel<<<(s.tiles + 255) / 256, 256, 0, stream>>>(in, in_size, fixed, s.tiles,
                                                               b.seed_raw);
  note_launch();
  seed_compact_kernel<<<1, 1024, 0, stream>>>(b.seed_raw, s.tiles, b.seeds, b.seed_total);
  note_launch();
  cand_count_kernel<<<s.compact_blocks, 256, 0, stream>>>(b.bitmap, b.extra,
                                                          u32(s.bitmap_words), b.block_counts);
  note_launch();
  cand_scan_kernel<<<1, 1024, 0, stream>>>(b.block_counts, s.compact_blocks, b.total);
  note_launch();
  cand_write_kernel<<<s.compact_blocks, 256, 0, stream>>>(b.bitmap, b.extra, u32(s.bitmap_words),
                                                          b.block_counts, b.cands, s.capacity);
  // Nodes stop at any candidate header: the reference rule's and the
  // stored-run seeds (b.extra holds their union after the OR kernel).
  note_launch();
  bitmap_or_kernel<<<u32(dev.sms) * 4, 256, 0, stream>>>(b.bitmap, b.extra,
                                                         u32(s.bitmap_words));
  const u32 node_grid = node_ctas(dev);
  profile_begin("describe_kernel", stream);
  note_launch();
  describe_kernel<<<node_grid, kNodeWarps * 32, 0, stream>>>(
      in, u32(in_size), expected, b.cands, b.total, s.capacity, b.seeds, b.seed_total, s.tiles,
      b.extra, b.counters, b.ends, b.sizes, b.blocks, b.infos, b.tokens, b.first_page, b.syms,
      b.page_next, b.page_used, b.page_cursor, s.pages, fixed, b.stash);
  profile_end(stream);
  note_launch();
  chain_kernel<<<1, 1024, 0, stream>>>(in, u32(in_size), expected, max_blocks, b.cands, b.total,
                                       s.capacity, b.seeds, b.seed_total, s.tiles, b.ends,
                                       b.sizes, b.blocks, b.infos, b.tokens, b.jump, s.levels,
                                       b.path, b.prefix, b.tprefix, b.state);
  profile_begin("symbols_kernel", stream);
  note_launch();
  symbols_kernel<<<node_grid, kNodeWarps * 32, 0, stream>>>(
      in, u32(in_size), expected, b.cands, b.total, s.capacity, b.seeds, b.seed_total, s.tiles,
      b.extra, b.path, b.tprefix, b.sizes, b.tokens, b.state, b.counters + 1, b.syms, b.fail,
      fixed, b.stash);
  profile_end(stream);
  // Expansion units: count per path node, scan, write.
  const u32 plan_grid = u32(dev.sms) * 8;
  const u32 unit_shift = unit_shift_for(expected, u32(dev.sms));
  note_launch();
  unit_plan_kernel<<<plan_grid, 256, 0, stream>>>(
      b.state, b.path, b.prefix, b.tprefix, b.sizes, b.tokens, b.syms, b.first_page, b.page_next,
      b.page_used, s.pages, unit_shift, b.unit_counts, nullptr, nullptr, nullptr, nullptr,
      nullptr, nullptr, nullptr, b.fail);
  note_launch();
  unit_scan_kernel<<<1, 1024, 0, stream>>>(b.state, b.unit_counts, b.item_units);
  note_launch();
  unit_plan_kernel<<<plan_grid, 256, 0, stream>>>(
      b.state, b.path, b.prefix, b.tprefix, b.sizes, b.tokens, b.syms, b.first_page, b.page_next,
      b.page_used, s.pages, unit_shift, b.unit_counts, b.item_units, b.unit_item, b.unit_page,
      b.unit_first, b.unit_tokens, b.unit_start, b.unit_bytes, b.fail);
  const u32 expand_grid = u32(dev.sms) * u32(dev.emit_per_sm > 0 ? dev.emit_per_sm : 1);
  profile_begin("expand_kernel", stream);
  note_launch();
  expand_kernel<<<expand_grid, kExpandWarps * 32, 0, stream>>>(
      in, u32(in_size), b.tprefix, b.state, b.syms, b.page_next, b.page_used, s.pages,
      b.item_units, b.unit_item, b.unit_page, b.unit_first, b.unit_tokens, b.unit_start,
      b.unit_bytes, b.counters + 2, out, b.source, b.unresolved, b.fail);
  profile_end(stream);
  profile_begin("resolve_kernel", stream);
  note_launch();
  resolve_kernel<<<u32(dev.sms) * 8, 256, 0, stream>>>(b.state, u32(s.out_words), b.unresolved,
                                                       b.source, out, b.longs, b.deep);
  profile_end(stream);
  profile_begin("stage_resolve_kernel", stream);
  note_launch();
  stage_resolve_kernel<<<u32(dev.sms) * 2, kStageThreads, 0, stream>>>(
      b.state, b.item_units, b.unit_start, u32(expected), b.longs, b.source, out,
      u32(dev.sms) * 2, b.stage_done, b.stage_done + s.stages, b.fail, b.deep);
  profile_end(stream);
  if (s.segments && checksum) {
    note_launch();
    adler_parts_kernel<<<s.segments, 256, 0, stream>>>(b.state, out, u32(expected), b.parts);
  }
  note_launch();
  parallel_finish_kernel<<<1, 1024, 0, stream>>>(in, u32(in_size), b.state, b.fail, b.parts,
                                                 s.segments, u32(expected), checksum ? 1u : 0u,
                                                 meta);
  return cudaGetLastError();
}

}  // namespace cz
