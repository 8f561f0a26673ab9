// Chunk-parallel Deflate encoder, byte-identical to the reference encoder.
//
// The reference (encode_chunk, src/cuda_zlib/_encode_kernels.py:283-400)
// parses each chunk greedily with a one-candidate hash table in which every
// position is inserted in order.  The candidate of position p is therefore a
// pure function of the data: the last earlier position q with the same 13-bit
// hash (enc_hash, :47-51).  This kernel exploits that:
//
//   1. stage the chunk in shared memory and fuse its Adler-32 partial sums;
//   2. every position's candidate: rounds of 4096 positions are sorted into
//      per-warp lists by hash mod 16; each warp takes its list in order and
//      finds equal hashes 32 at a time with a warp match;
//   3. 256 threads each walk the greedy parse from the start of their own
//      segment of the chunk, speculatively;
//   4. one thread stitches the segments: an entry point that differs from the
//      speculative start is re-walked until it meets the speculative chain,
//      which greedy parsing does within a token or two;
//   5. all threads build the literal/length and distance histograms;
//   6. the trees follow enc_tree (:65-157) exactly: the reference pops its
//      heap by (weight, node id); a two-queue merge over leaves sorted by
//      (weight, id) and internal nodes in creation order picks the same pair
//      at every step, so depths, flattening retries and codes are identical;
//   7. the exact stored/fixed/dynamic extents (:312-356) choose the block;
//   8. a block-wide prefix sum over per-segment bit counts places every
//      token, and threads pack their segments into 32-bit words in parallel
//      (word edges shared with a neighbour use atomicOr).
//
// A nonfinal chunk ends with an empty stored block so chunks concatenate
// byte-aligned (:384-388).  Finish kernels scan the chunk sizes on the device
// (no host round trip, unlike CompressionPrefix + ReadWords, codec_ffi.cu:
// 362-390,590-595), combine the Adler partials and pack the slots.
#include <mutex>

#include "kernels.h"
#include "common.cuh"
#include "../../include/cuda_zlib_b200.h"

namespace cz {

constexpr u32 kEncThreads = 512;
constexpr u32 kEncWarps = kEncThreads / 32;
constexpr u32 kOwnerBits = 4;  // log2(kEncWarps): hash slots are split over the warps
static_assert((1u << kOwnerBits) == kEncWarps, "one slot class per warp");
constexpr u32 kSortKeys = 512;  // bitonic sort width of the leaf ranking (>= 286)
static_assert(kSortKeys == kEncThreads, "one sort key per thread");
constexpr u32 kCodeWarps = (286 + 31) / 32;  // warps covering the largest alphabet
constexpr u32 kSerialMergeLeaves = 96;  // at most this many leaves: one-thread merge
// Candidate rounds: consecutive positions per thread (fewer for u32
// positions, whose round list would not fit the static shared limit).  The
// round list shares its shared memory with the arrays of the later phases.
template <typename Pos>
__host__ __device__ constexpr u32 per_thread() { return sizeof(Pos) == 2 ? 32u : 16u; }
constexpr u32 kHashSlots = 8192;
constexpr u32 kStitchRounds = 8;  // parallel stitch rounds before the serial finish
constexpr u32 kStoredMax = 65535;  // bytes of one stored block
constexpr u32 kMaxChunkBytes = 262144;  // largest accepted chunk
// Opt-in level 2 (EncodeSpill::dist set; no reference counterpart): the
// longest of a position's first kChainDepth hash-chain candidates within the
// window, length-3 matches farther than kTooFar dropped, and one-step lazy
// evaluation below kLazyLength.  oracle/zlib_oracle.c restates the same parse.
constexpr u32 kChainDepth = 32;
constexpr u32 kLazyLength = 32;
constexpr u32 kTooFar = 4096;

// Extra bits of a length or distance code (RFC 1951 section 3.2.5), by
// arithmetic rather than table lookups: the lanes of a warp look up different
// codes, which a __constant__ table would serialize.  Length symbols 8..27
// carry (symbol - 4) / 4 extra bits and distance symbols 4..29 carry
// (symbol - 2) / 2; the extra value is the low bits of (length - 3) or
// (distance - 1), whose high bits the symbol itself encodes.
__device__ __forceinline__ u32 length_extra_bits(u32 li) {
  return (li >= 8 && li < 28) ? (li - 4) >> 2 : 0u;
}
__device__ __forceinline__ u32 dist_extra_bits(u32 di) { return di >= 4 ? (di - 2) >> 1 : 0u; }
__device__ __forceinline__ u32 low_bits(u32 x, u32 n) { return x & ((1u << n) - 1u); }
__constant__ u8 kClOrder[19] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};

__device__ __forceinline__ u32 length_symbol(u32 len) {  // index 0..28 for 3..258
  if (len == 258) return 28;
  if (len <= 10) return len - 3;
  const u32 x = len - 3, b = 31 - __clz(x);
  return 4 * (b - 1) + ((x >> (b - 2)) & 3u);
}
__device__ __forceinline__ u32 dist_symbol(u32 dist) {  // index 0..29 for 1..32768
  if (dist <= 4) return dist - 1;
  const u32 x = dist - 1, b = 31 - __clz(x);
  return 2 * b + ((x >> (b - 1)) & 1u);
}
__device__ __forceinline__ u32 reverse_bits(u32 x, u32 n) { return n ? __brev(x) >> (32 - n) : 0; }
__device__ __forceinline__ u32 fixed_ll_len(u32 s) {
  return s <= 143 ? 8u : s <= 255 ? 9u : s <= 279 ? 7u : 8u;
}
__device__ __forceinline__ u32 fixed_ll_code(u32 s) {  // bit-reversed, ready to put
  u32 code;
  if (s <= 143) code = 0x30u + s;
  else if (s <= 255) code = 0x190u + s - 144u;
  else if (s <= 279) code = s - 256u;
  else code = 0xc0u + s - 280u;
  return reverse_bits(code, fixed_ll_len(s));
}
__device__ __forceinline__ u32 extent_of(u32 bits, bool final) {
  return final ? (bits + 7) / 8 : (bits + 3 + 7) / 8 + 4;
}
// Words of a chunk's member and match bitmaps, padded to 16 bytes so that the
// arrays after them (hash table, candidates) start 16-byte aligned.
__host__ __device__ __forceinline__ u32 bitmap_words(u32 chunk_bytes) {
  return ((chunk_bytes + 31) / 32 + 1 + 3) & ~3u;
}
// Stored blocks of an n-byte chunk's stored fallback (kStoredMax each).
__host__ __device__ __forceinline__ u32 stored_blocks(u32 n) {
  return n ? (n + kStoredMax - 1) / kStoredMax : 1u;
}

// Shared state of one chunk (beyond the dynamically sized arrays).  Pos
// holds a chunk position: u16 for chunks within the reference's 65535-byte
// bound, u32 for the larger chunks this codec also accepts.
template <typename Pos>
struct EncodeShared {
  u32 freq[335];        // 0..285 lit/len, 286..315 dist, 316..334 code-length
  u16 owner_count[kEncWarps][kEncWarps];   // per warp, per owner
  u16 owner_before[kEncWarps][kEncWarps];  // per warp, per owner: earlier warps' count
  u16 owner_total[kEncWarps], owner_start[kEncWarps];
  union {
    Pos round_list[kEncThreads * per_thread<Pos>()];  // candidate round: positions by owner
    struct {  // the phases after the candidates
      u8 lengths[336];
      u16 codes[336];
      u32 weight[576];
      u16 parent[576];
      u16 ancestor[2][576];
      u16 sorted[288];
      u32 leafw[288];      // weights in leaf rank order
      u32 sort_keys[kSortKeys];  // leaf ranking: (weight << 9 | id) keys
      u32 sort_swap[kSortKeys];  // the ranking's second exchange buffer
      u16 warp_len[kCodeWarps][16];  // codes: per warp, symbols of each length
      u8 depth[2][576];
      u8 rle_sym[320];
      u8 rle_extra[320];
      u32 seg_exit[kEncThreads];
      u32 seg_entry[kEncThreads];
      u32 seg_bits[kEncThreads];
      u32 sym_code[316];  // packing: code | length << 16 per symbol
    };
  };
  u32 warp_sums[kEncWarps];
  u32 rle_sums[kEncWarps];
  u64 adler_s1[kEncWarps];
  u64 adler_s2[kEncWarps];
  u32 extra_bits, token_count, dist_tokens;
  u32 mode, extent, status, ok, nll, ndist, ncl, rle_size, header_bits, leaves, only;
  u32 more, lcount[16], fixed_sum, ll_sum, tree_ok;
};

// Two-queue merge of m ranked leaves (s.sorted / s.leafw) on one thread:
// inner node k (id alphabet + k) gets its weight in s.weight and its
// children's s.parent.  Leaf ids are below every inner id, so equal weights
// take the leaf.  The head of each queue and the element after it stay in
// registers, so a pick compares registers and the shared-memory load it
// starts is needed only a pick later.
template <typename Shared>
__device__ void serial_merge(Shared& s, u32 alphabet, u32 m) {
  u32 leaf = 0, inner = alphabet, next = alphabet;
  u32 leaf_id = s.sorted[0], leaf_w = s.leafw[0];
  u32 leaf2_id = m > 1 ? u32(s.sorted[1]) : 0u, leaf2_w = m > 1 ? s.leafw[1] : 0u;
  u32 inner_w = 0, inner2_w = 0;  // nodes `inner` and `inner + 1`, when they exist
  for (u32 step = 0; step + 1 < m; ++step) {
    u32 pick[2], picked_w[2];
#pragma unroll
    for (u32 k = 0; k < 2; ++k) {
      const bool take_leaf = leaf < m && (inner == next || leaf_w <= inner_w);
      if (take_leaf) {
        pick[k] = leaf_id;
        picked_w[k] = leaf_w;
        ++leaf;
        leaf_id = leaf2_id;
        leaf_w = leaf2_w;
        if (leaf + 1 < m) { leaf2_id = s.sorted[leaf + 1]; leaf2_w = s.leafw[leaf + 1]; }
      } else {
        pick[k] = inner;
        picked_w[k] = inner_w;
        ++inner;
        inner_w = inner2_w;
        if (inner + 1 < next) inner2_w = s.weight[inner + 1];
      }
    }
    const u32 w = picked_w[0] + picked_w[1];
    s.weight[next] = w;
    s.parent[pick[0]] = u16(next);
    s.parent[pick[1]] = u16(next);
    if (inner == next) inner_w = w;             // the queue was empty
    else if (inner + 1 == next) inner2_w = w;   // it follows the head
    ++next;
  }
}

// The same build for an alphabet of at most 32 symbols (distances, code
// lengths) inside one warp, one symbol a lane: ballots count and place the
// leaves, a shuffle bitonic sort ranks them, lane 0 merges, and depths and
// canonical codes follow without block barriers.  The calling warp only;
// returns on its lanes whether a tree within `limit` was found.
template <typename Shared>
__device__ bool warp_tree(Shared& s, const u32* freq, u32 alphabet, u32 limit, u8* lengths,
                          u16* codes) {
  const u32 lane = threadIdx.x & 31u;
  const bool symbol = lane < alphabet;
  const u32 f = symbol ? freq[lane] : 0u;
  for (u32 shift = 0; shift <= 16; ++shift) {
    u32 w = f ? ((f + (1u << shift) - 1u) >> shift) : 0u;
    const u32 present = __ballot_sync(kFullMask, w != 0);
    u32 m = __popc(present), only = present ? 31 - __clz(present) : 0u;
    // The reference's dummy leaves for empty and one-symbol alphabets.
    if (!m) {
      if (lane == 0) w = 1;
      m = 1;
      only = 0;
    }
    if (m == 1) {
      if (lane == (only ? 0u : 1u)) w = 1;
      m = 2;
    }
    if (symbol) s.weight[lane] = w;
    u32 key = w ? (w << 9) | lane : ~0u;
    for (u32 k = 2; k <= 32; k <<= 1) {
      for (u32 j = k >> 1; j; j >>= 1) {
        const u32 other = __shfl_xor_sync(kFullMask, key, j);
        key = (((lane & j) == 0) == ((lane & k) == 0)) ? min_u32(key, other) : max_u32(key, other);
      }
    }
    if (lane < m) {
      s.sorted[lane] = u16(key & 511u);
      s.leafw[lane] = key >> 9;
    }
    __syncwarp();
    if (lane == 0) serial_merge(s, alphabet, m);
    __syncwarp();
    // Depths by pointer doubling over the alphabet + m - 1 <= 63 nodes.
    const u32 nodes = alphabet + m - 1, root = nodes - 1;
    for (u32 i = lane; i < nodes; i += 32) {
      const bool live = i >= alphabet || s.weight[i];
      const bool top = i == root || !live;
      s.ancestor[0][i] = u16(top ? root : s.parent[i]);
      s.depth[0][i] = top ? 0 : 1;
    }
    u32 cur = 0;
    for (;;) {
      __syncwarp();
      bool moved = false;
      for (u32 i = lane; i < nodes; i += 32) {
        const u32 up = s.ancestor[cur][i];
        s.depth[cur ^ 1][i] = u8(s.depth[cur][i] + (up == root ? 0u : s.depth[cur][up]));
        s.ancestor[cur ^ 1][i] = up == root ? u16(root) : s.ancestor[cur][up];
        moved |= up != root;
      }
      cur ^= 1;
      if (!__any_sync(kFullMask, moved)) break;
    }
    __syncwarp();
    const u32 d = w ? u32(s.depth[cur][lane]) : 0u;
    const bool overlong = __any_sync(kFullMask, d > limit);
    // Canonical codes: the first code of each length from the ballot counts,
    // plus the rank among the lower symbols of the same length.
    u32 code = 0, first = 0;
    for (u32 len = 1; len <= 15; ++len) {
      code = (code + __popc(__ballot_sync(kFullMask, d == len - 1 && len > 1))) << 1;
      if (len == d) first = code;
    }
    const u32 rank = __popc(__match_any_sync(kFullMask, d) & ((1u << lane) - 1u));
    if (symbol) {
      lengths[lane] = d <= limit ? u8(d) : 0;
      codes[lane] = overlong || !d ? 0 : u16(reverse_bits(first + rank, d));
    }
    __syncwarp();
    if (!overlong) return true;
  }
  return false;
}

// Huffman build with the reference's (weight, id) order and flattening
// retries, spread over the block.  The reference pops its heap by (weight,
// node id); with leaves ranked by (weight, id) and inner nodes queued in
// creation order (their weights never decrease), a two-queue merge that takes
// the leaf on equal weights picks the same pair at every step.  That merge
// runs in rounds: with t the weight of the next node (the sum of the next two
// picks), every node created from then on weighs at least t, so all queued
// leaves and inner nodes of weight <= t are picked before any of them, in the
// order of a stable merge of the two queues.  A round merges those in
// parallel (an odd last one waits for the next round) and pairs them into new
// nodes; t at least doubles every two rounds.  Depths follow by pointer
// doubling, codes by per-warp ranks.  For the literal/length alphabet (more
// than 32 symbols); all threads call; returns on all threads whether a tree
// within `limit` was found.
template <typename Shared>
__device__ bool cta_tree(Shared& s, const u32* freq, u32 alphabet, u32 limit, u8* lengths,
                         u16* codes) {
  const u32 tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  for (u32 shift = 0; shift <= 16; ++shift) {
    if (tid == 0) { s.leaves = 0; s.only = 0; }
    if (tid < 16) s.lcount[tid] = 0;
    if (tid < kCodeWarps * 16) (&s.warp_len[0][0])[tid] = 0;
    __syncthreads();
    for (u32 i = tid; i < alphabet; i += kEncThreads) {
      lengths[i] = 0;
      codes[i] = 0;
      const u32 w = freq[i] ? ((freq[i] + (1u << shift) - 1u) >> shift) : 0u;
      s.weight[i] = w;
      if (w) {
        atomicAdd(&s.leaves, 1u);
        atomicMax(&s.only, i);
      }
    }
    __syncthreads();
    if (tid == 0) {
      // The reference's dummy leaves for empty and one-symbol alphabets (a
      // complete tree is always produced).
      u32 m = s.leaves, only = s.only;
      if (!m) { s.weight[0] = 1; m = 1; only = 0; }
      if (m == 1) {
        s.weight[only ? 0u : 1u] = 1;
        m = 2;
      }
      s.leaves = m;
    }
    __syncthreads();
    // Rank leaves by (weight, id): a bitonic sort of (weight << 9 | id) keys,
    // zero weights last (weights stay below 2^19, ids below 2^9), one key per
    // thread.  Partners within a warp are exchanged by shuffles; farther ones
    // through two shared buffers used in turn, one barrier a stage.
    {
      const u32 w = tid < alphabet ? s.weight[tid] : 0u;
      u32 key = w ? (w << 9) | tid : ~0u;
      bool flip = false;
      for (u32 k = 2; k <= kSortKeys; k <<= 1) {
        for (u32 j = k >> 1; j; j >>= 1) {
          u32 other;
          if (j >= 32) {
            u32* buf = flip ? s.sort_swap : s.sort_keys;
            buf[tid] = key;
            __syncthreads();
            other = buf[tid ^ j];
            flip = !flip;
          } else {
            other = __shfl_xor_sync(kFullMask, key, j);
          }
          key = (((tid & j) == 0) == ((tid & k) == 0)) ? min_u32(key, other) : max_u32(key, other);
        }
      }
      if (tid < s.leaves) {
        s.sorted[tid] = u16(key & 511u);
        s.leafw[tid] = key >> 9;
      }
    }
    __syncthreads();
    const u32 m = s.leaves;
    const u32 nodes = alphabet + m - 1;  // leaves' ids stay below alphabet
    if (m <= kSerialMergeLeaves) {
      // Few leaves: one thread's merge costs less than the rounds' barriers.
      if (tid == 0) serial_merge(s, alphabet, m);
      __syncthreads();
    } else {
      const u32* leafw = s.leafw;
      u32* inner_w = s.weight + alphabet;  // inner node k has id alphabet + k
      u16* merged = s.ancestor[0];         // a round's picks, in order
      u32* merged_w = s.sort_keys;
      // First index in [lo, hi) whose weight is above (upper) or at least
      // (lower) w.
      auto upper = [](const u32* v, u32 lo, u32 hi, u32 w) {
        while (lo < hi) {
          const u32 mid = (lo + hi) >> 1;
          if (v[mid] <= w) lo = mid + 1;
          else hi = mid;
        }
        return lo;
      };
      auto lower = [](const u32* v, u32 lo, u32 hi, u32 w) {
        while (lo < hi) {
          const u32 mid = (lo + hi) >> 1;
          if (v[mid] < w) lo = mid + 1;
          else hi = mid;
        }
        return lo;
      };
      u32 a = 0, b = 0, c = 0;  // next leaf, next queued inner node, inner nodes made
      while ((m - a) + (c - b) > 1) {
        u32 la = a, ib = b, t = 0;
#pragma unroll
        for (u32 k = 0; k < 2; ++k) {
          const bool leaf = la < m && (ib == c || leafw[la] <= inner_w[ib]);
          t += leaf ? leafw[la++] : inner_w[ib++];
        }
        u32 nl = upper(leafw, a, m, t) - a, ni = upper(inner_w, b, c, t) - b;
        if ((nl + ni) & 1u) {
          if (ni && (!nl || inner_w[b + ni - 1] >= leafw[a + nl - 1])) --ni;
          else --nl;
        }
        for (u32 i = tid; i < nl + ni; i += kEncThreads) {
          u32 pos, id, w;
          if (i < nl) {
            w = leafw[a + i];
            pos = i + lower(inner_w, b, b + ni, w) - b;
            id = s.sorted[a + i];
          } else {
            const u32 j = i - nl;
            w = inner_w[b + j];
            pos = j + upper(leafw, a, a + nl, w) - a;
            id = alphabet + b + j;
          }
          merged[pos] = u16(id);
          merged_w[pos] = w;
        }
        __syncthreads();
        const u32 pairs = (nl + ni) >> 1;
        for (u32 k = tid; k < pairs; k += kEncThreads) {
          inner_w[c + k] = merged_w[2 * k] + merged_w[2 * k + 1];
          s.parent[merged[2 * k]] = u16(alphabet + c + k);
          s.parent[merged[2 * k + 1]] = u16(alphabet + c + k);
        }
        __syncthreads();
        a += nl;
        b += ni;
        c += pairs;
      }
    }
    // Depth of every node by pointer doubling towards the root.
    const u32 root = nodes - 1;
    for (u32 i = tid; i < nodes; i += kEncThreads) {
      const bool live = i >= alphabet || s.weight[i];
      const bool top = i == root || !live;
      s.ancestor[0][i] = u16(top ? root : s.parent[i]);
      s.depth[0][i] = top ? 0 : 1;
    }
    u32 cur = 0;
    for (;;) {
      __syncthreads();
      bool moved = false;
      for (u32 i = tid; i < nodes; i += kEncThreads) {
        const u32 up = s.ancestor[cur][i];
        s.depth[cur ^ 1][i] = u8(s.depth[cur][i] + (up == root ? 0u : s.depth[cur][up]));
        s.ancestor[cur ^ 1][i] = up == root ? u16(root) : s.ancestor[cur][up];
        moved |= up != root;
      }
      cur ^= 1;
      if (!__syncthreads_or(moved)) break;
    }
    bool overlong = false;
    for (u32 i = tid; i < alphabet; i += kEncThreads) {
      if (!s.weight[i]) continue;
      const u32 d = s.depth[cur][i];
      if (d > limit) { overlong = true; continue; }
      lengths[i] = u8(d);
      atomicAdd(&s.lcount[d], 1u);
    }
    if (__syncthreads_or(overlong)) continue;
    // Canonical codes: the first code of a symbol's length plus its rank
    // among the lower symbols of that length (within its warp by a match,
    // then the earlier warps' counts of that length).
    const u32 len = tid < alphabet ? lengths[tid] : 0u;
    u32 rank = 0;
    if (warp < kCodeWarps) {
      const u32 same = __match_any_sync(kFullMask, tid < alphabet ? len : 0xffu);
      rank = __popc(same & ((1u << lane) - 1u));
      if (len && !rank) s.warp_len[warp][len] = u16(__popc(same));
    }
    __syncthreads();
    if (len) {
      u32 code = 0;  // lcount[0] is zero: no leaf sits at the root
      for (u32 bit = 1; bit <= len; ++bit) code = (code + s.lcount[bit - 1]) << 1;
      for (u32 w = 0; w < warp; ++w) rank += s.warp_len[w][len];
      codes[tid] = u16(reverse_bits(code + rank, len));
    }
    __syncthreads();
    return true;
  }
  return false;
}

// Append `n` bits of `value` to the packing accumulator; full 32-bit words
// go to `words` (little-endian bit order, LSB first).  Edge words are ORed.
struct Packer {
  u32* words;
  u64 acc;
  u32 nacc;   // bits in acc
  u32 word;   // index of the word acc starts at (a slot holds under 2^16 words)
  u32 first_word, last_word;  // this thread's shared edge words
  u32 limit;  // words past the slot are dropped (the size check then fails)

  __device__ __forceinline__ void start(u32* w, u32 bit, u32 end_bit, u32 limit_words) {
    limit = limit_words;
    words = w;
    word = bit >> 5;
    nacc = bit & 31u;
    acc = 0;
    first_word = word;
    last_word = end_bit ? (end_bit - 1) >> 5 : 0;
  }
  __device__ __forceinline__ void flush_word(u32 v) {
    if (word < limit) {
      if (word == first_word || word == last_word) atomicOr(words + word, v);
      else words[word] = v;
    }
    ++word;
  }
  __device__ __forceinline__ void put(u32 value, u32 n) {
    acc |= u64(value) << nacc;
    nacc += n;
    if (nacc >= 32) {
      flush_word(u32(acc));
      acc >>= 32;
      nacc -= 32;
    }
  }
  __device__ __forceinline__ void finish() {
    if (nacc && word < limit) atomicOr(words + word, u32(acc));
  }
};

// Calls f(p, is_match) for every token start p in [a, b), in order, reading
// the membership and match bitmaps a word at a time.
template <class F>
__device__ __forceinline__ void for_each_token(const u32* member, const u32* ismatch, u32 a,
                                               u32 b, F f) {
  for (u32 lo = a & ~31u; lo < b; lo += 32) {
    u32 bits = member[lo >> 5];
    const u32 matches = ismatch[lo >> 5];
    if (lo < a) bits &= ~0u << (a - lo);
    if (b - lo < 32) bits &= (1u << (b - lo)) - 1u;
    while (bits) {
      const u32 k = __ffs(bits) - 1;
      bits &= bits - 1;
      f(lo + k, ((matches >> k) & 1u) != 0);
    }
  }
}

// Slot of chunk g: starts at 16-aligned (input position + 96 g), so a slot
// holds at least n + 80 bytes and all slots fit in in_bytes + 96 (chunks+1).
__device__ __forceinline__ u64 slot_start(u64 in_pos, u32 g) {
  return ((in_pos + 15) & ~u64(15)) + 96 * u64(g);
}
// Entry of chunk g in the global spill: 16-aligned, kSpillGap entries after
// the previous chunk's, so a chunk's slice holds its padded data (up to
// chunk + 31 bytes) and all slices fit in in_bytes + kSpillGap * (chunks + 2).
__device__ __forceinline__ u64 spill_offset(u64 in_pos, u32 g) {
  return ((in_pos + 15) & ~u64(15)) + kSpillGap * u64(g);
}

// Chunks above 65535 bytes: Pos = u32, and the chunk, its candidates and
// match lengths live in the global spill (256 KiB do not fit shared memory);
// its stored fallback takes several blocks of at most 65535 bytes.
template <typename Pos>
__global__ void __launch_bounds__(kEncThreads, 2)
encode_chunks_kernel(const u8* __restrict__ in, const EncodeFile* __restrict__ files, u32 nfiles,
                     u32 chunk_bytes, u32 total_chunks, u8* slots, u32* sizes, u32* status,
                     u64* adler, EncodeSpill spill, u32 in_smem) {
  constexpr bool kLarge = sizeof(Pos) == 4;
  extern __shared__ __align__(16) u8 smem[];
  __shared__ EncodeShared<Pos> s;
  const u32 tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const u32 g = blockIdx.x;
  if (g >= total_chunks) return;
  // File of this chunk (files are sorted by first_chunk).
  u32 lo = 0, hi = nfiles;
  while (hi - lo > 1) {
    const u32 mid = (lo + hi) >> 1;
    if (files[mid].first_chunk <= g) lo = mid;
    else hi = mid;
  }
  const EncodeFile f = files[lo];
  const u32 local = g - f.first_chunk;
  const u64 start = u64(local) * chunk_bytes;
  const u32 n = u32(min_u64(f.in_size - min_u64(start, f.in_size), chunk_bytes));
  const bool final = local + 1 == f.chunks && !(f.flags & kEncodeNotLast);
  const u8* src = in + f.in_offset + start;

  // Shared layout: data | member bits | match bits | hash table | prev | len
  // (large chunks: member bits | match bits | hash table).
  const u32 data_bytes = (chunk_bytes + 16 + 15) & ~15u;
  const u32 bit_words = bitmap_words(chunk_bytes);
  const u64 spill_at = spill_offset(f.in_offset + start, g);
  u8* data = kLarge ? spill.data + spill_at : smem;
  u32* member = reinterpret_cast<u32*>(kLarge ? smem : smem + data_bytes);
  u32* ismatch = member + bit_words;
  Pos* table = reinterpret_cast<Pos*>(ismatch + bit_words);
  Pos* prev;
  u8* lenv;
  if (in_smem) {
    prev = table + kHashSlots;
    lenv = reinterpret_cast<u8*>(prev + ((chunk_bytes + 7) & ~7u));
  } else {
    // 16-byte aligned (lenv is read as words), kSpillGap entries apart.
    prev = reinterpret_cast<Pos*>(spill.prev) + spill_at;
    lenv = spill.len + spill_at;
  }

  // 1. Stage the chunk (zero padded) and its Adler-32 partial sums.  Reads
  // never go past byte n + 7 (hashing reads the word after a position's
  // own); a spilled chunk pads only to n + 16, the end of its own slice's
  // guaranteed room (a chunk shorter than chunk_bytes is followed closely by
  // the next file's slice).
  u64 s1 = 0, s2 = 0;
  const u32 stage_bytes = kLarge ? min_u32(data_bytes, (n + 16 + 15) & ~15u) : data_bytes;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    // 16 bytes a step; a word's bytes b0..b3 at positions p..p+3 add
    // sum to s1 and (n - p) * sum - (b1 + 2 b2 + 3 b3) to s2 (zeros beyond n
    // add nothing, so the weight may wrap there).
    for (u32 i = 16 * tid; i < stage_bytes; i += 16 * kEncThreads) {
      uint4 q = make_uint4(0, 0, 0, 0);
      if (i + 16 <= n) {
        q = *reinterpret_cast<const uint4*>(src + i);
      } else if (i < n) {
        u64 lo = 0, hi = 0;
        for (u32 b = 0; i + b < n; ++b) {
          if (b < 8) lo |= u64(src[i + b]) << (8 * b);
          else hi |= u64(src[i + b]) << (8 * (b - 8));
        }
        q = make_uint4(u32(lo), u32(lo >> 32), u32(hi), u32(hi >> 32));
      }
      *reinterpret_cast<uint4*>(data + i) = q;
      const u32 words4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (u32 k = 0; k < 4; ++k) {
        const u32 w = words4[k];
        const u32 b0 = w & 255u, b1 = (w >> 8) & 255u, b2 = (w >> 16) & 255u, b3 = w >> 24;
        const u32 sum = b0 + b1 + b2 + b3;
        s1 += sum;
        s2 += u64(n - (i + 4 * k)) * sum - (b1 + 2 * b2 + 3 * b3);
      }
    }
  } else {
    for (u32 i = tid; i < stage_bytes; i += kEncThreads) {
      const u32 x = i < n ? u32(src[i]) : 0u;
      data[i] = u8(x);
      s1 += x;
      s2 += u64(n - i) * x;  // x == 0 beyond n
    }
  }
  for (u32 i = tid; i < bit_words; i += kEncThreads) { member[i] = 0; ismatch[i] = 0; }
  for (u32 i = tid; i < kHashSlots; i += kEncThreads) table[i] = 0;
  for (u32 i = tid; i < 335; i += kEncThreads) s.freq[i] = 0;
  for (u32 o = 16; o; o >>= 1) {
    s1 += __shfl_xor_sync(kFullMask, s1, o);
    s2 += __shfl_xor_sync(kFullMask, s2, o);
  }
  if (lane == 0) { s.adler_s1[warp] = s1; s.adler_s2[warp] = s2; }
  if (tid == 0) {
    s.extra_bits = 0;
    s.token_count = 0;
    s.dist_tokens = 0;
    s.status = 0;
    s.fixed_sum = 0;
    s.ll_sum = 0;
  }
  __syncthreads();
  if (tid == 0) {
    u64 a = 0, b = 0;
    for (u32 w = 0; w < kEncWarps; ++w) { a += s.adler_s1[w]; b += s.adler_s2[w]; }
    adler[2 * u64(g)] = a;
    adler[2 * u64(g) + 1] = b;
  }

  // 2. Candidates: prev[p] = 1 + the last earlier position with hash(p), or
  // 0 (the reference inserts every position into its one-entry table in
  // order, so this is the table's entry when p is reached).  Warp w owns the
  // table slots h with h % 16 == w.  Rounds of 16384 positions (8192 for
  // u32 positions), 32 (16) consecutive ones per thread: the block sorts the round's positions
  // into per-owner lists in position order (counts per owner packed four to
  // a u64 in 16-bit fields, a warp scan, then per-warp and per-owner
  // offsets), and each warp takes its list in batches of 32.  In a batch the
  // lanes hash their positions again from the staged chunk and find equal
  // hashes with one warp match; a lane's candidate is its last
  // earlier equal lane, else the table, and the last lane of each hash writes
  // the table.  Slots are disjoint between warps, so within a round the
  // warps never wait on one another.
  const u32 hashed = n >= 3 ? n - 2 : 0;  // positions 0..n-3 are hashed
  {
    const u32* words = reinterpret_cast<const u32*>(data);
    auto hash_at = [&](u32 p) -> u32 {
      const u32 lo = words[p >> 2], hi = words[(p >> 2) + 1];
      const u32 v = __funnelshift_r(lo, hi, (p & 3u) * 8u) & 0xffffffu;
      return (v * 2654435761u) >> 19;
    };
    Pos* list = s.round_list;
    auto batch = [&](u32 first, u32 count) {
      const bool valid = lane < count;
      const u32 pos = valid ? u32(list[first + lane]) : 0u;
      const u32 h = valid ? hash_at(pos) : 0u;
      const u32 key = h >> kOwnerBits;  // the low bits equal the warp index
      const u32 same = __match_any_sync(kFullMask, valid ? key : ~0u);
      const u32 lower = same & ((1u << lane) - 1u);
      const u32 from = __shfl_sync(kFullMask, pos, lower ? 31 - __clz(lower) : lane);
      u32 candidate = 0;
      if (valid) candidate = lower ? from + 1 : table[h];
      __syncwarp();
      if (valid) {
        if (!(same & ~((2u << lane) - 1u))) table[h] = Pos(pos + 1);
        prev[pos] = Pos(candidate);
      }
      __syncwarp();
    };
    constexpr u32 kPerThread = per_thread<Pos>(), kRoundPositions = kEncThreads * kPerThread;
    for (u32 base = 0; base < hashed; base += kRoundPositions) {
      const u32 p0 = base + kPerThread * tid;
      // Owner o's count in 16-bit field o % 4 of c[o / 4] (no runtime
      // indexing, so the four words stay in registers).  Owners are hashed
      // again for the scatter below rather than kept across the barriers:
      // the thread's positions lie in kPerThread / 4 + 1 aligned words (p0
      // is a multiple of 8), read once a pass, and position p0 + k hashes
      // from them by funnel shifts (a thread wholly past the hashed
      // positions reads nothing).
      constexpr u32 kWords = kPerThread / 4 + 1;
      u32 x[kWords];
      auto load_words = [&]() {
#pragma unroll
        for (u32 i = 0; i < kWords; ++i) x[i] = p0 < hashed ? words[(p0 >> 2) + i] : 0u;
      };
      auto owner_of = [&](u32 p) -> u32 {
        const u32 k = p - p0;  // a constant once the callers' loops unroll
        const u32 v = __funnelshift_r(x[k >> 2], x[(k >> 2) + 1], (k & 3u) * 8u) & 0xffffffu;
        return p < hashed ? ((v * 2654435761u) >> 19) & (kEncWarps - 1) : kEncWarps;
      };
      load_words();
      u64 c0 = 0, c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
      for (u32 k = 0; k < kPerThread; ++k) {
        const u32 o = owner_of(p0 + k);
        const u32 q = o >> 2;
        const u64 one = 1ull << (16 * (o & 3u));
        c0 += q == 0 ? one : 0;
        c1 += q == 1 ? one : 0;
        c2 += q == 2 ? one : 0;
        c3 += q == 3 ? one : 0;
      }
      u64 i0 = c0, i1 = c1, i2 = c2, i3 = c3;
#pragma unroll
      for (u32 o = 1; o < 32; o <<= 1) {
        const u64 v0 = __shfl_up_sync(kFullMask, i0, o), v1 = __shfl_up_sync(kFullMask, i1, o);
        const u64 v2 = __shfl_up_sync(kFullMask, i2, o), v3 = __shfl_up_sync(kFullMask, i3, o);
        if (lane >= o) {
          i0 += v0;
          i1 += v1;
          i2 += v2;
          i3 += v3;
        }
      }
      const u64 incl[4] = {i0, i1, i2, i3};
      if (lane == 31) {
#pragma unroll
        for (u32 o = 0; o < kEncWarps; ++o)
          s.owner_count[warp][o] = u16(incl[o >> 2] >> (16 * (o & 3u)));
      }
      __syncthreads();
      if (warp == 0) {
        // Lane o < 16: owner o's offset before each warp, its total, and the
        // start of its list (owners' lists one after another).
        u32 running = 0;
        if (lane < kEncWarps) {
          for (u32 w = 0; w < kEncWarps; ++w) {
            s.owner_before[w][lane] = u16(running);
            running += s.owner_count[w][lane];
          }
        }
        u32 start = running;
#pragma unroll
        for (u32 o = 1; o < 32; o <<= 1) {
          const u32 v = __shfl_up_sync(kFullMask, start, o);
          if (lane >= o) start += v;
        }
        if (lane < kEncWarps) {
          s.owner_total[lane] = u16(running);
          s.owner_start[lane] = u16(start - running);
        }
      }
      __syncthreads();
      u64 n0 = i0 - c0, n1 = i1 - c1, n2 = i2 - c2, n3 = i3 - c3;  // earlier lanes' counts
      load_words();
#pragma unroll
      for (u32 k = 0; k < kPerThread; ++k) {
        const u32 o = owner_of(p0 + k);
        if (o >= kEncWarps) continue;
        const u32 q = o >> 2, field = 16 * (o & 3u);
        const u64 seen = q == 0 ? n0 : q == 1 ? n1 : q == 2 ? n2 : n3;
        const u32 at = s.owner_start[o] + s.owner_before[warp][o] + u32((seen >> field) & 0xffffu);
        const u64 one = 1ull << field;
        n0 += q == 0 ? one : 0;
        n1 += q == 1 ? one : 0;
        n2 += q == 2 ? one : 0;
        n3 += q == 3 ? one : 0;
        list[at] = Pos(p0 + k);
      }
      __syncthreads();
      const u32 first = s.owner_start[warp], total = s.owner_total[warp];
      for (u32 i = 0; i < total; i += 32) batch(first + i, min_u32(32, total - i));
      __syncthreads();
    }
  }
  __syncthreads();

  // 3. Speculative greedy walks, one segment per thread.
  const u32 seg = (n + kEncThreads - 1) / kEncThreads;
  // Candidates through a register window of the 16 bytes of `prev` around
  // a position: walks move forward through their segment, so one load
  // serves 8 (u16) or 4 (u32) positions instead of one dependent load each.
  // `prev` is 16-byte aligned in every layout.
  constexpr u32 kPerWindow = 16 / sizeof(Pos);
  u32 window_base = ~0u;
  uint4 window = make_uint4(0, 0, 0, 0);
  auto candidate_of = [&](u32 p) -> u32 {
    const u32 base = p & ~(kPerWindow - 1);
    if (base != window_base) {
      window_base = base;
      window = *reinterpret_cast<const uint4*>(prev + base);
    }
    const u32 k = p - base;
    if (kPerWindow == 8) {
      const u32 word = k < 4 ? (k < 2 ? window.x : window.y) : (k < 6 ? window.z : window.w);
      return (k & 1) ? word >> 16 : word & 0xffffu;
    }
    return k < 2 ? (k == 0 ? window.x : window.y) : (k == 2 ? window.z : window.w);
  };
  // Match length of p against q < p, from 3 bytes known equal up to
  // `limit`: four bytes a step from funnel-shifted word loads, the first
  // differing byte from the lowest set bit of their difference.  Reads stay
  // within the staged chunk's zero padding (position + limit + 7 <= n + 7).
  const u32* chunk_words = reinterpret_cast<const u32*>(data);
  auto load4 = [&](u32 x) -> u32 {
    return __funnelshift_r(chunk_words[x >> 2], chunk_words[(x >> 2) + 1], (x & 3u) * 8u);
  };
  auto match_from = [&](u32 q, u32 p, u32 limit) -> u32 {
    u32 m = 3;
    while (m < limit) {
      const u32 diff = load4(q + m) ^ load4(p + m);
      if (diff) {
        m += (__ffs(diff) - 1) >> 3;
        break;
      }
      m += 4;
    }
    return min_u32(m, limit);
  };
  // Level 2: the chain of p runs through prev[] (each entry is 1 + the last
  // earlier position with the same hash).  Comparing the byte at the current
  // best length first skips candidates that cannot be longer.
  u16* distv = spill.dist ? spill.dist + spill_at : nullptr;
  const bool thorough = distv != nullptr;
  u32 token_q = 0;  // level 2: source of the last match token_at returned
  auto chain_best = [&](u32 p, u32* where) -> u32 {
    if (p >= hashed) return 0;
    const u32 limit = min_u32(n - p, 258u);
    u32 best = 0, at = 0, c = prev[p];
    for (u32 step = 0; c && step < kChainDepth; ++step) {
      const u32 q = c - 1;
      if (p - q > 32768u) break;
      if ((best < 3 || data[q + best] == data[p + best]) && data[q] == data[p] &&
          data[q + 1] == data[p + 1] && data[q + 2] == data[p + 2]) {
        const u32 m = match_from(q, p, limit);
        if (m > best) {
          best = m;
          at = q;
          if (m >= limit) break;
        }
      }
      c = prev[q];
    }
    if (best == 3 && p - at > kTooFar) best = 0;
    *where = at;
    return best;
  };
  auto token_at = [&](u32 p) -> u32 {  // match length at p, or 0 for a literal
    if (thorough) {
      const u32 m = chain_best(p, &token_q);
      if (!m || m >= kLazyLength) return m;
      u32 next = 0;
      return chain_best(p + 1, &next) > m ? 0u : m;
    }
    if (p >= hashed) return 0;
    const u32 c = candidate_of(p);
    if (!c) return 0;
    const u32 q = c - 1, dist = p - q;
    if (dist > 32768u || data[q] != data[p] || data[q + 1] != data[p + 1] ||
        data[q + 2] != data[p + 2])
      return 0;
    return match_from(q, p, min_u32(n - p, 258u));
  };
  {
    const u32 a = min_u32(tid * seg, n), b = min_u32(a + seg, n);
    u32 p = a;
    while (p < b) {
      const u32 m = token_at(p);
      atomicOr(&member[p >> 5], 1u << (p & 31));
      if (m) {
        atomicOr(&ismatch[p >> 5], 1u << (p & 31));
        lenv[p] = u8(m - 3);
        if (thorough) distv[p] = u16(p - token_q);
        p += m;
      } else {
        ++p;
      }
    }
    s.seg_exit[tid] = p;
  }
  __syncthreads();

  // 4. Stitch.  The true entry of a segment is the first token boundary at
  // or after its start on the chain from position 0.  A walk from a wrong
  // start usually lands on the segment's speculative chain within a token or
  // two, and from there follows it to the speculative exit.  So the entries
  // are found in parallel rounds: every segment whose entry changed walks
  // from it until it lands on one of its speculative token starts (its exit
  // is then the speculative exit) or passes its end (its exit is where the
  // walk stopped); then each entry becomes the previous segment's exit.
  // Round r makes the first r segments exact; the rounds stop when no entry
  // changes, normally after two (data whose chains take longer to re-join,
  // such as long byte runs, take a few more), and every segment applies its
  // re-walk in parallel.
  auto is_member = [&](u32 p) { return ((member[p >> 5] >> (p & 31)) & 1u) != 0; };
  auto clear_members = [&](u32 from, u32 to) {  // member bits of [from, to)
    while (from < to) {
      const u32 word = from >> 5, lo = from & 31u;
      const u32 hi = min_u32(to - (from & ~31u), 32u);
      const u32 mask = (hi == 32 ? ~0u : ((1u << hi) - 1u)) & ~((1u << lo) - 1u);
      atomicAnd(&member[word], ~mask);
      from = (from & ~31u) + hi;
    }
  };
  const u32 nseg = seg ? (n + seg - 1) / seg : 0;
  const u32 my_a = min_u32(tid * seg, n), my_b = min_u32(my_a + seg, n);
  const bool mine = tid < nseg;
  u32 entry = mine && tid ? s.seg_exit[tid - 1] : 0u, merge_at = my_b;
  // Exit of a segment entered at e (merge point in *merge).
  auto segment_exit = [&](u32 t, u32 e, u32 a_t, u32 b_t, u32* merge) -> u32 {
    *merge = b_t;
    if (e >= b_t) return e;  // an earlier token covers the whole segment
    u32 p = e;
    while (p < b_t && !is_member(p)) {
      const u32 m = token_at(p);
      p += m ? m : 1u;
    }
    *merge = p;
    return p < b_t ? s.seg_exit[t] : p;
  };
  u32 rounds = 0;
  bool unsettled = false;
  for (bool dirty = true;;) {
    if (mine && dirty) s.seg_entry[tid] = segment_exit(tid, entry, my_a, my_b, &merge_at);
    __syncthreads();
    const u32 next = mine && tid ? s.seg_entry[tid - 1] : 0u;
    dirty = mine && next != entry;
    entry = next;
    ++rounds;
    if (!__syncthreads_or(dirty)) break;
    // Chains that do not re-join for many segments (long runs of one byte)
    // would cost a round per segment, each re-walking every later segment:
    // after kStitchRounds rounds the first kStitchRounds entries are exact
    // and one thread walks the rest in order.
    if (rounds == kStitchRounds) {
      unsettled = true;
      break;
    }
  }
  if (unsettled) {
    __syncthreads();
    if (tid == 0) {
      u32 e = s.seg_entry[kStitchRounds - 1];  // exit of the last exact segment
      for (u32 t = kStitchRounds; t < nseg; ++t) {
        const u32 a_t = min_u32(t * seg, n), b_t = min_u32(a_t + seg, n);
        u32 merge = b_t;
        const u32 exit = segment_exit(t, e, a_t, b_t, &merge);
        s.seg_entry[t] = e;
        s.seg_bits[t] = merge;
        e = exit;
      }
    }
    __syncthreads();
    if (mine && tid >= kStitchRounds) {
      entry = s.seg_entry[tid];
      merge_at = s.seg_bits[tid];
    }
  }
  if (mine && tid > 0) {
    if (entry >= my_b) {
      clear_members(my_a, my_b);  // one earlier token covers the segment
    } else {
      clear_members(my_a, entry);
      for (u32 p = entry; p < merge_at;) {
        const u32 m = token_at(p);
        atomicOr(&member[p >> 5], 1u << (p & 31));
        if (m) {
          atomicOr(&ismatch[p >> 5], 1u << (p & 31));
          lenv[p] = u8(m - 3);
          if (thorough) distv[p] = u16(p - token_q);
          clear_members(p + 1, min_u32(p + m, my_b));
          p += m;
        } else {
          atomicAnd(&ismatch[p >> 5], ~(1u << (p & 31)));
          ++p;
        }
      }
    }
  }
  __syncthreads();

  // 5. Histograms over this thread's segment.
  const u32 a = min_u32(tid * seg, n), b = min_u32(a + seg, n);
  {
    u32 extra = 0, tokens = 0, dists = 0;
    for_each_token(member, ismatch, a, b, [&](u32 p, bool match) {
      ++tokens;
      if (match) {
        const u32 m = u32(lenv[p]) + 3, dist = thorough ? u32(distv[p]) : p - (u32(prev[p]) - 1);
        const u32 li = length_symbol(m), di = dist_symbol(dist);
        atomicAdd(&s.freq[257 + li], 1u);
        atomicAdd(&s.freq[286 + di], 1u);
        extra += length_extra_bits(li) + dist_extra_bits(di);
        ++dists;
      } else {
        atomicAdd(&s.freq[data[p]], 1u);
      }
    });
    atomicAdd(&s.extra_bits, extra);
    atomicAdd(&s.token_count, tokens);
    atomicAdd(&s.dist_tokens, dists);
  }
  __syncthreads();

  // 6-7. Block type by exact extent (encode_chunk, _encode_kernels.py:312-356).
  // Sums over the alphabet are warp reductions (unsigned, so the order of
  // the terms cannot change them).
  {
    u32 term = 0;
    if (tid < 286) {
      u32 f = s.freq[tid];
      if (tid == 256) s.freq[256] = ++f;  // the end-of-block code
      term = f * fixed_ll_len(tid);
    }
    term = __reduce_add_sync(kFullMask, term);
    if (lane == 0 && term) atomicAdd(&s.fixed_sum, term);
  }
  __syncthreads();
  if (tid == 0) {
    const u32 fixed_bits = 3 + s.extra_bits + s.fixed_sum + s.dist_tokens * 5;
    s.mode = 0;
    s.extent = n + 5 * stored_blocks(n);
    const u32 fixed_extent = extent_of(fixed_bits, final);
    if (fixed_extent < s.extent) { s.extent = fixed_extent; s.mode = 1; }
    s.ok = extent_of(29 + s.extra_bits + s.token_count + 1 + s.dist_tokens, final) < s.extent;
  }
  __syncthreads();
  bool trees = true;
  bool dynamic = s.ok != 0;
  if (dynamic) {
    trees = cta_tree(s, s.freq, 286, 15, s.lengths, s.codes);
    u32 term = tid < 286 ? s.freq[tid] * s.lengths[tid] : 0u;
    term = __reduce_add_sync(kFullMask, term);
    if (lane == 0 && term) atomicAdd(&s.ll_sum, term);
    __syncthreads();
    if (tid == 0) {
      const u32 ll_bits = s.ll_sum;
      s.header_bits = ll_bits;  // reused below as ll_bits
      s.ok = extent_of(29 + s.extra_bits + ll_bits + s.dist_tokens, final) < s.extent;
    }
    __syncthreads();
    dynamic = s.ok != 0;
  }
  if (trees && dynamic) {
    if (warp == 0) {
      const bool built = warp_tree(s, s.freq + 286, 30, 15, s.lengths + 286, s.codes + 286);
      if (lane == 0) {
        u32 nll = 286, ndist = 30;
        while (nll > 257 && !s.lengths[nll - 1]) --nll;
        while (ndist > 1 && !s.lengths[286 + ndist - 1]) --ndist;
        s.nll = nll;
        s.ndist = ndist;
        s.tree_ok = built;
      }
    }
    __syncthreads();
    trees = s.tree_ok != 0;
    // Run-length code the code lengths (enc_rle, _encode_kernels.py:163-191):
    // the thread at the start of each run of equal lengths emits that run's
    // symbols, in the reference's order, at the place a block scan gives.
    const u32 nll = s.nll, total = nll + s.ndist;
    auto code_length = [&](u32 i) -> u32 {
      return i < nll ? s.lengths[i] : s.lengths[286 + i - nll];
    };
    u32 value = 0, run = 0, count = 0;
    const bool first = tid < total && (tid == 0 || code_length(tid) != code_length(tid - 1));
    if (first) {
      value = code_length(tid);
      run = 1;
      while (tid + run < total && code_length(tid + run) == value) ++run;
      if (value) {
        // The length, then repeats of 3..6 (code 16), then single lengths.
        const u32 r = run - 1, tail = r % 6;
        count = 1 + r / 6 + (tail >= 3 ? 1u : tail);
      } else {
        // Zero runs of 11..138 (code 18), then one of 3..10 (code 17), then
        // single zeros.
        const u32 tail = run % 138;
        count = run / 138 + (tail >= 11 ? 1u : tail >= 3 ? 1u : tail);
      }
    }
    u32 incl_count = count;
    for (u32 o = 1; o < 32; o <<= 1) {
      const u32 v = __shfl_up_sync(kFullMask, incl_count, o);
      if (lane >= o) incl_count += v;
    }
    if (lane == 31) s.warp_sums[warp] = incl_count;
    __syncthreads();
    u32 at = incl_count - count, rle_size = 0;
    for (u32 w = 0; w < kEncWarps; ++w) {
      if (w < warp) at += s.warp_sums[w];
      rle_size += s.warp_sums[w];
    }
    if (first) {
      u32* cf = s.freq + 316;
      auto emit = [&](u32 sym, u32 extra) {
        s.rle_sym[at] = u8(sym);
        s.rle_extra[at] = u8(extra);
        atomicAdd(&cf[sym], 1u);
        ++at;
      };
      if (value) {
        emit(value, 0);
        u32 left = run - 1;
        while (left >= 3) {
          const u32 take = left < 6 ? left : 6;
          emit(16, take - 3);
          left -= take;
        }
        while (left--) emit(value, 0);
      } else {
        u32 left = run;
        while (left >= 11) {
          const u32 take = left < 138 ? left : 138;
          emit(18, take - 11);
          left -= take;
        }
        if (left >= 3) {
          emit(17, left - 3);
          left = 0;
        }
        while (left--) emit(0, 0);
      }
    }
    if (tid == 0) s.rle_size = rle_size;
    __syncthreads();
    if (warp == 0) {
      const bool built =
          trees && warp_tree(s, s.freq + 316, 19, 7, s.lengths + 316, s.codes + 316);
      if (lane == 0) {
        u32 ncl = 19;
        while (ncl > 4 && !s.lengths[316 + kClOrder[ncl - 1]]) --ncl;
        s.ncl = ncl;
        s.tree_ok = built;
      }
    }
    __syncthreads();
    trees = s.tree_ok != 0;
  }
  if (warp == 0) {
    // Distance and code-length symbol bits (the latter with their repeat
    // codes' extra bits), two terms a lane.
    u32 tail_bits = 0;
    if (trees && dynamic) {
      for (u32 i = lane; i < 49; i += 32) {
        const u32 j = i - 30;
        tail_bits += i < 30 ? s.freq[286 + i] * s.lengths[286 + i]
                            : s.freq[316 + j] * (s.lengths[316 + j] +
                                                 (j == 16 ? 2u : j == 17 ? 3u : j == 18 ? 7u : 0u));
      }
      tail_bits = __reduce_add_sync(kFullMask, tail_bits);
    }
    if (lane == 0) {
      if (!trees) {
        s.mode = 3;
        s.status = 1;
      } else if (dynamic) {
        const u32 bits = 17 + 3 * s.ncl + s.extra_bits + s.header_bits + tail_bits;
        const u32 dyn_extent = extent_of(bits, final);
        if (dyn_extent < s.extent) { s.extent = dyn_extent; s.mode = 2; }
      }
    }
  }
  __syncthreads();
  u8* slot = slots + slot_start(f.in_offset + start, g);
  const u32 slot_bytes = n + 80;
  const u32 mode = s.mode;
  if (mode == 3) {
    if (tid == 0) { status[g] = 1; sizes[g] = 0; }
    return;
  }
  if (mode == 0) {
    // Blocks of kStoredMax bytes (one for chunks within the reference's
    // bound), the last one shorter; only the stream's last block is final.
    const u32 blocks = stored_blocks(n);
    for (u32 i = tid; i < n; i += kEncThreads) slot[5 * (i / kStoredMax + 1) + i] = data[i];
    if (tid < blocks) {
      const u32 len = min_u32(n - tid * kStoredMax, kStoredMax);
      u8* head = slot + tid * (kStoredMax + 5);
      head[0] = final && tid + 1 == blocks ? 1 : 0;
      head[1] = u8(len);
      head[2] = u8(len >> 8);
      const u32 c = len ^ 0xffffu;
      head[3] = u8(c);
      head[4] = u8(c >> 8);
    }
    if (tid == 0) {
      sizes[g] = n + 5 * blocks;
      status[g] = 0;
    }
    return;
  }

  // 8. Parallel bit packing.
  const bool dyn = mode == 2;
  // Each literal/length and distance symbol's code (low 16 bits, ready to
  // put) and code length (high bits), dynamic or fixed, read once a token.
  for (u32 i = tid; i < 316; i += kEncThreads) {
    u32 code, len;
    if (dyn) {
      code = s.codes[i];
      len = s.lengths[i];
    } else if (i < 286) {
      code = fixed_ll_code(i);
      len = fixed_ll_len(i);
    } else {
      code = reverse_bits(i - 286, 5);
      len = 5;
    }
    s.sym_code[i] = code | (len << 16);
  }
  __syncthreads();
  u32 my_bits = 0;
  for_each_token(member, ismatch, a, b, [&](u32 p, bool match) {
    if (match) {
      const u32 m = u32(lenv[p]) + 3, dist = thorough ? u32(distv[p]) : p - (u32(prev[p]) - 1);
      const u32 li = length_symbol(m), di = dist_symbol(dist);
      my_bits += (s.sym_code[257 + li] >> 16) + length_extra_bits(li) +
                 (s.sym_code[286 + di] >> 16) + dist_extra_bits(di);
    } else {
      my_bits += s.sym_code[data[p]] >> 16;
    }
  });
  // Bits of this thread's run-length coded length (a dynamic header codes at
  // most 320 of them, fewer than the threads); a block scan places them.
  u32 rle_bits = 0;
  if (dyn && tid < s.rle_size) {
    const u32 sym = s.rle_sym[tid];
    rle_bits = s.lengths[316 + sym] + (sym == 16 ? 2u : sym == 17 ? 3u : sym == 18 ? 7u : 0u);
  }
  // Exclusive block scans of my_bits and rle_bits.
  u32 incl = my_bits, rle_incl = rle_bits;
  for (u32 o = 1; o < 32; o <<= 1) {
    const u32 v = __shfl_up_sync(kFullMask, incl, o);
    const u32 rv = __shfl_up_sync(kFullMask, rle_incl, o);
    if (lane >= o) {
      incl += v;
      rle_incl += rv;
    }
  }
  if (lane == 31) {
    s.warp_sums[warp] = incl;
    s.rle_sums[warp] = rle_incl;
  }
  // Zero the slot words the packed block occupies (edge words are ORed).
  u32* words = reinterpret_cast<u32*>(slot);
  const u32 used_words = min_u32((s.extent + 3) / 4 + 1, slot_bytes / 4);
  for (u32 i = tid; i < used_words; i += kEncThreads) words[i] = 0;
  __syncthreads();
  u32 before = 0, rle_before = 0, body_bits = 0, rle_total = 0;
  for (u32 w = 0; w < kEncWarps; ++w) {
    if (w < warp) {
      before += s.warp_sums[w];
      rle_before += s.rle_sums[w];
    }
    body_bits += s.warp_sums[w];
    rle_total += s.rle_sums[w];
  }
  // Block header, then (dynamic) the three counts and the code-length lengths.
  const u32 fixed_head = dyn ? 17 + 3 * s.ncl : 3;
  const u32 header_bits = fixed_head + (dyn ? rle_total : 0u);
  const u32 my_start = header_bits + before + incl - my_bits;
  if (tid == 0) {
    Packer pk;
    pk.start(words, 0, fixed_head, used_words);
    pk.put((final ? 1u : 0u) | (dyn ? 4u : 2u), 3);
    if (dyn) {
      pk.put(s.nll - 257, 5);
      pk.put(s.ndist - 1, 5);
      pk.put(s.ncl - 4, 4);
      for (u32 i = 0; i < s.ncl; ++i) pk.put(s.lengths[316 + kClOrder[i]], 3);
    }
    pk.finish();
  }
  // The run-length coded lengths, one per thread.
  if (rle_bits) {
    const u32 at = fixed_head + rle_before + rle_incl - rle_bits;
    const u32 sym = s.rle_sym[tid];
    Packer pk;
    pk.start(words, at, at + rle_bits, used_words);
    pk.put(s.codes[316 + sym], s.lengths[316 + sym]);
    if (sym >= 16) pk.put(s.rle_extra[tid], sym == 16 ? 2u : sym == 17 ? 3u : 7u);
    pk.finish();
  }
  {
    Packer pk;
    pk.start(words, my_start, my_start + my_bits, used_words);
    for_each_token(member, ismatch, a, b, [&](u32 p, bool match) {
      if (match) {
        const u32 m = u32(lenv[p]) + 3, dist = thorough ? u32(distv[p]) : p - (u32(prev[p]) - 1);
        const u32 li = length_symbol(m), di = dist_symbol(dist);
        // Each code with its extra bits in one put (at most 20 and 28 bits).
        const u32 lsym = s.sym_code[257 + li], ll = lsym >> 16;
        const u32 le = length_extra_bits(li);
        pk.put((lsym & 0xffffu) | (low_bits(m - 3, le) << ll), ll + le);
        const u32 dsym = s.sym_code[286 + di], dl = dsym >> 16;
        const u32 de = dist_extra_bits(di);
        pk.put((dsym & 0xffffu) | (low_bits(dist - 1, de) << dl), dl + de);
      } else {
        const u32 lsym = s.sym_code[data[p]];
        pk.put(lsym & 0xffffu, lsym >> 16);
      }
    });
    pk.finish();
  }
  if (tid == kEncThreads - 1) {
    // End of block, then the empty stored block that realigns a nonfinal chunk.
    const u32 at = header_bits + body_bits;
    Packer pk;
    u32 tail_bits = dyn ? s.lengths[256] : 7u;
    pk.start(words, at, at + tail_bits + 3, used_words);
    pk.first_word = pk.word;
    pk.last_word = ~0u;
    if (dyn) pk.put(s.codes[256], s.lengths[256]);
    else pk.put(fixed_ll_code(256), 7);
    u32 end = at + tail_bits;
    if (!final) {
      pk.put(0, 3);
      end += 3;
    }
    pk.finish();
    s.ok = (end + 7) / 8;
  }
  __syncthreads();
  if (tid == 0) {
    u32 bytes = s.ok;
    bool good = bytes + 8 <= slot_bytes;
    if (good && !final) {
      // LEN = 0, NLEN = 0xffff of the realigning empty stored block.
      slot[bytes] = 0;
      slot[bytes + 1] = 0;
      slot[bytes + 2] = 0xff;
      slot[bytes + 3] = 0xff;
      bytes += 4;
    }
    good = good && bytes == s.extent;
    sizes[g] = good ? bytes : 0;
    status[g] = good ? 0u : 1u;
  }
}

// Finish, one CTA per file: scan chunk sizes, check statuses and capacity,
// combine Adler partials, write the wrapper bytes and metadata
// [encoded_length, status] (FinishEncodedFile, batch_encode.cuh:39-112).
// Each warp takes a contiguous range of the file's chunks: a first pass sums
// its bytes, statuses and Adler terms (each chunk's term is independent of
// the others), then, with the earlier warps' byte totals, a warp scan writes
// every chunk's output offset.
constexpr u32 kFinishWarps = 8;
__global__ void __launch_bounds__(kFinishWarps * 32)
encode_finish_kernel(const EncodeFile* files, u32 nfiles, const u32* sizes, const u32* status,
                     const u64* adler, u64* offsets, u8* out, u32* meta, u32* range_adler,
                     u32 defer_wrapper) {
  __shared__ u64 part_bytes[kFinishWarps], part_s1[kFinishWarps], part_s2[kFinishWarps];
  __shared__ u32 part_bad[kFinishWarps];
  const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const u32 f = blockIdx.x;
  if (f >= nfiles) return;
  const EncodeFile file = files[f];
  const bool raw = (file.flags & kEncodeRaw) != 0, gzip = (file.flags & kEncodeGzip) != 0;
  // Wrapper bytes before and after the body: zlib 2 + 4, gzip 10 + 8, raw none.
  const u32 head = raw ? 0 : gzip ? 10 : 2, tail = raw ? 0 : gzip ? 8 : 4;
  const u32 per = (file.chunks + kFinishWarps - 1) / kFinishWarps;
  const u32 c0 = min_u32(warp * per, file.chunks), c1 = min_u32(c0 + per, file.chunks);
  u64 bytes = 0, s1 = 0, s2 = 0;
  u32 bad = 0;
  for (u32 c = c0 + lane; c < c1; c += 32) {
    const u32 g = file.first_chunk + c;
    bytes += sizes[g];
    bad |= status[g];
    const u64 a1 = adler[2 * u64(g)] % kAdlerMod, a2 = adler[2 * u64(g) + 1] % kAdlerMod;
    const u64 chunk_end = min_u64(u64(c + 1) * file.chunk_bytes, file.in_size);
    const u64 after = (file.in_size - chunk_end) % kAdlerMod;
    s1 += a1;
    s2 += (a2 + a1 * after) % kAdlerMod;
  }
  for (u32 o = 16; o; o >>= 1) {
    bytes += __shfl_xor_sync(kFullMask, bytes, o);
    s1 += __shfl_xor_sync(kFullMask, s1, o);
    s2 += __shfl_xor_sync(kFullMask, s2, o);
  }
  bad = __reduce_or_sync(kFullMask, bad);
  if (lane == 0) {
    part_bytes[warp] = bytes;
    part_s1[warp] = s1;
    part_s2[warp] = s2;
    part_bad[warp] = bad;
  }
  __syncthreads();
  u64 running = head;
  for (u32 w = 0; w < warp; ++w) running += part_bytes[w];
  for (u32 base = c0; base < c1; base += 32) {
    const u32 c = base + lane;
    const u64 size = c < c1 ? sizes[file.first_chunk + c] : 0u;
    u64 incl = size;
    for (u32 o = 1; o < 32; o <<= 1) {
      const u64 v = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += v;
    }
    if (c < c1) offsets[file.first_chunk + c] = running + incl - size;
    running += __shfl_sync(kFullMask, incl, 31);
  }
  if (threadIdx.x == 0) {
    u64 body = 0, t1 = 0, t2 = 0;
    u32 any_bad = 0;
    for (u32 w = 0; w < kFinishWarps; ++w) {
      body += part_bytes[w];
      t1 += part_s1[w];
      t2 += part_s2[w];
      any_bad |= part_bad[w];
    }
    const u64 total = body + head + tail;
    u32 st = any_bad ? u32(kCompressionOverflow) : 0u;
    if (!st && total > file.capacity) st = kCompressionOverflow;
    u8* dst = out + file.out_offset;
    const u32 checksum = adler_finish(t1, t2, file.in_size);
    if (range_adler) range_adler[f] = st ? 0u : checksum;
    if (defer_wrapper) {
      // Packed output: encode_wrap_kernel writes the wrapper once the file's
      // place is known (range_adler holds the checksum).
    } else if (!st && gzip) {
      // ID1 ID2 CM=8 FLG=0 MTIME=0 XFL=0 OS=255 (unknown); the trailer
      // (CRC-32, ISIZE) comes from launch_gzip_trailer.
      const u8 header[10] = {0x1f, 0x8b, 8, 0, 0, 0, 0, 0, 0, 0xff};
      for (u32 i = 0; i < 10; ++i) dst[i] = header[i];
    } else if (!st && !raw) {
      dst[0] = 0x78;
      dst[1] = 0x01;
      dst[total - 4] = u8(checksum >> 24);
      dst[total - 3] = u8(checksum >> 16);
      dst[total - 2] = u8(checksum >> 8);
      dst[total - 1] = u8(checksum);
    }
    meta[2 * f] = st ? 0u : u32(total);
    meta[2 * f + 1] = st;
  }
}

// Packed output: each file's stream starts where the previous file's ends
// (failed files take no bytes).  One CTA scans the encoded lengths.
__global__ void encode_scan_kernel(u32 nfiles, const u32* meta, u64* bases) {
  __shared__ u64 warp_total[32];
  __shared__ u64 carry;
  const u32 lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (u32 base = 0; base < nfiles; base += blockDim.x) {
    const u32 f = base + threadIdx.x;
    const u64 v = f < nfiles && !meta[2 * f + 1] ? u64(meta[2 * f]) : 0u;
    u64 incl = v;
    for (u32 o = 1; o < 32; o <<= 1) {
      const u64 t = __shfl_up_sync(kFullMask, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_total[warp] = incl;
    __syncthreads();
    u64 before = carry;
    for (u32 w = 0; w < warp; ++w) before += warp_total[w];
    if (f < nfiles) bases[f] = before + incl - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = before + incl;
    __syncthreads();
  }
}

// Packed output: the zlib header and Adler-32 trailer of every file that
// encoded, at its packed place.
__global__ void encode_wrap_kernel(u32 nfiles, const u32* meta, const u64* bases,
                                   const u32* checksums, u8* out) {
  const u32 f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= nfiles || meta[2 * f + 1]) return;
  u8* dst = out + bases[f];
  const u32 total = meta[2 * f], checksum = checksums[f];
  dst[0] = 0x78;
  dst[1] = 0x01;
  dst[total - 4] = u8(checksum >> 24);
  dst[total - 3] = u8(checksum >> 16);
  dst[total - 2] = u8(checksum >> 8);
  dst[total - 1] = u8(checksum);
}

// Copy every chunk's slot to its place in its file's output (skipped for
// files whose finish reported an error): the file's padded slot, or with
// `bases` its packed place.
__global__ void encode_pack_kernel(const EncodeFile* files, u32 nfiles, const u8* slots,
                                   const u32* sizes, const u64* offsets, const u32* meta, u8* out,
                                   u32 chunk_bytes, u32 total_chunks, const u64* bases) {
  const u32 g = blockIdx.x;
  if (g >= total_chunks) return;
  u32 lo = 0, hi = nfiles;
  while (hi - lo > 1) {
    const u32 mid = (lo + hi) >> 1;
    if (files[mid].first_chunk <= g) lo = mid;
    else hi = mid;
  }
  if (meta[2 * lo + 1]) return;
  const u32 size = sizes[g];
  const u64 start = u64(g - files[lo].first_chunk) * chunk_bytes;
  const u8* src = slots + slot_start(files[lo].in_offset + start, g);
  u8* dst = out + (bases ? bases[lo] : files[lo].out_offset) + offsets[g];
  for (u32 i = threadIdx.x; i < size; i += blockDim.x) dst[i] = src[i];
}

size_t encode_smem_bytes(u32 chunk_bytes, bool in_smem) {
  const size_t data_bytes = (chunk_bytes + 16 + 15) & ~15u;
  const size_t bit_words = bitmap_words(chunk_bytes);
  if (chunk_bytes >= kLargeChunk)  // bitmaps and a table of u32 positions
    return (2 * bit_words * 4 + kHashSlots * 4 + 15) & ~size_t(15);
  size_t bytes = data_bytes + 2 * bit_words * 4 + kHashSlots * 2;
  if (in_smem) bytes += ((chunk_bytes + 7) & ~7u) * 2 + chunk_bytes + 16;
  return (bytes + 15) & ~size_t(15);
}

cudaError_t configure_encode(int* max_dynamic_smem) {
  int device = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (e != cudaSuccess) return e;
  const int limit = optin - int(sizeof(EncodeShared<u16>)) - 1024;
  e = cudaFuncSetAttribute(encode_chunks_kernel<u16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           limit);
  if (e != cudaSuccess) return e;
  const int large = int(encode_smem_bytes(kMaxChunkBytes, false));
  if (large > optin - int(sizeof(EncodeShared<u32>)) - 1024) return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(encode_chunks_kernel<u32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           large);
  *max_dynamic_smem = limit;
  return e;
}

cudaError_t launch_encode(const u8* in, const EncodeFile* files, u32 nfiles, u32 chunk_bytes,
                          u32 total_chunks, u8* slots, u32* sizes, u32* status, u64* adler,
                          u64* offsets, const EncodeSpill& spill, u8* out, u32* meta,
                          const DeviceInfo& dev, cudaStream_t stream, u32* range_adler,
                          u64* packed_bases) {
  // Without spill buffers (the allocation-free entry point) the per-position
  // arrays stay in shared memory.
  const bool in_smem = spill.prev == nullptr;
  if (in_smem && !encode_in_smem(chunk_bytes, dev)) return cudaErrorInvalidValue;
  const size_t smem = encode_smem_bytes(chunk_bytes, in_smem);
  profile_begin("encode_chunks_kernel", stream);
  note_launch();
  if (chunk_bytes >= kLargeChunk)
    encode_chunks_kernel<u32><<<total_chunks, kEncThreads, smem, stream>>>(
        in, files, nfiles, chunk_bytes, total_chunks, slots, sizes, status, adler, spill, 0u);
  else
    encode_chunks_kernel<u16><<<total_chunks, kEncThreads, smem, stream>>>(
        in, files, nfiles, chunk_bytes, total_chunks, slots, sizes, status, adler, spill,
        in_smem ? 1u : 0u);
  profile_end(stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  note_launch();
  encode_finish_kernel<<<nfiles, kFinishWarps * 32, 0, stream>>>(
      files, nfiles, sizes, status, adler, offsets, out, meta, range_adler,
      packed_bases ? 1u : 0u);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (packed_bases) {
    note_launch();
    encode_scan_kernel<<<1, 1024, 0, stream>>>(nfiles, meta, packed_bases);
    note_launch();
    encode_wrap_kernel<<<(nfiles + 255) / 256, 256, 0, stream>>>(nfiles, meta, packed_bases,
                                                                 range_adler, out);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  profile_begin("encode_pack_kernel", stream);
  note_launch();
  encode_pack_kernel<<<total_chunks, 256, 0, stream>>>(files, nfiles, slots, sizes, offsets, meta,
                                                       out, chunk_bytes, total_chunks,
                                                       packed_bases);
  profile_end(stream);
  return cudaGetLastError();
}

bool encode_in_smem(u32 chunk_bytes, const DeviceInfo& dev) {
  return chunk_bytes < kLargeChunk &&
         encode_smem_bytes(chunk_bytes, true) <= size_t(dev.encode_smem_limit);
}

}  // namespace cz

// ---------------------------------------------------------------------------
// Compression without device allocation (cuda_zlib_compress_noalloc).
//
// Some callers cannot allocate device memory while they compress: a service
// whose allocator has reserved the whole device up front and hands out only
// its own buffers, or a latency-critical loop that must not wait on an
// allocation or a pool release.  For them this entry point runs the same
// encoder with its scratch in one file-scope device array, sized for the
// largest admitted call, which every GPU that loads the library keeps until
// the process exits.  Calls share that array: two calls that overlap on the
// GPU (different streams, or different host threads without ordering) race
// and may corrupt each other's output.  No scratch needs clearing between
// calls: every scratch word a call reads is written earlier in that call
// (the encoder zeroes the slot words it packs into).
// ---------------------------------------------------------------------------
namespace cz {
namespace {

constexpr u64 kNoAllocMaxInput = CUDA_ZLIB_NOALLOC_MAX_INPUT;
constexpr u32 kNoAllocMaxChunk = CUDA_ZLIB_NOALLOC_MAX_CHUNK;
constexpr u64 kNoAllocMaxChunks = (kNoAllocMaxInput + 255) / 256;

// Scratch layout for n input bytes in c chunks; offsets 256-byte aligned.
struct NoAllocLayout {
  u64 files, sizes, status, offsets, adler, slots, end;
};
constexpr u64 align256(u64 v) { return (v + 255) & ~u64(255); }
constexpr NoAllocLayout noalloc_layout(u64 n, u64 c) {
  NoAllocLayout l{};
  l.files = 0;
  l.sizes = align256(sizeof(EncodeFile));
  l.status = align256(l.sizes + 4 * c);
  l.offsets = align256(l.status + 4 * c);
  l.adler = align256(l.offsets + 8 * c);
  l.slots = align256(l.adler + 16 * c);
  l.end = align256(l.slots + n + 96 * (c + 2));
  return l;
}
constexpr u64 kNoAllocScratchBytes = noalloc_layout(kNoAllocMaxInput, kNoAllocMaxChunks).end;

static __device__ __align__(256) u8 noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDevice {
  bool ready = false;
  u8* scratch = nullptr;  // device address of noalloc_scratch on this device
  DeviceInfo info{};
};
std::mutex noalloc_mutex;
NoAllocDevice noalloc_devices[64];

__global__ void noalloc_set_file_kernel(EncodeFile* dst, EncodeFile file) { *dst = file; }

// One-time set-up per device, called with that device current: the array's
// device address (the host-side symbol is not one) and kernel attributes.
cudaError_t noalloc_device(int device, NoAllocDevice** out) {
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(noalloc_mutex);
  NoAllocDevice& d = noalloc_devices[device];
  if (!d.ready) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, noalloc_scratch);
    if (e != cudaSuccess) return e;
    DeviceInfo info{};
    info.device = device;
    e = cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return e;
    e = configure_encode(&info.encode_smem_limit);
    if (e != cudaSuccess) return e;
    d.scratch = static_cast<u8*>(ptr);
    d.info = info;
    d.ready = true;
  }
  *out = &d;
  return cudaSuccess;
}

cudaError_t compress_noalloc(const u8* in, u64 size, int64_t chunk_bytes, u8* out, u64 capacity,
                             u32* meta, cudaStream_t stream) {
  if (!meta || !out) return cudaErrorInvalidValue;
  if (size > kNoAllocMaxInput || chunk_bytes < 256 || chunk_bytes > int64_t(kNoAllocMaxChunk) ||
      (size && !in))
    return cudaErrorInvalidValue;
  const u32 chunk = u32(chunk_bytes);
  const u64 chunks = size ? (size + chunk - 1) / chunk : 1;
  if (capacity != size + chunks * 5 + 6) return cudaErrorInvalidValue;
  int previous = 0;
  cudaError_t e = cudaGetDevice(&previous);
  if (e != cudaSuccess) return e;
  int device = previous;
  if (stream) {
    e = cudaStreamGetDevice(stream, &device);
    if (e != cudaSuccess) return e;
  }
  if (device != previous) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return e;
  }
  NoAllocDevice* d = nullptr;
  e = noalloc_device(device, &d);
  if (e == cudaSuccess && !encode_in_smem(chunk, d->info)) e = cudaErrorInvalidValue;
  if (e == cudaSuccess) {
    const NoAllocLayout l = noalloc_layout(size, chunks);
    u8* base = d->scratch;
    EncodeFile* files = reinterpret_cast<EncodeFile*>(base + l.files);
    const EncodeFile file{0, size, 0, capacity, 0, u32(chunks), chunk, 0};
    e = cudaMemsetAsync(out, 0, capacity, stream);
    if (e == cudaSuccess) {
      note_launch();
      noalloc_set_file_kernel<<<1, 1, 0, stream>>>(files, file);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess)
      e = launch_encode(in, files, 1, chunk, u32(chunks), base + l.slots,
                        reinterpret_cast<u32*>(base + l.sizes),
                        reinterpret_cast<u32*>(base + l.status),
                        reinterpret_cast<u64*>(base + l.adler),
                        reinterpret_cast<u64*>(base + l.offsets), EncodeSpill{}, out, meta,
                        d->info, stream);
  }
  if (device != previous) cudaSetDevice(previous);
  return e;
}

}  // namespace
}  // namespace cz

extern "C" int cuda_zlib_compress_noalloc(const uint8_t* input, uint64_t size,
                                          int64_t chunk_bytes, uint8_t* output,
                                          uint64_t capacity, uint32_t* metadata, void* stream) {
  try {
    return int(cz::compress_noalloc(input, size, chunk_bytes, output, capacity, metadata,
                                    static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}
