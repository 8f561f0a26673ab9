// Host-side launchers of the codec kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace cz {

typedef uint8_t u8;
typedef uint16_t u16;
typedef uint32_t u32;
typedef uint64_t u64;

// One independent zlib stream of a decode call: input and output byte
// ranges inside the call's packed buffers.
struct StreamDesc {
  u64 in_offset, in_size, out_offset, out_size;
};

// Opt-in kernel timing (cuda_zlib_b200_profile): when enabled, launchers
// bracket their kernels with CUDA events on the launching stream.  No-ops
// otherwise.  begin/end pairs must come from the same host thread.
// Counts every kernel launch this library issues (cuda_zlib_b200_launches).
void note_launch();
void profile_begin(const char* kernel, cudaStream_t stream);
void profile_end(cudaStream_t stream);

// Per-device launch facts, filled once per device by the host layer.
struct DeviceInfo {
  int device;
  int sms;
  int serial_per_sm;    // resident CTAs of the warp-per-stream inflate kernel
  int encode_smem_limit;  // dynamic shared memory available to the chunk encoder
  int emit_per_sm;        // resident CTAs of the block-parallel emit kernel
  const void* fixed_tables;  // device copy of the fixed Huffman tables
};

// One file of an encode call.  Chunks of all files are numbered
// consecutively; files are ordered by first_chunk.
struct EncodeFile {
  u64 in_offset, in_size;    // input bytes
  u64 out_offset, capacity;  // padded output slot: size + 5 * stored blocks + 6
  u32 first_chunk, chunks, chunk_bytes, flags;
};
// EncodeFile::flags.  A range of a longer stream leaves its last chunk
// nonfinal (the stream continues) and/or omits the zlib header and trailer.
constexpr uint32_t kEncodeNotLast = 1u;
constexpr uint32_t kEncodeRaw = 2u;
// A gzip member: the 10-byte header before the body; launch_gzip_trailer
// writes the 8-byte trailer (the capacity counts 18 wrapper bytes).
constexpr uint32_t kEncodeGzip = 4u;

// CRC-32 (gzip) over a device buffer (crc32.cu).  parts: crc_segments(n)
// words of scratch; crc: the result, written on the stream.
constexpr u32 kCrcSegment = 65536;
u32 crc_segments(u64 n);
cudaError_t launch_crc32(const u8* buf, u64 n, u32* parts, u32* crc, const DeviceInfo& dev,
                         cudaStream_t stream);
// Writes CRC-32 and ISIZE into the last 8 bytes of an encoded member whose
// metadata is [length, status] (nothing when status != 0).
cudaError_t launch_gzip_trailer(u8* out, const u32* meta, const u32* crc, u64 isize,
                                cudaStream_t stream);
// After a member's body decoded with meta[0] == 0: checks its magic bytes,
// CRC-32 and ISIZE and sets meta[0] to 24, 25 or 26 on a mismatch.
cudaError_t launch_gzip_check(const u8* member, u64 size, u64 expected, const u32* crc, u32* meta,
                              cudaStream_t stream);

// Warp-per-stream inflate (serial route semantics).  `next` is a zeroed
// device counter; `order` (optional) lists stream indices largest first;
// `encoded` (optional) holds compression metadata [length, status] per
// stream, whose lengths replace desc.in_size.  meta receives [status, 0].
cudaError_t configure_serial_inflate(int* per_sm);
cudaError_t launch_serial_inflate(const u8* in, u8* out, const StreamDesc* descs,
                                  const StreamDesc& single, u32 count, const u32* order, u32* next,
                                  u32* meta, const u32* encoded, u32 max_blocks,
                                  const DeviceInfo& dev, cudaStream_t stream,
                                  bool checksum = true);

// Chunk encoder + device-side finish.  Slots: in_bytes + 96 * (chunks + 2)
// bytes; `sizes`, `status` per chunk; `adler` 2 u64 per chunk; `offsets` 1 u64
// per chunk.  With a spill (spill.prev set) the per-position arrays live in
// the global spill: `prev` (u16 entries, u32 for chunks above 65535 bytes)
// and `len` (u8), and for chunks above 65535 bytes also `data` (u8), each
// encode_spill_entries() entries; without one they stay in shared memory,
// which encode_in_smem() says the chunk fits.  `out` must be zeroed; `meta` receives
// [encoded_length, status] per file, and `range_adler` (optional) the
// Adler-32 of each file's input bytes.
struct EncodeSpill {
  void* prev;
  u8* len;
  u8* data;
  // Set: level 2 (hash-chain search, lazy evaluation), each match's distance
  // stored here (u16, same entries as prev).  Null: the reference's parse.
  u16* dist;
};
constexpr u32 kSpillGap = 64;  // spill entries between consecutive chunks' slices
inline u64 encode_spill_entries(u64 in_bytes, u32 chunks) {
  return in_bytes + u64(kSpillGap) * (u64(chunks) + 2);
}
// Chunks above the reference's 65535 bytes use 32-bit positions.
constexpr u32 kLargeChunk = 65536;
cudaError_t configure_encode(int* max_dynamic_smem);
bool encode_in_smem(u32 chunk_bytes, const DeviceInfo& dev);
cudaError_t launch_encode(const u8* in, const EncodeFile* files, u32 nfiles, u32 chunk_bytes,
                          u32 total_chunks, u8* slots, u32* sizes, u32* status, u64* adler,
                          u64* offsets, const EncodeSpill& spill, u8* out, u32* meta,
                          const DeviceInfo& dev, cudaStream_t stream,
                          u32* range_adler = nullptr, u64* packed_bases = nullptr);
// packed_bases (files u64): the streams go back to back from out[0] in file
// order (failed files take no bytes); range_adler must then be set (files
// u32: each file's Adler-32 for its trailer).

// Block-parallel inflate of one large stream (inflate_parallel.cu).
struct ParallelScratch {
  u64 bitmap_words;   // candidate bitmap words (one bit per body bit offset)
  u32 compact_blocks; // CTAs of the candidate compaction
  u32 capacity;       // candidates: min(max_candidates, 9 * body + 1) + stored-run seeds
  u32 tiles;          // fixed-region seed probes (one per 32 KiB of body)
  u32 node_capacity;  // nodes: capacity + 2 per seed
  u32 levels;         // pointer-doubling levels over node_capacity + 2 nodes
  u64 out_words;      // unresolved-position bitmap words
  u32 segments;       // Adler-32 segments of the output
  u64 symbol_words;   // contiguous token layout of the path nodes
  u32 pages;          // token arena pages (1024 words each, at least symbol_words)
  u32 max_units;      // expansion units: node_capacity + expected / 32 KiB + 2
  u32 stages;         // staged-resolve stages (32 units each) over max_units
};
struct ParallelBuffers {
  u32* bitmap;        // bitmap_words, from discover_kernel (the reference's rule)
  u32* extra;         // bitmap_words, zeroed: stored-run seeds (fast path only)
  u32* seed_raw;      // tiles: probe result per tile
  u32* seeds;         // tiles: sorted fixed-region seeds
  u32* seed_total;    // 1
  u32* block_counts;  // compact_blocks
  u32* total;         // 1: distinct candidates
  u32* cands;         // capacity
  u32 *ends, *sizes, *blocks, *infos, *tokens;  // node_capacity each
  u32* jump;          // (node_capacity + 2) * levels
  u32 *path, *prefix, *tprefix;  // node_capacity each: path nodes, output and token offsets
  u32* state;         // 3: path length, chain ok, contiguous-layout fallback
  u32* counters;      // 3, zeroed: describe / symbols / expand work counters
  u32* syms;          // pages * 1024 words: the token arena
  u32 *first_page, *page_next, *page_used;  // node_capacity, pages, pages
  u32* page_cursor;   // 1, zeroed: next free arena page
  u32* source;        // expected + 32: absolute source of unresolved positions
  u32* unresolved;    // out_words, zeroed
  u64* parts;         // 2 * segments
  u32* fail;          // 1, zeroed
  u32* deep;          // 1, zeroed: some marker chain is too long to chase
  u32* longs;         // out_words: markers whose chase ran out of hops
  u32* stage_done;    // stages + 1, zeroed: tiles done per stage, then the ticket
  u32* unit_counts;   // node_capacity: expansion units per path item
  u32* item_units;    // node_capacity + 1: their exclusive prefix, then the total
  u32 *unit_item, *unit_page, *unit_first, *unit_tokens, *unit_start, *unit_bytes;  // max_units
  u32* stash;         // round_stash_words: tokens the node warps keep per round
};
ParallelScratch parallel_scratch_layout(u64 in_size, u64 expected, u32 capacity,
                                        u64 arena_slack);
u64 round_stash_words(const DeviceInfo& dev);
// Allocates and builds the fixed Huffman tables on the current device.
cudaError_t build_fixed_tables(void** out);
cudaError_t configure_parallel_inflate(int* emit_per_sm);
// Writes the fast-path verdict to meta[0]: 0 ok, 21 checksum, 1 other failure.
// checksum false skips the Adler-32 trailer (a body framed for decoding).
cudaError_t launch_parallel_inflate(const u8* in, u64 in_size, u8* out, u64 expected,
                                    u32 max_blocks, const ParallelScratch& s,
                                    const ParallelBuffers& b, u32* meta, const DeviceInfo& dev,
                                    cudaStream_t stream, bool checksum = true);

// General-route status path (single streams outside the small route).
// bitmap: one bit per body bit offset, zeroed; count: zeroed u32.
// queue: discover_queue_capacity(in_size) u32; queued: zeroed u32[2] (offsets
// queued, validation cursor).
u32 discover_queue_capacity(u64 in_size);
// extra: zeroed bitmap that receives the stored-run seeds (fast path only;
// the reference's candidate rule and event count are in bitmap / count).
cudaError_t launch_discover(const u8* in, u64 in_size, u32* bitmap, u32* extra, u32* count,
                            u32* queue, u32 queue_cap, u32* queued, const u32* gate,
                            const DeviceInfo& dev, cudaStream_t stream);
// meta[0] holds the fast path status; rewritten with the route's status;
// a failed output is zeroed.
cudaError_t launch_general_status(const u8* in, u64 in_size, u64 expected, u32 max_candidates,
                                  u32 max_blocks, const u32* bitmap, const u32* count, u32* meta,
                                  u8* out, cudaStream_t stream);
// Zeroes out[0, expected) when meta[0] != 0.
cudaError_t launch_clear_on_failure(const u32* meta, u8* out, u64 expected, cudaStream_t stream);

}  // namespace cz
