// Host orchestration and the C ABI (include/cuda_zlib_b200.h).
//
// Mirrors the reference's handler layer (src/cuda_zlib/native/codec_ffi.cu):
// argument validation with the same statuses and error returns, a per-device
// stream-ordered scratch pool with a release threshold and stats/trim
// controls, and route selection for single-stream decode.  Unlike the
// reference, compression never reads its chunk sizes back to the host: the
// sizes are scanned on the device, so every call is asynchronous.
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <numeric>
#include <string>
#include <utility>
#include <vector>

#include "../../include/cuda_zlib_b200.h"
#include "kernels.h"

namespace cz {
namespace {

constexpr u32 kMaxBytes = 1u << 28;
// Single-stream bounds, a deliberate superset of the reference's 2**28
// (_codec.py:13,28,103; codec_ffi.cu:42): a stream decodes to at most 2**31
// bytes from at most 2**29 - 2**16 compressed bytes (body bit offsets stay
// below 2**32), and compresses at most 2**31 input bytes.  Batch calls keep
// the reference's 2**28 totals.
constexpr u64 kMaxStreamBytes = u64(1) << 31;
constexpr u64 kMaxStreamInput = (u64(1) << 29) - (u64(1) << 16);
// Chunk sizes: the reference's [256, 65535] (_codec.py:158-159) and, beyond
// it, chunks up to 2**18 whose stored fallback takes several blocks.
constexpr int64_t kMinChunk = 256;
constexpr int64_t kMaxChunk = 262144;
constexpr u32 kStoredMax = 65535;
constexpr u32 kMaxBlocks = 262144;
constexpr u32 kMaxCandidates = 262144;
constexpr u32 kTruncated = 1;
constexpr u32 kTruncatedZlib = 14;
constexpr u32 kInvalidBounds = 23;
constexpr u32 kGzipHeader = 24;
constexpr int kMaxDevices = 64;

#define CZ_TRY(expression)                     \
  do {                                         \
    cudaError_t error_ = (expression);         \
    if (error_ != cudaSuccess) return error_;  \
  } while (false)

// ---------------------------------------------------------------------------
// Per-device state: launch facts and the scratch pool.
// ---------------------------------------------------------------------------
// Page-locked staging for the small host tables a call uploads (file and
// stream descriptors).  A copy from pageable memory makes CUDA wait for the
// stream to drain before it starts, which would stall every batch call
// behind the previous call's kernels; from here the copy is asynchronous.
// Slots are reused round robin once the copy that last read them is done.
constexpr int kStagingSlots = 16;
constexpr size_t kStagingSlotBytes = size_t(512) << 10;
struct StagingSlot {
  std::mutex mutex;  // held while the slot is filled and its copy issued
  cudaEvent_t done = nullptr;
};
struct Staging {
  std::mutex mutex;
  u8* host = nullptr;  // kStagingSlots * kStagingSlotBytes, page-locked
  int next = 0;
  StagingSlot slots[kStagingSlots];
};

struct DeviceState {
  bool ready = false;
  DeviceInfo info{};
  cudaMemPool_t pool = nullptr;
  Staging* staging = nullptr;
};

struct Registry {
  std::mutex mutex;
  u64 retention = 1ull << 30;
  bool pools_created = false;
  std::array<DeviceState, kMaxDevices> devices;
};

Registry& registry() {
  static Registry* r = new Registry;  // process lifetime, no teardown CUDA calls
  return *r;
}

cudaError_t device_state(int device, DeviceState** out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  Registry& r = registry();
  std::lock_guard<std::mutex> lock(r.mutex);
  DeviceState& d = r.devices[device];
  if (!d.ready) {
    DeviceInfo info{};
    info.device = device;
    CZ_TRY(cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, device));
    CZ_TRY(configure_serial_inflate(&info.serial_per_sm));
    CZ_TRY(configure_encode(&info.encode_smem_limit));
    CZ_TRY(configure_parallel_inflate(&info.emit_per_sm));
    void* fixed = nullptr;
    CZ_TRY(build_fixed_tables(&fixed));
    info.fixed_tables = fixed;
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    cudaMemPool_t pool = nullptr;
    CZ_TRY(cudaMemPoolCreate(&pool, &props));
    cudaError_t e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &r.retention);
    if (e != cudaSuccess) {
      cudaMemPoolDestroy(pool);
      return e;
    }
    Staging* staging = new Staging;
    e = cudaHostAlloc(reinterpret_cast<void**>(&staging->host),
                      kStagingSlots * kStagingSlotBytes, cudaHostAllocPortable);
    for (int k = 0; e == cudaSuccess && k < kStagingSlots; ++k)
      e = cudaEventCreateWithFlags(&staging->slots[k].done, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      cudaMemPoolDestroy(pool);
      return e;  // the staging block is kept: a failed set-up is not retried cheaply
    }
    d.info = info;
    d.pool = pool;
    d.staging = staging;
    d.ready = true;
    r.pools_created = true;
  }
  *out = &d;
  return cudaSuccess;
}

// Makes the stream's device current for the call and restores the caller's.
class DeviceScope {
 public:
  explicit DeviceScope(cudaStream_t stream) {
    error_ = cudaGetDevice(&previous_);
    if (error_ != cudaSuccess) return;
    device_ = previous_;
    if (stream) {
      error_ = cudaStreamGetDevice(stream, &device_);
      if (error_ != cudaSuccess) return;
    }
    if (device_ != previous_) {
      error_ = cudaSetDevice(device_);
      switched_ = error_ == cudaSuccess;
    }
  }
  ~DeviceScope() {
    if (switched_) cudaSetDevice(previous_);
  }
  cudaError_t error() const { return error_; }
  int device() const { return device_; }

 private:
  int previous_ = 0, device_ = 0;
  bool switched_ = false;
  cudaError_t error_ = cudaSuccess;
};

// Stream-ordered scratch for one call; freed on the same stream.
class Workspace {
 public:
  Workspace(cudaMemPool_t pool, cudaStream_t stream) : pool_(pool), stream_(stream) {}
  ~Workspace() { release(); }
  template <typename T>
  cudaError_t allocate(T** out, size_t count) {
    void* p = nullptr;
    CZ_TRY(cudaMallocFromPoolAsync(&p, std::max<size_t>(1, count) * sizeof(T), pool_, stream_));
    held_.push_back(p);
    *out = static_cast<T*>(p);
    return cudaSuccess;
  }
  cudaError_t release() {
    cudaError_t first = cudaSuccess;
    while (!held_.empty()) {
      cudaError_t e = cudaFreeAsync(held_.back(), stream_);
      if (first == cudaSuccess) first = e;
      held_.pop_back();
    }
    return first;
  }

 private:
  cudaMemPool_t pool_;
  cudaStream_t stream_;
  std::vector<void*> held_;
};

// ---------------------------------------------------------------------------
// Opt-in kernel timing.
// ---------------------------------------------------------------------------
struct ProfileRecord {
  const char* kernel;
  cudaEvent_t start, stop;
  int device;
};
struct ProfileTotals {
  std::string kernel;
  double ms = 0;
  u64 launches = 0;
};
// Events are created ahead (when timing is switched on) and reused, so a
// timed region makes no event-creation calls, which go through the driver
// and can wait behind other processes' queries of the GPU.
constexpr int kSpareEvents = 512;
struct Profiler {
  std::mutex mutex;
  bool enabled = false;
  std::vector<ProfileRecord> pending;
  std::vector<ProfileTotals> totals;
  std::vector<std::pair<int, cudaEvent_t>> spare;  // (device, event)
  cudaEvent_t take(int device) {  // caller holds the mutex
    for (size_t i = spare.size(); i-- > 0;) {
      if (spare[i].first == device) {
        const cudaEvent_t e = spare[i].second;
        spare[i] = spare.back();
        spare.pop_back();
        return e;
      }
    }
    cudaEvent_t e = nullptr;
    return cudaEventCreate(&e) == cudaSuccess ? e : nullptr;
  }
};
Profiler& profiler() {
  static Profiler* p = new Profiler;
  return *p;
}
thread_local ProfileRecord open_record{nullptr, nullptr, nullptr, 0};

// Fold completed records into the totals (waits for their stop events).
cudaError_t profile_drain(Profiler& p) {
  for (ProfileRecord& r : p.pending) {
    CZ_TRY(cudaEventSynchronize(r.stop));
    float ms = 0;
    CZ_TRY(cudaEventElapsedTime(&ms, r.start, r.stop));
    auto it = std::find_if(p.totals.begin(), p.totals.end(),
                           [&](const ProfileTotals& t) { return t.kernel == r.kernel; });
    if (it == p.totals.end()) {
      p.totals.push_back(ProfileTotals{r.kernel, 0, 0});
      it = p.totals.end() - 1;
    }
    it->ms += ms;
    it->launches += 1;
    p.spare.emplace_back(r.device, r.start);
    p.spare.emplace_back(r.device, r.stop);
  }
  p.pending.clear();
  return cudaSuccess;
}

}  // namespace

namespace {
std::atomic<uint64_t> launches_issued{0};
}

void note_launch() { launches_issued.fetch_add(1, std::memory_order_relaxed); }

void profile_begin(const char* kernel, cudaStream_t stream) {
  Profiler& p = profiler();
  ProfileRecord r{kernel, nullptr, nullptr, 0};
  {
    std::lock_guard<std::mutex> lock(p.mutex);
    if (!p.enabled) return;
    if (cudaGetDevice(&r.device) != cudaSuccess) return;
    r.start = p.take(r.device);
    r.stop = p.take(r.device);
    if (!r.start || !r.stop) {
      if (r.start) p.spare.emplace_back(r.device, r.start);
      if (r.stop) p.spare.emplace_back(r.device, r.stop);
      return;
    }
  }
  cudaEventRecord(r.start, stream);
  open_record = r;
}

void profile_end(cudaStream_t stream) {
  if (!open_record.kernel) return;
  cudaEventRecord(open_record.stop, stream);
  Profiler& p = profiler();
  std::lock_guard<std::mutex> lock(p.mutex);
  p.pending.push_back(open_record);
  open_record = ProfileRecord{nullptr, nullptr, nullptr, 0};
}

namespace {

__global__ void set_meta_kernel(u32* meta, u32 first, u32 second) {
  meta[0] = first;
  meta[1] = second;
}

cudaError_t set_meta(u32* meta, u32 first, u32 second, cudaStream_t stream) {
  note_launch();
  set_meta_kernel<<<1, 1, 0, stream>>>(meta, first, second);
  return cudaGetLastError();
}

template <typename T>
cudaError_t upload(const DeviceState& dev, Workspace& ws, T** out, const std::vector<T>& host,
                   cudaStream_t stream) {
  CZ_TRY(ws.allocate(out, host.size()));
  if (host.empty()) return cudaSuccess;
  const size_t bytes = host.size() * sizeof(T);
  if (bytes > kStagingSlotBytes || !dev.staging) {
    // Larger tables copy from pageable memory: the copy stages the bytes
    // before returning, so the vector may be released right after.
    return cudaMemcpyAsync(*out, host.data(), bytes, cudaMemcpyHostToDevice, stream);
  }
  Staging& st = *dev.staging;
  int k = 0;
  {
    std::lock_guard<std::mutex> lock(st.mutex);
    k = st.next;
    st.next = (st.next + 1) % kStagingSlots;
  }
  StagingSlot& slot = st.slots[k];
  std::lock_guard<std::mutex> hold(slot.mutex);
  CZ_TRY(cudaEventSynchronize(slot.done));  // the slot's previous copy has read it
  u8* pinned = st.host + size_t(k) * kStagingSlotBytes;
  std::memcpy(pinned, host.data(), bytes);
  CZ_TRY(cudaMemcpyAsync(*out, pinned, bytes, cudaMemcpyHostToDevice, stream));
  return cudaEventRecord(slot.done, stream);
}

// ---------------------------------------------------------------------------
// Encode (single stream and batch share one path).
// ---------------------------------------------------------------------------
// Worst-case layout of n input bytes at `chunk`: chunk count, stored blocks
// of the chunks' stored fallbacks (one per chunk up to 65535 bytes), which
// size the padded capacity n + 5 * stored + 6, and the most Deflate blocks the
// stream can hold (the reference's 2 * chunks - 1 for chunks <= 65535:
// every nonfinal chunk ends with an empty stored block).
struct StreamLayout {
  u64 chunks, stored, blocks, capacity;
};
u64 stored_blocks(u64 n) { return n ? (n + kStoredMax - 1) / kStoredMax : 1; }
StreamLayout stream_layout(u64 n, u32 chunk) {
  StreamLayout l{};
  l.chunks = n ? (n + chunk - 1) / chunk : 1;
  const u64 full = stored_blocks(chunk), tail = stored_blocks(n - (l.chunks - 1) * chunk);
  l.stored = (l.chunks - 1) * full + tail;
  l.blocks = (l.chunks - 1) * std::max<u64>(full, 2) + tail;
  l.capacity = n + 5 * l.stored + 6;
  return l;
}
bool chunk_ok(int64_t chunk_bytes) { return chunk_bytes >= kMinChunk && chunk_bytes <= kMaxChunk; }

cudaError_t encode_files(const DeviceState& dev, const u8* in, u64 in_bytes,
                         std::vector<EncodeFile>& files, u32 chunk_bytes, u32 total_chunks,
                         u8* out, u32* meta, cudaStream_t stream, u32* range_adler = nullptr,
                         u32 level = 1, bool packed = false) {
  Workspace ws(dev.pool, stream);
  EncodeFile* d_files = nullptr;
  u8* slots = nullptr;
  u32 *sizes = nullptr, *status = nullptr;
  u64 *adler = nullptr, *offsets = nullptr;
  EncodeSpill spill{};
  CZ_TRY(upload(dev, ws, &d_files, files, stream));
  CZ_TRY(ws.allocate(&slots, in_bytes + 96 * (u64(total_chunks) + 2)));
  CZ_TRY(ws.allocate(&sizes, total_chunks));
  CZ_TRY(ws.allocate(&status, total_chunks));
  CZ_TRY(ws.allocate(&adler, 2 * u64(total_chunks)));
  CZ_TRY(ws.allocate(&offsets, total_chunks));
  {
    // Pooled calls use the global spill: with the per-position arrays there,
    // two encoder CTAs fit an SM's shared memory instead of one.  Level 2
    // follows hash chains through prev[], so it keeps them in shared memory
    // where they fit, and stores its match distances in the spill.
    const u64 entries = encode_spill_entries(in_bytes, total_chunks);
    if (level == 2) CZ_TRY(ws.allocate(&spill.dist, entries));
    if (level != 2 || !encode_in_smem(chunk_bytes, dev.info)) {
      u8* prev = nullptr;
      CZ_TRY(ws.allocate(&prev, entries * (chunk_bytes >= kLargeChunk ? 4 : 2)));
      CZ_TRY(ws.allocate(&spill.len, entries));
      if (chunk_bytes >= kLargeChunk) CZ_TRY(ws.allocate(&spill.data, entries));
      spill.prev = prev;
    }
  }
  u64* bases = nullptr;
  if (packed) {
    CZ_TRY(ws.allocate(&bases, files.size()));
    CZ_TRY(ws.allocate(&range_adler, files.size()));
  }
  CZ_TRY(launch_encode(in, d_files, u32(files.size()), chunk_bytes, total_chunks, slots, sizes,
                       status, adler, offsets, spill, out, meta, dev.info, stream, range_adler,
                       bases));
  return ws.release();
}

// Extra words of the token arena beyond the exact bound of the path's tokens
// (CUDA_ZLIB_TOKEN_ARENA_SLACK, default 8 Mi words): room for the partial
// last page of every candidate.  When it runs out the stream is still decoded
// exactly, with a second decoding pass into the exact layout.
u64 token_arena_slack() {
  const char* text = std::getenv("CUDA_ZLIB_TOKEN_ARENA_SLACK");
  u64 value = u64(1) << 23;
  if (text && *text) {
    char* end = nullptr;
    const unsigned long long v = std::strtoull(text, &end, 10);
    if (end && !*end && v <= (u64(1) << 32)) value = v;
  }
  return value;
}

// ---------------------------------------------------------------------------
// Entry point bodies (validation follows codec_ffi.cu line for line in effect).
// ---------------------------------------------------------------------------
cudaError_t compress(const u8* in, u64 size, int64_t chunk_bytes, u8* out, u64 capacity,
                     u32* meta, cudaStream_t stream) {
  if (!meta) return cudaErrorInvalidValue;
  DeviceScope scope(stream);
  CZ_TRY(scope.error());
  DeviceState* dev = nullptr;
  CZ_TRY(device_state(scope.device(), &dev));
  // Compress (codec_ffi.cu:551-571): output bound, then zero, then input and
  // chunk bounds; any violation is metadata [0, 23].  The bounds are this
  // codec's single-stream ones (2**31 input bytes, chunks up to 2**18).
  if (capacity > kMaxStreamBytes + 5 * stored_blocks(kMaxStreamBytes) + 6)
    return set_meta(meta, 0, kInvalidBounds, stream);
  if (capacity) {
    if (!out) return cudaErrorInvalidValue;
    CZ_TRY(cudaMemsetAsync(out, 0, capacity, stream));
  }
  if (size > kMaxStreamBytes || !chunk_ok(chunk_bytes) || (size && !in))
    return set_meta(meta, 0, kInvalidBounds, stream);
  const u32 chunk = u32(chunk_bytes);
  const StreamLayout l = stream_layout(size, chunk);
  if (l.blocks > kMaxBlocks || capacity != l.capacity)
    return set_meta(meta, 0, kInvalidBounds, stream);
  std::vector<EncodeFile> files(1);
  files[0] = EncodeFile{0, size, 0, capacity, 0, u32(l.chunks), chunk, 0};
  return encode_files(*dev, in, size, files, chunk, u32(l.chunks), out, meta, stream);
}

// One contiguous range of a longer stream: raw Deflate chunks, the last one
// nonfinal unless `last`, and the range's Adler-32 in meta[2].  Splicing the
// ranges of a stream (header + bodies + combined Adler-32) gives exactly the
// stream that compress() makes of the whole input, since chunks are encoded
// independently.
cudaError_t compress_range(const u8* in, u64 size, int64_t chunk_bytes, int last, u8* out,
                           u64 capacity, u32* meta, cudaStream_t stream) {
  if (!meta || !out || (size && !in)) return cudaErrorInvalidValue;
  if (size > kMaxStreamBytes || !chunk_ok(chunk_bytes)) return cudaErrorInvalidValue;
  const u32 chunk = u32(chunk_bytes);
  const StreamLayout l = stream_layout(size, chunk);
  const u64 chunks = l.chunks;
  if (l.blocks > kMaxBlocks || capacity != l.capacity || (!last && size % chunk))
    return cudaErrorInvalidValue;
  DeviceScope scope(stream);
  CZ_TRY(scope.error());
  DeviceState* dev = nullptr;
  CZ_TRY(device_state(scope.device(), &dev));
  CZ_TRY(cudaMemsetAsync(out, 0, capacity, stream));
  std::vector<EncodeFile> files(1);
  files[0] = EncodeFile{0, size, 0, capacity, 0, u32(chunks), chunk,
                        kEncodeRaw | (last ? 0u : kEncodeNotLast)};
  return encode_files(*dev, in, size, files, chunk, u32(chunks), out, meta, stream, meta + 2);
}

cudaError_t compress_batch(const u8* in, u64 in_bytes, const int64_t* sizes, u64 count,
                           int64_t chunk_bytes, u8* out, u64 out_bytes, u32* meta,
                           cudaStream_t stream, bool packed = false) {
  // CompressBatchImpl (codec_ffi.cu:1002-1063).
  if (!count || count > kMaxBlocks || !sizes || !meta) return cudaErrorInvalidValue;
  if (in_bytes > kMaxBytes || out_bytes > kMaxBytes || !chunk_ok(chunk_bytes))
    return cudaErrorInvalidValue;
  const u32 chunk = u32(chunk_bytes);
  std::vector<EncodeFile> files(count);
  u64 in_extent = 0, out_extent = 0, total_chunks = 0;
  for (u64 i = 0; i < count; ++i) {
    const int64_t size = sizes[i];
    if (size < 0 || size > int64_t(kMaxBytes)) return cudaErrorInvalidValue;
    const StreamLayout l = stream_layout(u64(size), chunk);
    const u64 n = l.chunks, cap = l.capacity;
    if (l.blocks > kMaxBlocks || in_extent + u64(size) > kMaxBytes ||
        out_extent + cap > kMaxBytes || total_chunks + n > kMaxBlocks)
      return cudaErrorInvalidValue;
    files[i] = EncodeFile{in_extent, u64(size), out_extent, cap, u32(total_chunks), u32(n), chunk,
                          0};
    in_extent += u64(size);
    out_extent += cap;
    total_chunks += n;
  }
  if (in_extent != in_bytes || out_extent != out_bytes) return cudaErrorInvalidValue;
  if ((in_bytes && !in) || !out) return cudaErrorInvalidValue;
  DeviceScope scope(stream);
  CZ_TRY(scope.error());
  DeviceState* dev = nullptr;
  CZ_TRY(device_state(scope.device(), &dev));
  CZ_TRY(cudaMemsetAsync(out, 0, out_bytes, stream));
  return encode_files(*dev, in, in_bytes, files, chunk, u32(total_chunks), out, meta, stream,
                      nullptr, 1, packed);
}

cudaError_t decompress(const u8* in, u64 size, int64_t max_candidates, int64_t max_blocks,
                       u8* out, u64 expected, u32* meta, cudaStream_t stream,
                       bool checksum = true) {
  if (!meta) return cudaErrorInvalidValue;
  DeviceScope scope(stream);
  CZ_TRY(scope.error());
  DeviceState* dev = nullptr;
  CZ_TRY(device_state(scope.device(), &dev));
  // Decompress (codec_ffi.cu:662-680), with this codec's single-stream bounds.
  if (expected > kMaxStreamBytes) return set_meta(meta, kInvalidBounds, 0, stream);
  if (expected && !out) return cudaErrorInvalidValue;
  auto fail = [&](u32 status) -> cudaError_t {
    if (expected) CZ_TRY(cudaMemsetAsync(out, 0, expected, stream));
    return set_meta(meta, status, 0, stream);
  };
  if (size > kMaxStreamInput || max_candidates < 1 ||
      max_candidates > int64_t(kMaxCandidates) || max_blocks < 1 ||
      max_blocks > int64_t(kMaxBlocks))
    return fail(kInvalidBounds);
  if (size < 8) return fail(kTruncatedZlib);
  if (!in) return cudaErrorInvalidValue;
  const StreamDesc single{0, size, 0, expected};
  const bool defaults = max_candidates == int64_t(kMaxCandidates) &&
                        max_blocks == int64_t(kMaxBlocks);
  Workspace ws(dev->pool, stream);
  u32* counter = nullptr;
  CZ_TRY(ws.allocate(&counter, 1));
  CZ_TRY(cudaMemsetAsync(counter, 0, sizeof(u32), stream));
  if (expected <= 65536 && size <= 131072 && defaults) {
    // Small route: serial semantics (codec_ffi.cu:681-695).
    CZ_TRY(launch_serial_inflate(in, out, nullptr, single, 1, nullptr, counter, meta, nullptr,
                                 u32(max_blocks), dev->info, stream, checksum));
    return ws.release();
  }
  // General route: candidate discovery (always: its count alone can fail a
  // valid stream), the block-parallel decode, then the route's exact status
  // if the fast path failed.
  const u64 body = size - 6;
  const u32 capacity = u32(std::min<u64>(u64(max_candidates), body * 9 + 1));
  const ParallelScratch layout = parallel_scratch_layout(size, expected, capacity,
                                                         token_arena_slack());
  const u32 nodes = layout.node_capacity;
  ParallelBuffers b{};
  u32* count = nullptr;
  CZ_TRY(ws.allocate(&b.bitmap, layout.bitmap_words));
  CZ_TRY(ws.allocate(&b.extra, layout.bitmap_words));
  CZ_TRY(ws.allocate(&b.seed_raw, layout.tiles));
  CZ_TRY(ws.allocate(&b.seeds, layout.tiles));
  CZ_TRY(ws.allocate(&b.seed_total, 1));
  CZ_TRY(ws.allocate(&count, 1));
  const u32 queue_cap = discover_queue_capacity(size);
  u32 *queue = nullptr, *queued = nullptr;
  CZ_TRY(ws.allocate(&queue, queue_cap));
  CZ_TRY(ws.allocate(&queued, 2));
  CZ_TRY(ws.allocate(&b.block_counts, layout.compact_blocks));
  CZ_TRY(ws.allocate(&b.total, 1));
  CZ_TRY(ws.allocate(&b.cands, layout.capacity));
  CZ_TRY(ws.allocate(&b.ends, nodes));
  CZ_TRY(ws.allocate(&b.sizes, nodes));
  CZ_TRY(ws.allocate(&b.blocks, nodes));
  CZ_TRY(ws.allocate(&b.infos, nodes));
  CZ_TRY(ws.allocate(&b.tokens, nodes));
  CZ_TRY(ws.allocate(&b.jump, (u64(nodes) + 2) * layout.levels));
  CZ_TRY(ws.allocate(&b.path, nodes));
  CZ_TRY(ws.allocate(&b.prefix, nodes));
  CZ_TRY(ws.allocate(&b.tprefix, nodes));
  CZ_TRY(ws.allocate(&b.syms, u64(layout.pages) * 1024));
  CZ_TRY(ws.allocate(&b.first_page, nodes));
  CZ_TRY(ws.allocate(&b.page_next, layout.pages));
  CZ_TRY(ws.allocate(&b.page_used, layout.pages));
  CZ_TRY(ws.allocate(&b.page_cursor, 1));
  CZ_TRY(ws.allocate(&b.state, 3));
  CZ_TRY(ws.allocate(&b.counters, 3));
  CZ_TRY(ws.allocate(&b.source, expected + 32));  // read in 32-entry words
  CZ_TRY(ws.allocate(&b.unresolved, layout.out_words));
  CZ_TRY(ws.allocate(&b.parts, 2 * u64(layout.segments)));
  CZ_TRY(ws.allocate(&b.fail, 1));
  CZ_TRY(ws.allocate(&b.deep, 1));
  CZ_TRY(ws.allocate(&b.longs, layout.out_words));
  CZ_TRY(ws.allocate(&b.stage_done, u64(layout.stages) + 1));
  CZ_TRY(ws.allocate(&b.unit_counts, nodes));
  CZ_TRY(ws.allocate(&b.item_units, u64(nodes) + 1));
  for (u32** unit_array : {&b.unit_item, &b.unit_page, &b.unit_first, &b.unit_tokens,
                           &b.unit_start, &b.unit_bytes})
    CZ_TRY(ws.allocate(unit_array, layout.max_units));
  CZ_TRY(ws.allocate(&b.stash, round_stash_words(dev->info)));
  CZ_TRY(cudaMemsetAsync(b.bitmap, 0, layout.bitmap_words * sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(b.extra, 0, layout.bitmap_words * sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(count, 0, sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(queued, 0, 2 * sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(b.counters, 0, 3 * sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(b.page_cursor, 0, sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(b.unresolved, 0, layout.out_words * sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(b.fail, 0, sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(b.deep, 0, sizeof(u32), stream));
  CZ_TRY(cudaMemsetAsync(b.stage_done, 0, (u64(layout.stages) + 1) * sizeof(u32), stream));
  CZ_TRY(launch_discover(in, size, b.bitmap, b.extra, count, queue, queue_cap, queued, nullptr,
                         dev->info, stream));
  CZ_TRY(launch_parallel_inflate(in, size, out, expected, u32(max_blocks), layout, b, meta,
                                 dev->info, stream, checksum));
  CZ_TRY(launch_general_status(in, size, expected, u32(max_candidates), u32(max_blocks), b.bitmap,
                               count, meta, out, stream));
  return ws.release();
}

// ---------------------------------------------------------------------------
// gzip (RFC 1952) and raw Deflate (RFC 1951) wrappers around the same body
// codec.  The reference supports RFC 1950 only; these are this codec's.
// ---------------------------------------------------------------------------
enum Format : int32_t { kFormatZlib = 0, kFormatRaw = 1, kFormatGzip = 2 };

// Wrapper bytes of a member around its Deflate body.
u64 wrapper_bytes(int32_t format) {
  return format == kFormatRaw ? 0 : format == kFormatGzip ? 18 : 6;
}

// Bitwise CRC-32 for the few bytes of a gzip header (FHCRC).
u32 host_crc32(const u8* p, u64 n) {
  u32 r = 0xFFFFFFFFu;
  for (u64 i = 0; i < n; ++i) {
    r ^= p[i];
    for (int k = 0; k < 8; ++k) r = (r >> 1) ^ ((r & 1u) ? 0xEDB88320u : 0u);
  }
  return r ^ 0xFFFFFFFFu;
}

// Length of the gzip member header at host bytes [0, available): magic,
// CM = 8, no reserved flag bits, the optional FEXTRA / FNAME / FCOMMENT
// fields and, with FHCRC, the header CRC-16.  0 when valid and complete,
// else kGzipHeader.
u32 gzip_header(const u8* p, u64 available, u64* header_bytes) {
  *header_bytes = 0;
  if (!p || available < 10 || p[0] != 0x1f || p[1] != 0x8b || p[2] != 8 || (p[3] & 0xe0))
    return kGzipHeader;
  const u32 flags = p[3];
  u64 at = 10;
  if (flags & 4) {  // FEXTRA: XLEN, then XLEN bytes
    if (available < at + 2) return kGzipHeader;
    at += 2 + (u64(p[at]) | (u64(p[at + 1]) << 8));
  }
  for (u32 field : {8u, 16u}) {  // FNAME, FCOMMENT: zero-terminated
    if (!(flags & field)) continue;
    while (at < available && p[at]) ++at;
    if (at >= available) return kGzipHeader;
    ++at;
  }
  if (flags & 2) {  // FHCRC: the low 16 bits of the CRC-32 of the bytes before
    if (available < at + 2) return kGzipHeader;
    const u32 want = u32(p[at]) | (u32(p[at + 1]) << 8);
    if ((host_crc32(p, at) & 0xffffu) != want) return kGzipHeader;
    at += 2;
  }
  if (at > available) return kGzipHeader;
  *header_bytes = at;
  return 0;
}

cudaError_t compress_format(const u8* in, u64 size, int64_t chunk_bytes, int32_t format,
                            int32_t level, u8* out, u64 capacity, u32* meta, cudaStream_t stream) {
  if (level != 1 && level != 2) return cudaErrorInvalidValue;
  if (format == kFormatZlib && level == 1)
    return compress(in, size, chunk_bytes, out, capacity, meta, stream);
  if (!meta || (format != kFormatZlib && format != kFormatRaw && format != kFormatGzip))
    return cudaErrorInvalidValue;
  DeviceScope scope(stream);
  CZ_TRY(scope.error());
  DeviceState* dev = nullptr;
  CZ_TRY(device_state(scope.device(), &dev));
  // compress()'s order: output bound, zero, input and chunk bounds.
  const u64 wrap = wrapper_bytes(format);
  if (capacity > kMaxStreamBytes + 5 * stored_blocks(kMaxStreamBytes) + wrap)
    return set_meta(meta, 0, kInvalidBounds, stream);
  if (capacity) {
    if (!out) return cudaErrorInvalidValue;
    CZ_TRY(cudaMemsetAsync(out, 0, capacity, stream));
  }
  if (size > kMaxStreamBytes || !chunk_ok(chunk_bytes) || (size && !in))
    return set_meta(meta, 0, kInvalidBounds, stream);
  const u32 chunk = u32(chunk_bytes);
  const StreamLayout l = stream_layout(size, chunk);
  if (l.blocks > kMaxBlocks || capacity != l.capacity - 6 + wrap)
    return set_meta(meta, 0, kInvalidBounds, stream);
  std::vector<EncodeFile> files(1);
  files[0] = EncodeFile{0, size, 0, capacity, 0, u32(l.chunks), chunk,
                        format == kFormatRaw ? kEncodeRaw
                                             : format == kFormatGzip ? kEncodeGzip : 0u};
  if (format != kFormatGzip)
    return encode_files(*dev, in, size, files, chunk, u32(l.chunks), out, meta, stream, nullptr,
                        u32(level));
  Workspace ws(dev->pool, stream);
  u32 *parts = nullptr, *crc = nullptr;
  CZ_TRY(ws.allocate(&parts, std::max<u32>(1, crc_segments(size))));
  CZ_TRY(ws.allocate(&crc, 1));
  CZ_TRY(launch_crc32(in, size, parts, crc, dev->info, stream));
  CZ_TRY(encode_files(*dev, in, size, files, chunk, u32(l.chunks), out, meta, stream, nullptr,
                      u32(level)));
  CZ_TRY(launch_gzip_trailer(out, meta, crc, size, stream));
  return ws.release();
}

// A raw body or a gzip member decodes as the body of a zlib-framed copy in
// scratch (two header bytes before it, four after) with the Adler-32 check
// off; a gzip member then checks CRC-32 and ISIZE on the output.
cudaError_t decompress_format(const u8* in, u64 size, int32_t format, u64 header_bytes,
                              int64_t max_candidates, int64_t max_blocks, u8* out, u64 expected,
                              u32* meta, cudaStream_t stream) {
  if (format == kFormatZlib)
    return decompress(in, size, max_candidates, max_blocks, out, expected, meta, stream);
  if (!meta || (format != kFormatRaw && format != kFormatGzip)) return cudaErrorInvalidValue;
  DeviceScope scope(stream);
  CZ_TRY(scope.error());
  DeviceState* dev = nullptr;
  CZ_TRY(device_state(scope.device(), &dev));
  if (expected > kMaxStreamBytes) return set_meta(meta, kInvalidBounds, 0, stream);
  if (expected && !out) return cudaErrorInvalidValue;
  auto fail = [&](u32 status) -> cudaError_t {
    if (expected) CZ_TRY(cudaMemsetAsync(out, 0, expected, stream));
    return set_meta(meta, status, 0, stream);
  };
  const u64 wrap = wrapper_bytes(format);
  if (size > kMaxStreamInput - 6 + wrap) return fail(kInvalidBounds);
  u64 head = 0, body = size;
  if (format == kFormatGzip) {
    if (header_bytes < 10 || size < header_bytes + 8) return fail(kGzipHeader);
    head = header_bytes;
    body = size - header_bytes - 8;
  }
  // A complete Deflate body has at least two bytes (an empty fixed block).
  if (body < 2) return fail(kTruncated);
  if (!in) return cudaErrorInvalidValue;
  Workspace ws(dev->pool, stream);
  u8* view = nullptr;
  CZ_TRY(ws.allocate(&view, body + 6 + 64));
  CZ_TRY(cudaMemsetAsync(view, 0x78, 1, stream));
  CZ_TRY(cudaMemsetAsync(view + 1, 0x9c, 1, stream));
  CZ_TRY(cudaMemcpyAsync(view + 2, in + head, body, cudaMemcpyDeviceToDevice, stream));
  CZ_TRY(cudaMemsetAsync(view + 2 + body, 0, 4 + 64, stream));
  CZ_TRY(decompress(view, body + 6, max_candidates, max_blocks, out, expected, meta, stream,
                    false));
  if (format == kFormatGzip) {
    u32 *parts = nullptr, *crc = nullptr;
    CZ_TRY(ws.allocate(&parts, std::max<u32>(1, crc_segments(expected))));
    CZ_TRY(ws.allocate(&crc, 1));
    CZ_TRY(launch_crc32(out, expected, parts, crc, dev->info, stream));
    CZ_TRY(launch_gzip_check(in, size, expected, crc, meta, stream));
    CZ_TRY(launch_clear_on_failure(meta, out, expected, stream));
  }
  return ws.release();
}

cudaError_t decompress_batch(const u8* in, u64 in_bytes, const int64_t* in_sizes,
                             const int64_t* out_sizes, u64 count, const u32* encoded, u8* out,
                             u64 out_bytes, u32* meta, cudaStream_t stream) {
  // DecompressBatchImpl (codec_ffi.cu:1065-1107).
  if (!count || count > kMaxBlocks || !in_sizes || !out_sizes || !meta)
    return cudaErrorInvalidValue;
  if (in_bytes > kMaxBytes || out_bytes > kMaxBytes) return cudaErrorInvalidValue;
  std::vector<StreamDesc> descs(count);
  u64 in_extent = 0, out_extent = 0;
  for (u64 i = 0; i < count; ++i) {
    const int64_t size = in_sizes[i], want = out_sizes[i];
    if (size < 0 || want < 0 || size > int64_t(kMaxBytes) || want > int64_t(kMaxBytes) ||
        in_extent + u64(size) > kMaxBytes || out_extent + u64(want) > kMaxBytes)
      return cudaErrorInvalidValue;
    descs[i] = StreamDesc{in_extent, u64(size), out_extent, u64(want)};
    in_extent += u64(size);
    out_extent += u64(want);
  }
  if (in_extent != in_bytes || out_extent != out_bytes) return cudaErrorInvalidValue;
  if ((in_bytes && !in) || (out_bytes && !out)) return cudaErrorInvalidValue;
  // Costliest streams first, so the last ones a warp picks up are short.
  // Decode time grows with the Huffman symbols read (about the input bytes)
  // and, more slowly, with the bytes written; a stream whose input is not
  // smaller than its output is stored, a copy.  Fitted to 64 KiB text,
  // run-length and random files: 11 in + out for coded streams, 2/3 out for
  // stored ones.
  auto cost = [&](u32 i) -> u64 {
    const StreamDesc& d = descs[i];
    return d.in_size < d.out_size ? 11 * d.in_size + d.out_size : 2 * d.out_size / 3;
  };
  std::vector<u32> order(count);
  std::iota(order.begin(), order.end(), 0u);
  std::stable_sort(order.begin(), order.end(), [&](u32 a, u32 b) { return cost(a) > cost(b); });
  DeviceScope scope(stream);
  CZ_TRY(scope.error());
  DeviceState* dev = nullptr;
  CZ_TRY(device_state(scope.device(), &dev));
  Workspace ws(dev->pool, stream);
  StreamDesc* d_descs = nullptr;
  u32 *d_order = nullptr, *counter = nullptr;
  CZ_TRY(upload(*dev, ws, &d_descs, descs, stream));
  CZ_TRY(upload(*dev, ws, &d_order, order, stream));
  CZ_TRY(ws.allocate(&counter, 1));
  CZ_TRY(cudaMemsetAsync(counter, 0, sizeof(u32), stream));
  CZ_TRY(launch_serial_inflate(in, out, d_descs, descs[0], u32(count), d_order, counter, meta,
                               encoded, kMaxBlocks, dev->info, stream));
  return ws.release();
}

cudaError_t inspect_pools(int device, u64* stats, bool trim) {
  Registry& r = registry();
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lock(r.mutex);
    stats[0] = r.retention;
    stats[1] = stats[2] = stats[3] = 0;
    if (device >= 0 && device < kMaxDevices && r.devices[device].ready)
      pool = r.devices[device].pool;
  }
  if (!pool) return cudaSuccess;
  if (trim) CZ_TRY(cudaMemPoolTrimTo(pool, 0));
  u64 reserved = 0, used = 0;
  CZ_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &reserved));
  CZ_TRY(cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, &used));
  stats[1] = reserved;
  stats[2] = used;
  stats[3] = 1;
  return cudaSuccess;
}

}  // namespace
}  // namespace cz

extern "C" {

int cuda_zlib_compress(const uint8_t* input, uint64_t size, int64_t chunk_bytes, uint8_t* output,
                       uint64_t capacity, uint32_t* metadata, void* stream) {
  try {
    return int(cz::compress(input, size, chunk_bytes, output, capacity, metadata,
                            static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int cuda_zlib_compress_range(const uint8_t* input, uint64_t size, int64_t chunk_bytes,
                             int32_t last, uint8_t* output, uint64_t capacity, uint32_t* metadata,
                             void* stream) {
  try {
    return int(cz::compress_range(input, size, chunk_bytes, last, output, capacity, metadata,
                                  static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int cuda_zlib_decompress(const uint8_t* input, uint64_t size, int64_t max_candidates,
                         int64_t max_blocks, uint8_t* output, uint64_t expected,
                         uint32_t* metadata, void* stream) {
  try {
    return int(cz::decompress(input, size, max_candidates, max_blocks, output, expected, metadata,
                              static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int cuda_zlib_compress_format(const uint8_t* input, uint64_t size, int64_t chunk_bytes,
                              int32_t format, int32_t level, uint8_t* output, uint64_t capacity,
                              uint32_t* metadata, void* stream) {
  try {
    return int(cz::compress_format(input, size, chunk_bytes, format, level, output, capacity,
                                   metadata, static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int cuda_zlib_decompress_format(const uint8_t* input, uint64_t size, int32_t format,
                                uint64_t header_bytes, int64_t max_candidates,
                                int64_t max_blocks, uint8_t* output, uint64_t expected,
                                uint32_t* metadata, void* stream) {
  try {
    return int(cz::decompress_format(input, size, format, header_bytes, max_candidates,
                                     max_blocks, output, expected, metadata,
                                     static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int cuda_zlib_gzip_header(const uint8_t* bytes, uint64_t available, uint64_t* header_bytes) {
  if (!header_bytes) return int(cz::kGzipHeader);
  return int(cz::gzip_header(bytes, available, header_bytes));
}

int cuda_zlib_compress_batch(const uint8_t* input, uint64_t input_bytes,
                             const int64_t* input_sizes, uint64_t files, int64_t chunk_bytes,
                             uint8_t* output, uint64_t output_bytes, uint32_t* metadata,
                             void* stream) {
  try {
    return int(cz::compress_batch(input, input_bytes, input_sizes, files, chunk_bytes, output,
                                  output_bytes, metadata, static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int cuda_zlib_compress_batch_packed(const uint8_t* input, uint64_t input_bytes,
                                    const int64_t* input_sizes, uint64_t files,
                                    int64_t chunk_bytes, uint8_t* output, uint64_t output_bytes,
                                    uint32_t* metadata, void* stream) {
  try {
    return int(cz::compress_batch(input, input_bytes, input_sizes, files, chunk_bytes, output,
                                  output_bytes, metadata, static_cast<cudaStream_t>(stream),
                                  true));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int cuda_zlib_decompress_batch(const uint8_t* input, uint64_t input_bytes,
                               const int64_t* input_sizes, const int64_t* output_sizes,
                               uint64_t files, const uint32_t* encoded_metadata, uint8_t* output,
                               uint64_t output_bytes, uint32_t* metadata, void* stream) {
  try {
    return int(cz::decompress_batch(input, input_bytes, input_sizes, output_sizes, files,
                                    encoded_metadata, output, output_bytes, metadata,
                                    static_cast<cudaStream_t>(stream)));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int CudaZlibSetWorkspaceRetention(uint64_t bytes) {
  cz::Registry& r = cz::registry();
  std::lock_guard<std::mutex> lock(r.mutex);
  if (r.pools_created) return int(cudaErrorInvalidValue);
  r.retention = bytes;
  return int(cudaSuccess);
}

int CudaZlibWorkspacePoolStats(int device, uint64_t* stats) {
  if (device < 0 || !stats) return int(cudaErrorInvalidValue);
  try {
    return int(cz::inspect_pools(device, stats, false));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

int CudaZlibTrimWorkspacePool(int device) {
  if (device < 0) return int(cudaErrorInvalidValue);
  try {
    uint64_t stats[4];
    return int(cz::inspect_pools(device, stats, true));
  } catch (...) {
    return int(cudaErrorUnknown);
  }
}

const char* cuda_zlib_b200_version(void) { return "0.1.0"; }

int cuda_zlib_b200_profile(int enable) {
  cz::Profiler& p = cz::profiler();
  std::lock_guard<std::mutex> lock(p.mutex);
  cudaError_t e = cz::profile_drain(p);
  p.totals.clear();
  p.enabled = enable != 0;
  // Spare events for the current device, made now rather than while timing.
  int device = 0;
  if (p.enabled && e == cudaSuccess && cudaGetDevice(&device) == cudaSuccess) {
    int have = 0;
    for (const auto& d : p.spare) have += d.first == device ? 1 : 0;
    for (; have < cz::kSpareEvents; ++have) {
      cudaEvent_t event = nullptr;
      e = cudaEventCreate(&event);
      if (e != cudaSuccess) break;
      p.spare.emplace_back(device, event);
    }
  }
  return int(e);
}

uint64_t cuda_zlib_b200_launches(void) {
  return cz::launches_issued.load(std::memory_order_relaxed);
}

int cuda_zlib_b200_profile_read(const char* kernel, double* total_ms, uint64_t* launches) {
  if (!kernel || !total_ms || !launches) return int(cudaErrorInvalidValue);
  cz::Profiler& p = cz::profiler();
  std::lock_guard<std::mutex> lock(p.mutex);
  cudaError_t e = cz::profile_drain(p);
  *total_ms = 0;
  *launches = 0;
  for (const cz::ProfileTotals& t : p.totals) {
    if (t.kernel == kernel) {
      *total_ms = t.ms;
      *launches = t.launches;
    }
  }
  return int(e);
}

}  // extern "C"
