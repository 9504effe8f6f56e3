// UnchainKV splitzip bf16 KV codec for B200 (sm_100a): host side + C ABI.
//
// Drop-in for native/unchain_kv/kvq_splitzip_cuda.cu of the reference: every
// kvq_splitzip_* entry point keeps the reference's name, argument order,
// argument meaning, decline rules (return 0), return values and error strings
// ("<Kernel>: <cudaGetErrorString>", return -1).  Streams are the caller's
// cudaStream_t; nothing is synchronised.  Extensions (fused gather, batches
// of calls, device-side mode choice) follow the same conventions.
//
// Stream formats (the reference's bytes, in canonical order):
//   top16 (mode 5): [0]=5|255, [1..4] u32 LE escape count, body n bytes
//     (mantissa7 | sign<<7), codes ceil(n/2) bytes (4-bit exponent codes, even
//     word in the low nibble), ceil(n/200) five-byte escape entries
//     {u32 LE position, u8 exponent} sorted by position, unused slots zero.
//   fixed6 (mode 3) / fixed5 (mode 4): [0]=3|4|255, 64/32-byte palette of
//     distinct high bytes in ascending order (zero padded), low-byte plane n
//     bytes, 6-bit codes 4->3 bytes LE / 5-bit codes 8->5 bytes LE.
//   raw (mode 6): [6] + the n words little endian.
// Kernels are in splitzip_kernels.cuh (codec) and splitzip_attention.cuh
// (decode attention over streams).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <atomic>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "splitzip_attention.cuh"
#include "splitzip_torchop.cuh"
#include "splitzip_kernels.cuh"
#include "unchain_kv_splitzip.h"

using namespace ukv;

namespace {

thread_local std::string g_last_error;

long long Fail(const char* what, cudaError_t status) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(status);
  return -1;
}

// ---------------------------------------------------------------- profiler
//
// When enabled, every kernel launch of this library is bracketed by two CUDA
// events recorded on the launching stream; kvq_splitzip_profile_collect()
// waits for them and sums device time and launch count per kernel name.
// The device-side analogue of the reference's UNCHAIN_KV_TRACE_CUDA event
// pairs (src/unchain_kv/vllm_connector.py:3100-3124).

struct ProfRecord {
  const char* name;
  cudaEvent_t begin;
  cudaEvent_t end;
};

std::mutex g_prof_mu;
std::atomic<bool> g_prof_on{false};
std::vector<ProfRecord> g_prof_pending;
std::vector<cudaEvent_t> g_prof_pool;
std::vector<std::string> g_prof_names;
std::vector<double> g_prof_ms;
std::vector<long long> g_prof_launches;

cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Records the begin event of a launch; returns its slot (or -1 when off).
long long prof_begin(cudaStream_t stream) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return -1;
  std::lock_guard<std::mutex> lock(g_prof_mu);
  ProfRecord r{nullptr, prof_event(), prof_event()};
  cudaEventRecord(r.begin, stream);
  g_prof_pending.push_back(r);
  return static_cast<long long>(g_prof_pending.size()) - 1;
}

void prof_end(long long slot, const char* name, cudaStream_t stream) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lock(g_prof_mu);
  if (slot >= static_cast<long long>(g_prof_pending.size())) return;
  g_prof_pending[slot].name = name;
  cudaEventRecord(g_prof_pending[slot].end, stream);
}

// ----------------------------------------------------------- launch sizing
//
// The kernels are persistent: the grid is the number of CTAs that fit on the
// device at once (occupancy x SMs), capped by the tile count.  Dynamic
// shared memory above 48 KiB is opted into once per kernel and device.

struct GeometryKey {
  const void* kernel;
  int device;
  bool operator<(const GeometryKey& o) const {
    return kernel < o.kernel || (kernel == o.kernel && device < o.device);
  }
};

std::mutex g_geometry_mu;
std::map<GeometryKey, int> g_geometry;  // resident CTAs per device

// Launch with programmatic stream serialization: the kernel may be scheduled
// while the previous kernel of the stream finishes; it waits for that
// kernel (grid_dependency_wait) before touching global memory.  Only
// kernels that call grid_dependency_sync() first go through here.
template <typename Kernel, typename... Args>
cudaError_t launch_dependent(Kernel kernel, dim3 grid, dim3 block, size_t dyn_smem, cudaStream_t stream,
                             const Args&... args) {
  cudaLaunchConfig_t config{};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = dyn_smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, args...);
}

template <typename Kernel>
long long grid_for(Kernel kernel, size_t dyn_smem, uint64_t tiles, unsigned* grid, int threads = kCtaThreads) {
  int device = 0;
  cudaError_t st = cudaGetDevice(&device);
  if (st != cudaSuccess) return Fail("cudaGetDevice", st);
  const GeometryKey key{reinterpret_cast<const void*>(kernel), device};
  int resident = 0;
  {
    std::lock_guard<std::mutex> lock(g_geometry_mu);
    auto it = g_geometry.find(key);
    if (it != g_geometry.end()) resident = it->second;
  }
  if (resident == 0) {
    st = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn_smem));
    if (st != cudaSuccess) return Fail("cudaFuncSetAttribute", st);
    int per_sm = 0, sms = 0;
    st = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, dyn_smem);
    if (st != cudaSuccess) return Fail("cudaOccupancyMaxActiveBlocksPerMultiprocessor", st);
    st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (st != cudaSuccess) return Fail("cudaDeviceGetAttribute", st);
    resident = std::max(1, per_sm) * std::max(1, sms);
    std::lock_guard<std::mutex> lock(g_geometry_mu);
    g_geometry[key] = resident;
  }
  *grid = static_cast<unsigned>(std::min<uint64_t>(tiles, static_cast<uint64_t>(resident)));
  if (*grid == 0) *grid = 1;
  return 0;
}

// ------------------------------------------------------------------ layouts

int log2_exact(uint64_t v) {
  if (v == 0 || (v & (v - 1))) return -1;
  int s = 0;
  while ((1ull << s) != v) ++s;
  return s;
}

Layout flat_layout(uint64_t n) {
  Layout L{};
  L.n = n;
  L.bw_shift = -1;
  return L;
}

Layout block_layout(uint64_t block_count, uint64_t block_words, uint64_t plane_stride,
                    uint64_t block_stride, uint64_t block_start, const int64_t* ids) {
  Layout L{};
  L.n = 2 * block_count * block_words;
  L.plane_words = block_count * block_words;
  L.block_words = block_words;
  L.plane_stride = plane_stride;
  L.block_stride = block_stride;
  L.block_start = block_start;
  L.ids = ids;
  L.bw_shift = log2_exact(block_words);
  return L;
}

// TMA bulk staging needs 16-byte aligned runs of whole 8-word groups.
bool bulk_ok(const void* base, const Layout& L) {
  if (reinterpret_cast<uintptr_t>(base) % 16) return false;
  if (L.block_words == 0) return true;
  return L.block_words % 8 == 0 && L.plane_stride % 8 == 0 && L.block_stride % 8 == 0;
}

// 16-byte vector stores of 16-word units into the paged cache.
bool vec_ok(const void* dst, const Layout& L) {
  return reinterpret_cast<uintptr_t>(dst) % 16 == 0 && L.block_words % 16 == 0 &&
         L.plane_stride % 8 == 0 && L.block_stride % 8 == 0;
}

uint64_t tiles_for(uint64_t n) { return (n + kTileWords - 1) / kTileWords; }
uint64_t top16_size(uint64_t n) { return 5 + n + (n + 1) / 2 + 5 * ((n + 199) / 200); }
uint64_t fixed_size(uint64_t n, int bits) {
  return bits == 5 ? 33 + n + ((n + 7) / 8) * 5 : 65 + n + ((n + 3) / 4) * 3;
}

// Offset of the first 16-byte aligned address at or after dst + offset.
uint64_t align16_from(const uint8_t* dst, uint64_t offset) {
  const uintptr_t end = reinterpret_cast<uintptr_t>(dst) + offset;
  return ((end + 15) & ~static_cast<uintptr_t>(15)) - reinterpret_cast<uintptr_t>(dst);
}

// ---------------------------------------------------------- job preparation

struct Prepared {
  EncJob job;
  uint8_t* zero_ptr;
  uint64_t zero_bytes;
  uint64_t result;
};

EncJob base_job(const uint16_t* src, const Layout& L, uint8_t* dst, const uint8_t* tables) {
  EncJob j{};
  j.src = src;
  j.L = L;
  j.dst = dst;
  j.n = L.n;
  j.half = L.n / 2;
  j.cap = (L.n + 199) / 200;
  j.tables = tables;
  j.tiles = static_cast<uint32_t>(tiles_for(L.n));
  j.bulk = bulk_ok(src, L);
  return j;
}

// top16: exactly the reference's rules (.cu:385-395).  The statistics pass
// keeps its per-tile counts inside the stream's own body region (and, for a
// last tile of fewer than 47 words, in the reference's 8 scratch bytes at
// align4(encoded)), so nothing else past the stream is needed and nothing
// is cleared beforehand; the encode kernel clears the unused escape slots.
bool prepare_top16(const uint16_t* src, const Layout& L, uint8_t* dst, uint64_t capacity,
                   const uint8_t* tables, Prepared& p) {
  const uint64_t n = L.n;
  if (!src || !dst || !tables || n == 0 || n > 0xFFFFFFFFULL) return false;
  const uint64_t encoded = top16_size(n);
  if (encoded >= n * 2 || ((encoded + 3) & ~3ULL) + 8 > capacity) return false;
  p.job = base_job(src, L, dst, tables);
  p.job.scratch = nullptr;
  p.zero_ptr = nullptr;
  p.zero_bytes = 0;
  p.result = encoded;
  return true;
}

// fixed6/fixed5: the reference's rules (.cu:298-306); the bitmap lives at
// the reference's scratch offset align4(encoded).
bool prepare_fixed(const uint16_t* src, const Layout& L, uint8_t* dst, uint64_t capacity, int bits,
                   Prepared& p) {
  const uint64_t n = L.n;
  if (!src || !dst || n == 0) return false;
  if (bits != 5 && bits != 6) return false;
  const uint64_t encoded = fixed_size(n, bits);
  const uint64_t so = (encoded + 3) & ~3ULL;
  if (encoded >= n * 2 || so + 256 * sizeof(int) + 2 * sizeof(int) > capacity) return false;
  if ((reinterpret_cast<uintptr_t>(dst) + so) % 4) return false;
  p.job = base_job(src, L, dst, nullptr);
  p.job.scratch = dst + so;
  p.job.error = reinterpret_cast<uint32_t*>(dst + so + 32);
  p.zero_ptr = dst + so;
  p.zero_bytes = kFixedScratchBytes;
  p.result = encoded;
  return true;
}

// auto: top16 if the escapes fit, else fixed6, else raw (if the buffer
// holds [6]+raw and the scratch after it), else a mode-255 stream.
bool prepare_auto(const uint16_t* src, const Layout& L, uint8_t* dst, uint64_t capacity,
                  const uint8_t* tables, Prepared& p) {
  const uint64_t n = L.n;
  if (!src || !dst || !tables || n == 0 || n > 0xFFFFFFFFULL) return false;
  if (top16_size(n) >= n * 2) return false;
  const uint64_t tiles = tiles_for(n);
  const uint64_t scratch = auto_scratch_bytes(tiles);
  const uint64_t compressed = std::max(top16_size(n), fixed_size(n, 6));
  const uint64_t raw_so = align16_from(dst, 1 + 2 * n);
  const uint64_t so = align16_from(dst, compressed);
  const bool raw_ok = raw_so + scratch <= capacity;
  if (!raw_ok && so + scratch > capacity) return false;
  p.job = base_job(src, L, dst, tables);
  p.job.raw_ok = raw_ok;
  p.job.scratch = dst + (raw_ok ? raw_so : so);
  p.job.error = reinterpret_cast<uint32_t*>(p.job.scratch + 4);
  p.zero_ptr = p.job.scratch;
  p.zero_bytes = scratch;  // totals, bitmap, group sums and tile counts start at zero
  p.result = raw_ok ? 1 + 2 * n : compressed;
  return true;
}

void prepare_decode(const uint8_t* src, uint64_t src_bytes, uint16_t* dst, const Layout& L,
                    const uint8_t* tables, DecJob& d) {
  d = DecJob{};
  d.src = src;
  d.src_bytes = src_bytes;
  d.dst = dst;
  d.L = L;
  d.n = L.n;
  d.half = L.n / 2;
  d.cap = (L.n + 199) / 200;
  d.tables = tables;
  d.tiles = static_cast<uint32_t>(tiles_for(L.n));
  d.vec = vec_ok(dst, L);
}

// ------------------------------------------------------------------ launch

enum class EncOp { kTop16, kTop16Scratch, kFixed6, kFixed5, kAuto };

template <int kMax>
long long launch_zero(const std::vector<Prepared>& jobs, size_t first, size_t count,
                      cudaStream_t stream) {
  if (count == 1) {
    const cudaError_t st = cudaMemsetAsync(jobs[first].zero_ptr, 0, jobs[first].zero_bytes, stream);
    return st == cudaSuccess ? 0 : Fail("cudaMemsetAsync", st);
  }
  ZeroBatch<kMax> z{};
  z.count = static_cast<uint32_t>(count);
  uint64_t largest = 0;
  for (size_t i = 0; i < count; ++i) {
    z.ptr[i] = jobs[first + i].zero_ptr;
    z.bytes[i] = jobs[first + i].zero_bytes;
    largest = std::max(largest, z.bytes[i]);
  }
  const unsigned bx =
      static_cast<unsigned>(std::min<uint64_t>(64, (largest / 16 + kThreads - 1) / kThreads + 1));
  const long long prof = prof_begin(stream);
  cudaError_t st = launch_dependent(ZeroKernel<kMax>, dim3(bx, static_cast<unsigned>(count)), dim3(kThreads), 0,
                                    stream, z);
  prof_end(prof, "ZeroKernel", stream);
  if (st == cudaSuccess) st = cudaGetLastError();
  return st == cudaSuccess ? 0 : Fail("ZeroKernel", st);
}

// Launch one persistent kernel over `tiles` tiles, bracketed by the profiler.
template <typename Kernel, typename Batch>
long long launch_persistent(Kernel kernel, const char* name, size_t dyn_smem, const Batch& b, uint64_t tiles,
                            cudaStream_t stream) {
  unsigned grid = 0;
  const long long rc = grid_for(kernel, dyn_smem, tiles, &grid);
  if (rc < 0) return rc;
  const long long prof = prof_begin(stream);
  cudaError_t st = launch_dependent(kernel, dim3(grid), dim3(kCtaThreads), dyn_smem, stream, b);
  prof_end(prof, name, stream);
  if (st == cudaSuccess) st = cudaGetLastError();
  return st == cudaSuccess ? 0 : Fail(name, st);
}

template <int kMax>
long long launch_encode_kernels(EncOp op, const EncBatch<kMax>& b, uint32_t tiles, cudaStream_t stream) {
  switch (op) {
    case EncOp::kTop16: {
      // escape counts of every tile into its record in the stream, their
      // scan per job (+ header), then the top16 streams at known offsets
      long long rc =
          launch_persistent(PresenceKernel<kMax, kStatsTop16Rec>, "Top16StatsKernel", kEncSmemBytes, b, tiles, stream);
      if (rc < 0) return rc;
      const long long prof = prof_begin(stream);
      cudaError_t st = launch_dependent(Top16ScanKernel<kMax>, dim3(b.jobs), dim3(kScanThreads), 0, stream, b);
      prof_end(prof, "Top16ScanKernel", stream);
      if (st == cudaSuccess) st = cudaGetLastError();
      if (st != cudaSuccess) return Fail("Top16ScanKernel", st);
      return launch_persistent(EncodeAutoKernel<kMax, kEncTop16Rec>, "EncodeTop16Kernel", kEncSmemBytes, b, tiles,
                               stream);
    }
    case EncOp::kTop16Scratch: {
      // escape counts of every tile into the scratch array, then the top16
      // streams at known offsets
      const long long rc =
          launch_persistent(PresenceKernel<kMax, kStatsTop16>, "Top16StatsKernel", kEncSmemBytes, b, tiles, stream);
      if (rc < 0) return rc;
      return launch_persistent(EncodeAutoKernel<kMax, kEncTop16Scratch>, "EncodeTop16Kernel", kEncSmemBytes, b,
                               tiles, stream);
    }
    case EncOp::kFixed6:
    case EncOp::kFixed5: {
      const long long rc =
          launch_persistent(PresenceKernel<kMax, kStatsPresence>, "PresenceKernel", kEncSmemBytes, b, tiles, stream);
      if (rc < 0) return rc;
      return op == EncOp::kFixed6
                 ? launch_persistent(EncodeFixedKernel<kMax, 6>, "EncodeFixed6Kernel", kEncSmemBytes, b, tiles, stream)
                 : launch_persistent(EncodeFixedKernel<kMax, 5>, "EncodeFixed5Kernel", kEncSmemBytes, b, tiles, stream);
    }
    case EncOp::kAuto: {
      const long long rc =
          launch_persistent(PresenceKernel<kMax, kStatsAuto>, "StatsKernel", kEncSmemBytes, b, tiles, stream);
      if (rc < 0) return rc;
      return launch_persistent(EncodeAutoKernel<kMax, kEncAuto>, "EncodeAutoKernel", kEncSmemBytes, b, tiles, stream);
    }
  }
  return 0;
}

template <int kMax>
long long launch_encode(EncOp op, const std::vector<Prepared>& jobs, size_t first, size_t count,
                        cudaStream_t stream) {
  if (op != EncOp::kTop16) {  // the top16 encode keeps no scratch to clear
    const long long rc = launch_zero<kMax>(jobs, first, count, stream);
    if (rc < 0) return rc;
  }
  EncBatch<kMax> b{};
  b.jobs = static_cast<uint32_t>(count);
  uint32_t tiles = 0;
  for (size_t i = 0; i < count; ++i) {
    b.tile_start[i] = tiles;
    b.job[i] = jobs[first + i].job;
    tiles += b.job[i].tiles;
  }
  b.tile_start[count] = tiles;
  return launch_encode_kernels(op, b, tiles, stream);
}

long long run_encode(EncOp op, const std::vector<Prepared>& jobs, cudaStream_t stream) {
  long long total = 0;
  for (const Prepared& p : jobs) total += static_cast<long long>(p.result);
  if (jobs.size() == 1) {
    const long long rc = launch_encode<1>(op, jobs, 0, 1, stream);
    return rc < 0 ? rc : total;
  }
  for (size_t first = 0; first < jobs.size(); first += kMaxBatch) {
    const size_t count = std::min<size_t>(kMaxBatch, jobs.size() - first);
    const long long rc = launch_encode<kMaxBatch>(op, jobs, first, count, stream);
    if (rc < 0) return rc;
  }
  return total;
}

template <int kMax, int kMode>
long long launch_decode(const std::vector<DecJob>& jobs, size_t first, size_t count,
                        cudaStream_t stream) {
  DecBatch<kMax> b{};
  b.jobs = static_cast<uint32_t>(count);
  uint32_t tiles = 0;
  for (size_t i = 0; i < count; ++i) {
    b.tile_start[i] = tiles;
    b.job[i] = jobs[first + i];
    tiles += b.job[i].tiles;
  }
  b.tile_start[count] = tiles;
  const char* name =
      kMode == 5 ? "DecodeTop16Kernel" : kMode == 3 ? "DecodeFixed6Kernel" : "DecodeAutoKernel";
  const long long rc = launch_persistent(DecodeKernel<kMax, kMode>, name, kDecCtaSmemBytes, b, tiles, stream);
  if constexpr (kMode == 3) {
    return rc;
  } else {
    if (rc < 0) return rc;
    // the escaped words of the top16 streams: grid rows are the jobs (all
    // patched at once), each row striding over its job's entries; the grid
    // holds about 8 CTAs per SM in all, so a batch without top16 streams
    // (each CTA reads one mode byte) costs one short wave
    static thread_local PatchBatch<kMax> pb;
    pb.jobs = b.jobs;
    uint64_t entries = 0;
    for (size_t i = 0; i < count; ++i) {
      pb.job[i] = b.job[i];
      entries = std::max<uint64_t>(entries, b.job[i].cap);
    }
    int device = 0, sms = 0;
    cudaError_t st = cudaGetDevice(&device);
    if (st == cudaSuccess) st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (st != cudaSuccess) return Fail("cudaDeviceGetAttribute", st);
    const uint64_t per_row = std::max<uint64_t>(1, static_cast<uint64_t>(sms) * 8 / std::max<uint32_t>(1, b.jobs));
    const uint64_t blocks = std::max<uint64_t>(1, std::min<uint64_t>((entries + 255) / 256, per_row));
    const long long prof = prof_begin(stream);
    st = launch_dependent(EscapePatchKernel<kMax, kMode>, dim3(static_cast<unsigned>(blocks), b.jobs), dim3(256), 0,
                          stream, pb);
    prof_end(prof, "EscapePatchKernel", stream);
    if (st == cudaSuccess) st = cudaGetLastError();
    return st == cudaSuccess ? 0 : Fail("EscapePatchKernel", st);
  }
}

template <int kMode>
long long run_decode(const std::vector<DecJob>& jobs, cudaStream_t stream) {
  long long total = 0;
  for (const DecJob& d : jobs) total += static_cast<long long>(d.n * sizeof(uint16_t));
  if (jobs.size() == 1) {
    const long long rc = launch_decode<1, kMode>(jobs, 0, 1, stream);
    return rc < 0 ? rc : total;
  }
  for (size_t first = 0; first < jobs.size(); first += kMaxBatch) {
    const size_t count = std::min<size_t>(kMaxBatch, jobs.size() - first);
    const long long rc = launch_decode<kMaxBatch, kMode>(jobs, first, count, stream);
    if (rc < 0) return rc;
  }
  return total;
}

Layout job_layout(const kvq_splitzip_job& j) {
  return block_layout(j.block_count, j.block_words, j.plane_stride, j.block_stride, j.block_start,
                      reinterpret_cast<const int64_t*>(j.block_ids_ptr));
}

bool job_shape_ok(const kvq_splitzip_job& j) {
  return j.cache_ptr != 0 && j.stream_ptr != 0 && j.block_count != 0 && j.block_words != 0;
}

long long encode_batch(EncOp op, const kvq_splitzip_job* jobs, unsigned long long count,
                       cudaStream_t stream) {
  if (!jobs || count == 0) return 0;
  std::vector<Prepared> prepared(count);
  for (unsigned long long i = 0; i < count; ++i) {
    const kvq_splitzip_job& j = jobs[i];
    if (!job_shape_ok(j)) return 0;
    const Layout L = job_layout(j);
    const auto* src = reinterpret_cast<const uint16_t*>(j.cache_ptr);
    auto* dst = reinterpret_cast<uint8_t*>(j.stream_ptr);
    const auto* tables = reinterpret_cast<const uint8_t*>(j.tables_ptr);
    bool ok = false;
    switch (op) {
      case EncOp::kTop16: ok = prepare_top16(src, L, dst, j.stream_bytes, tables, prepared[i]); break;
      case EncOp::kFixed6: ok = prepare_fixed(src, L, dst, j.stream_bytes, 6, prepared[i]); break;
      case EncOp::kFixed5: ok = prepare_fixed(src, L, dst, j.stream_bytes, 5, prepared[i]); break;
      case EncOp::kAuto: ok = prepare_auto(src, L, dst, j.stream_bytes, tables, prepared[i]); break;
    }
    if (!ok) return 0;
  }
  return run_encode(op, prepared, stream);
}

template <int kMode>
long long decode_batch(const kvq_splitzip_job* jobs, unsigned long long count, cudaStream_t stream) {
  if (!jobs || count == 0) return 0;
  std::vector<DecJob> prepared(count);
  for (unsigned long long i = 0; i < count; ++i) {
    const kvq_splitzip_job& j = jobs[i];
    if (!job_shape_ok(j)) return 0;
    if (kMode != 3 && j.tables_ptr == 0) return 0;
    const Layout L = job_layout(j);
    const uint64_t n = L.n;
    if (kMode == 5 && j.stream_bytes != top16_size(n)) return 0;
    if (kMode == 3 && j.stream_bytes != fixed_size(n, 6)) return 0;
    if (kMode == 0 && j.stream_bytes < std::min(top16_size(n), fixed_size(n, 6))) return 0;
    prepare_decode(reinterpret_cast<const uint8_t*>(j.stream_ptr), j.stream_bytes,
                   reinterpret_cast<uint16_t*>(j.cache_ptr), L,
                   reinterpret_cast<const uint8_t*>(j.tables_ptr), prepared[i]);
  }
  return run_decode<kMode>(prepared, stream);
}

}  // namespace

// =====================================================================
// C ABI (names, argument order and return conventions of the reference,
// native/unchain_kv/kvq_splitzip_cuda.cu:288-463)
// =====================================================================

extern "C" KVQ_API const char* kvq_splitzip_last_error() { return g_last_error.c_str(); }

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_mode(unsigned long long src_ptr,
                                                           unsigned long long dst_ptr,
                                                           unsigned long long count,
                                                           unsigned long long capacity,
                                                           unsigned long long stream_ptr, int bits) {
  if (src_ptr == 0 || dst_ptr == 0 || count == 0) return 0;
  if (bits != 5 && bits != 6) return 0;
  std::vector<Prepared> p(1);
  if (!prepare_fixed(reinterpret_cast<const uint16_t*>(src_ptr), flat_layout(count),
                     reinterpret_cast<uint8_t*>(dst_ptr), capacity, bits, p[0]))
    return 0;
  return run_encode(bits == 5 ? EncOp::kFixed5 : EncOp::kFixed6, p,
                    reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_encode(unsigned long long src_ptr,
                                                      unsigned long long dst_ptr,
                                                      unsigned long long count,
                                                      unsigned long long capacity,
                                                      unsigned long long stream_ptr) {
  return kvq_splitzip_bf16_encode_mode(src_ptr, dst_ptr, count, capacity, stream_ptr, 6);
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_fixed6_blocks(
    unsigned long long src_ptr, unsigned long long encoded_bytes, unsigned long long dst_ptr,
    unsigned long long count_words, unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride, unsigned long long block_start,
    unsigned long long block_ids_ptr, unsigned long long stream_ptr) {
  if (src_ptr == 0 || dst_ptr == 0 || count_words == 0 || block_count == 0 || block_words == 0 ||
      count_words != 2 * block_count * block_words) {
    return 0;
  }
  if (encoded_bytes != fixed_size(count_words, 6)) return 0;
  std::vector<DecJob> d(1);
  prepare_decode(reinterpret_cast<const uint8_t*>(src_ptr), encoded_bytes,
                 reinterpret_cast<uint16_t*>(dst_ptr),
                 block_layout(block_count, block_words, plane_stride, block_stride, block_start,
                              reinterpret_cast<const int64_t*>(block_ids_ptr)),
                 nullptr, d[0]);
  return run_decode<3>(d, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_fixed6(
    unsigned long long src_ptr, unsigned long long encoded_bytes, unsigned long long dst_ptr,
    unsigned long long count_words, unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride, unsigned long long block_start,
    unsigned long long stream_ptr) {
  return kvq_splitzip_bf16_decode_fixed6_blocks(src_ptr, encoded_bytes, dst_ptr, count_words,
                                                block_count, block_words, plane_stride, block_stride,
                                                block_start, 0, stream_ptr);
}

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_top16(unsigned long long src_ptr,
                                                            unsigned long long dst_ptr,
                                                            unsigned long long count,
                                                            unsigned long long capacity,
                                                            unsigned long long tables_ptr,
                                                            unsigned long long stream_ptr) {
  if (src_ptr == 0 || dst_ptr == 0 || tables_ptr == 0 || count == 0 || count > 0xFFFFFFFFULL) {
    return 0;
  }
  std::vector<Prepared> p(1);
  if (!prepare_top16(reinterpret_cast<const uint16_t*>(src_ptr), flat_layout(count),
                     reinterpret_cast<uint8_t*>(dst_ptr), capacity,
                     reinterpret_cast<const uint8_t*>(tables_ptr), p[0]))
    return 0;
  return run_encode(EncOp::kTop16, p, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_top16_blocks(
    unsigned long long src_ptr, unsigned long long encoded_bytes, unsigned long long dst_ptr,
    unsigned long long count_words, unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride, unsigned long long block_start,
    unsigned long long block_ids_ptr, unsigned long long tables_ptr, unsigned long long stream_ptr) {
  if (src_ptr == 0 || dst_ptr == 0 || tables_ptr == 0 || count_words == 0 || block_count == 0 ||
      block_words == 0 || count_words != 2 * block_count * block_words) {
    return 0;
  }
  if (encoded_bytes != top16_size(count_words)) return 0;
  std::vector<DecJob> d(1);
  prepare_decode(reinterpret_cast<const uint8_t*>(src_ptr), encoded_bytes,
                 reinterpret_cast<uint16_t*>(dst_ptr),
                 block_layout(block_count, block_words, plane_stride, block_stride, block_start,
                              reinterpret_cast<const int64_t*>(block_ids_ptr)),
                 reinterpret_cast<const uint8_t*>(tables_ptr), d[0]);
  return run_decode<5>(d, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_top16(
    unsigned long long src_ptr, unsigned long long encoded_bytes, unsigned long long dst_ptr,
    unsigned long long count_words, unsigned long long block_count, unsigned long long block_words,
    unsigned long long plane_stride, unsigned long long block_stride, unsigned long long block_start,
    unsigned long long tables_ptr, unsigned long long stream_ptr) {
  return kvq_splitzip_bf16_decode_top16_blocks(src_ptr, encoded_bytes, dst_ptr, count_words,
                                               block_count, block_words, plane_stride, block_stride,
                                               block_start, 0, tables_ptr, stream_ptr);
}

// ---------------------------------------------------------------------
// Extensions (no counterpart in the reference ABI; same conventions)
// ---------------------------------------------------------------------

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_top16_blocks(
    unsigned long long cache_ptr, unsigned long long plane_stride, unsigned long long block_stride,
    unsigned long long block_words, unsigned long long block_ids_ptr, unsigned long long block_start,
    unsigned long long block_count, unsigned long long dst_ptr, unsigned long long capacity,
    unsigned long long tables_ptr, unsigned long long stream_ptr) {
  const kvq_splitzip_job job{cache_ptr, plane_stride, block_stride, block_words, block_ids_ptr,
                             block_start, block_count, dst_ptr, capacity, tables_ptr};
  return encode_batch(EncOp::kTop16, &job, 1, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_mode_blocks(
    unsigned long long cache_ptr, unsigned long long plane_stride, unsigned long long block_stride,
    unsigned long long block_words, unsigned long long block_ids_ptr, unsigned long long block_start,
    unsigned long long block_count, unsigned long long dst_ptr, unsigned long long capacity,
    unsigned long long stream_ptr, int bits) {
  if (bits != 5 && bits != 6) return 0;
  const kvq_splitzip_job job{cache_ptr, plane_stride, block_stride, block_words, block_ids_ptr,
                             block_start, block_count, dst_ptr, capacity, 0};
  return encode_batch(bits == 5 ? EncOp::kFixed5 : EncOp::kFixed6, &job, 1,
                      reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_top16_batch(const kvq_splitzip_job* jobs,
                                                                  unsigned long long count,
                                                                  unsigned long long stream_ptr) {
  return encode_batch(EncOp::kTop16, jobs, count, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_mode_batch(const kvq_splitzip_job* jobs,
                                                                 unsigned long long count,
                                                                 unsigned long long stream_ptr,
                                                                 int bits) {
  if (bits != 5 && bits != 6) return 0;
  return encode_batch(bits == 5 ? EncOp::kFixed5 : EncOp::kFixed6, jobs, count,
                      reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_auto_batch(const kvq_splitzip_job* jobs,
                                                                 unsigned long long count,
                                                                 unsigned long long stream_ptr) {
  return encode_batch(EncOp::kAuto, jobs, count, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_top16_batch(const kvq_splitzip_job* jobs,
                                                                  unsigned long long count,
                                                                  unsigned long long stream_ptr) {
  return decode_batch<5>(jobs, count, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_fixed6_batch(const kvq_splitzip_job* jobs,
                                                                   unsigned long long count,
                                                                   unsigned long long stream_ptr) {
  return decode_batch<3>(jobs, count, reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_auto_batch(const kvq_splitzip_job* jobs,
                                                                 unsigned long long count,
                                                                 unsigned long long stream_ptr) {
  return decode_batch<0>(jobs, count, reinterpret_cast<cudaStream_t>(stream_ptr));
}

// ---------------------------------------------------------- peer streams
//
// Host plumbing of the GPU-to-GPU stream transport: stream buffers the
// sender allocates here (whole cudaMalloc allocations, so an IPC handle
// covers them from offset 0) are opened by the receiving process on its own
// device with lazy peer access, and its decode kernels read the streams
// straight from the sender's HBM over NVLink.

extern "C" KVQ_API unsigned long long kvq_splitzip_ipc_alloc(unsigned long long bytes) {
  void* p = nullptr;
  const cudaError_t st = cudaMalloc(&p, bytes);
  if (st != cudaSuccess) {
    Fail("cudaMalloc", st);
    return 0;
  }
  return reinterpret_cast<unsigned long long>(p);
}

extern "C" KVQ_API long long kvq_splitzip_ipc_free(unsigned long long ptr) {
  const cudaError_t st = cudaFree(reinterpret_cast<void*>(ptr));
  return st == cudaSuccess ? 0 : Fail("cudaFree", st);
}

// The 64-byte IPC handle of an allocation made by kvq_splitzip_ipc_alloc.
extern "C" KVQ_API long long kvq_splitzip_ipc_get_handle(unsigned long long ptr, unsigned char* handle64) {
  if (ptr == 0 || handle64 == nullptr) return 0;
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == 64, "IPC handle size");
  const cudaError_t st = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr));
  if (st != cudaSuccess) return Fail("cudaIpcGetMemHandle", st);
  std::memcpy(handle64, &h, sizeof(h));
  return 64;
}

// Open another process's allocation on the current device (peer access
// enabled lazily); returns its address here, 0 on failure.
extern "C" KVQ_API unsigned long long kvq_splitzip_ipc_open(const unsigned char* handle64) {
  if (handle64 == nullptr) return 0;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  const cudaError_t st = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (st != cudaSuccess) {
    Fail("cudaIpcOpenMemHandle", st);
    return 0;
  }
  return reinterpret_cast<unsigned long long>(p);
}

extern "C" KVQ_API long long kvq_splitzip_ipc_close(unsigned long long ptr) {
  const cudaError_t st = cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
  return st == cudaSuccess ? 0 : Fail("cudaIpcCloseMemHandle", st);
}

// 1 when the current device can read `peer_device`'s memory directly.
extern "C" KVQ_API long long kvq_splitzip_peer_access(long long peer_device) {
  int device = 0, ok = 0;
  cudaError_t st = cudaGetDevice(&device);
  if (st == cudaSuccess) st = cudaDeviceCanAccessPeer(&ok, device, static_cast<int>(peer_device));
  if (st != cudaSuccess) return Fail("cudaDeviceCanAccessPeer", st);
  return ok ? 1 : 0;
}

// -------------------------------------------------------------- writeback

namespace {

template <int kMax>
long long launch_writeback(const std::vector<WritebackJob>& jobs, size_t first, size_t count, cudaStream_t stream) {
  static thread_local WritebackBatch<kMax> b;
  b.jobs = static_cast<uint32_t>(count);
  uint64_t chunks = 0;
  for (size_t i = 0; i < count; ++i) {
    b.chunk_start[i] = chunks;
    b.job[i] = jobs[first + i];
    chunks += b.job[i].chunks;
  }
  b.chunk_start[count] = chunks;
  int device = 0, sms = 0;
  cudaError_t st = cudaGetDevice(&device);
  if (st == cudaSuccess) st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (st != cudaSuccess) return Fail("cudaDeviceGetAttribute", st);
  const uint64_t blocks = std::max<uint64_t>(1, std::min<uint64_t>((chunks + 255) / 256, static_cast<uint64_t>(sms) * 8));
  const long long prof = prof_begin(stream);
  WritebackKernel<kMax><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(b);
  prof_end(prof, "WritebackKernel", stream);
  st = cudaGetLastError();
  return st == cudaSuccess ? 0 : Fail("WritebackKernel", st);
}

}  // namespace

extern "C" KVQ_API long long kvq_splitzip_writeback_batch(const kvq_splitzip_job* jobs, unsigned long long count,
                                                          unsigned long long stream_ptr) {
  if (!jobs || count == 0) return 0;
  const auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  std::vector<WritebackJob> prepared(count);
  long long total = 0;
  for (unsigned long long i = 0; i < count; ++i) {
    const kvq_splitzip_job& j = jobs[i];
    // one contiguous run of whole, adjacent blocks (the reference skips
    // fragmented or non-contiguous segments), and a stream that fits them
    // and does not overlap them
    if (!job_shape_ok(j) || j.block_ids_ptr != 0 || j.block_stride != j.block_words || j.stream_bytes == 0)
      return 0;
    auto* cache = reinterpret_cast<uint8_t*>(j.cache_ptr);
    const uint64_t seg_bytes = 2 * j.block_count * j.block_words;
    if (j.stream_bytes > 2 * seg_bytes) return 0;
    WritebackJob& w = prepared[i];
    w.src = reinterpret_cast<const uint8_t*>(j.stream_ptr);
    w.bytes = j.stream_bytes;
    w.seg[0] = cache + 2 * j.block_start * j.block_stride;
    w.seg[1] = w.seg[0] + 2 * j.plane_stride;
    w.seg_bytes = seg_bytes;
    w.chunks = (w.bytes + 15) / 16;
    for (int s = 0; s < 2; ++s) {
      const uintptr_t a = reinterpret_cast<uintptr_t>(w.seg[s]), e = a + seg_bytes;
      const uintptr_t sa = reinterpret_cast<uintptr_t>(w.src), se = sa + w.bytes;
      if (sa < e && a < se) return 0;  // the stream aliases the blocks
    }
    w.vec = (reinterpret_cast<uintptr_t>(w.src) % 16 == 0 && reinterpret_cast<uintptr_t>(w.seg[0]) % 16 == 0 &&
             reinterpret_cast<uintptr_t>(w.seg[1]) % 16 == 0 && seg_bytes % 16 == 0)
                ? 1
                : 0;
    total += static_cast<long long>(w.bytes);
  }
  for (size_t first = 0; first < count; first += kMaxBatch) {
    const long long rc = launch_writeback<kMaxBatch>(prepared, first, std::min<size_t>(kMaxBatch, count - first), stream);
    if (rc < 0) return rc;
  }
  return total;
}

// --------------------------------------------------- torch-op encoder

namespace {

template <int kMax>
long long launch_torchop(const std::vector<Prepared>& jobs, size_t first, size_t count, cudaStream_t stream) {
  long long rc = launch_zero<kMax>(jobs, first, count, stream);
  if (rc < 0) return rc;
  EncBatch<kMax> e{};
  e.jobs = static_cast<uint32_t>(count);
  uint32_t tiles = 0;
  for (size_t i = 0; i < count; ++i) {
    e.tile_start[i] = tiles;
    e.job[i] = jobs[first + i].job;
    tiles += e.job[i].tiles;
  }
  e.tile_start[count] = tiles;
  rc = launch_persistent(TorchopStatsKernel<kMax>, "TorchopStatsKernel", kEncSmemBytes, e, tiles, stream);
  if (rc < 0) return rc;
  long long prof = prof_begin(stream);
  TorchopDecideKernel<kMax><<<static_cast<unsigned>(count), 32, 0, stream>>>(e);
  prof_end(prof, "TorchopDecideKernel", stream);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return Fail("TorchopDecideKernel", st);
  static thread_local TorchopBatch<kMax> b;
  b.jobs = e.jobs;
  uint64_t units = 0;
  for (size_t i = 0; i < count; ++i) {
    b.unit_start[i] = units;
    b.job[i] = e.job[i];
    b.vec[i] = vec_ok(e.job[i].src, e.job[i].L) ? 1 : 0;
    // whole warps per job: a warp's units store one run of each plane
    units += ((e.job[i].n + kUnitWords - 1) / kUnitWords + 31) / 32 * 32;
  }
  b.unit_start[count] = units;
  int device = 0, sms = 0;
  st = cudaGetDevice(&device);
  if (st == cudaSuccess) st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (st != cudaSuccess) return Fail("cudaDeviceGetAttribute", st);
  const uint64_t blocks = std::max<uint64_t>(1, std::min<uint64_t>((units + 255) / 256, static_cast<uint64_t>(sms) * 8));
  prof = prof_begin(stream);
  TorchopEncodeKernel<kMax><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(b);
  prof_end(prof, "TorchopEncodeKernel", stream);
  st = cudaGetLastError();
  return st == cudaSuccess ? 0 : Fail("TorchopEncodeKernel", st);
}

}  // namespace

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_torchop_batch(const kvq_splitzip_job* jobs,
                                                                    unsigned long long count,
                                                                    unsigned long long stream_ptr) {
  if (!jobs || count == 0) return 0;
  const auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  std::vector<Prepared> prepared(count);
  long long total = 0;
  for (unsigned long long i = 0; i < count; ++i) {
    const kvq_splitzip_job& j = jobs[i];
    if (!job_shape_ok(j)) return 0;
    const Layout L = job_layout(j);
    auto* dst = reinterpret_cast<uint8_t*>(j.stream_ptr);
    const uint64_t n = L.n;
    if (n == 0 || n > 0xFFFFFFFFULL) return 0;
    const uint64_t so = align16_from(dst, 1 + 2 * n);
    if (so + kTorchopScratch > j.stream_bytes) return 0;
    Prepared& p = prepared[i];
    p.job = base_job(reinterpret_cast<const uint16_t*>(j.cache_ptr), L, dst, nullptr);
    p.job.scratch = dst + so;
    p.zero_ptr = p.job.scratch;
    p.zero_bytes = kTorchopScratch;
    p.result = 1 + 2 * n;
    total += static_cast<long long>(p.result);
  }
  if (count == 1) {
    const long long rc = launch_torchop<1>(prepared, 0, 1, stream);
    return rc < 0 ? rc : total;
  }
  for (size_t first = 0; first < count; first += kMaxBatch) {
    const long long rc = launch_torchop<kMaxBatch>(prepared, first, std::min<size_t>(kMaxBatch, count - first), stream);
    if (rc < 0) return rc;
  }
  return total;
}

// ------------------------------------------------- every receiver mode

namespace {

template <int kMax>
long long launch_modes(const std::vector<DecJob>& jobs, size_t first, size_t count, cudaStream_t stream) {
  static thread_local ModeBatch<kMax> b;
  b.jobs = static_cast<uint32_t>(count);
  uint64_t units = 0;
  for (size_t i = 0; i < count; ++i) {
    b.unit_start[i] = units;
    b.job[i] = jobs[first + i];
    // whole warps per job: a warp keeps one job's palette
    units += ((b.job[i].n + kUnitWords - 1) / kUnitWords + 31) / 32 * 32;
  }
  b.unit_start[count] = units;
  int device = 0, sms = 0;
  cudaError_t st = cudaGetDevice(&device);
  if (st == cudaSuccess) st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (st != cudaSuccess) return Fail("cudaDeviceGetAttribute", st);
  const uint64_t blocks = std::min<uint64_t>((units + 255) / 256, static_cast<uint64_t>(sms) * 8);
  const long long prof = prof_begin(stream);
  ModeDecodeKernel<kMax><<<static_cast<unsigned>(std::max<uint64_t>(blocks, 1)), 256, 0, stream>>>(b);
  prof_end(prof, "ModeDecodeKernel", stream);
  st = cudaGetLastError();
  return st == cudaSuccess ? 0 : Fail("ModeDecodeKernel", st);
}

}  // namespace

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_any_batch(const kvq_splitzip_job* jobs,
                                                                unsigned long long count,
                                                                unsigned long long stream_ptr) {
  if (!jobs || count == 0) return 0;
  const auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  std::vector<DecJob> prepared(count);
  for (unsigned long long i = 0; i < count; ++i) {
    const kvq_splitzip_job& j = jobs[i];
    if (!job_shape_ok(j) || j.tables_ptr == 0 || j.stream_bytes == 0) return 0;
    prepare_decode(reinterpret_cast<const uint8_t*>(j.stream_ptr), j.stream_bytes,
                   reinterpret_cast<uint16_t*>(j.cache_ptr), job_layout(j),
                   reinterpret_cast<const uint8_t*>(j.tables_ptr), prepared[i]);
  }
  // modes 5, 3 and 6 by the staged decoder, modes 0, 1, 2 and 4 by the unit
  // decoder; each leaves the other's streams alone
  const long long total = run_decode<0>(prepared, stream);
  if (total < 0) return total;
  for (size_t first = 0; first < prepared.size(); first += kMaxBatch) {
    const size_t n = std::min<size_t>(kMaxBatch, prepared.size() - first);
    const long long rc = n == 1 && prepared.size() == 1 ? launch_modes<1>(prepared, 0, 1, stream)
                                                         : launch_modes<kMaxBatch>(prepared, first, n, stream);
    if (rc < 0) return rc;
  }
  return total;
}

// -------------------------------------------------------------- calibration

namespace {

template <int kMax>
long long launch_histograms(const std::vector<EncJob>& jobs, size_t first, size_t count, cudaStream_t stream) {
  EncBatch<kMax> b{};
  b.jobs = static_cast<uint32_t>(count);
  uint32_t tiles = 0;
  for (size_t i = 0; i < count; ++i) {
    b.tile_start[i] = tiles;
    b.job[i] = jobs[first + i];
    tiles += b.job[i].tiles;
  }
  b.tile_start[count] = tiles;
  return launch_persistent(ExpHistogramKernel<kMax>, "ExpHistogramKernel", kEncSmemBytes, b, tiles, stream);
}

}  // namespace

extern "C" KVQ_API long long kvq_splitzip_bf16_exponent_histogram_batch(const kvq_splitzip_job* jobs,
                                                                       unsigned long long count,
                                                                       unsigned long long stream_ptr) {
  if (!jobs || count == 0) return 0;
  const auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  std::vector<EncJob> prepared(count);
  for (unsigned long long i = 0; i < count; ++i) {
    const kvq_splitzip_job& j = jobs[i];
    if (!job_shape_ok(j) || j.stream_bytes < 2048 || j.stream_ptr % 4) return 0;
    const Layout L = job_layout(j);
    if (L.n == 0 || L.n > 0xFFFFFFFFULL) return 0;
    prepared[i] = base_job(reinterpret_cast<const uint16_t*>(j.cache_ptr), L, reinterpret_cast<uint8_t*>(j.stream_ptr),
                           nullptr);
  }
  if (count == 1) {
    const long long rc = launch_histograms<1>(prepared, 0, 1, stream);
    return rc < 0 ? rc : 1;
  }
  for (size_t first = 0; first < count; first += kMaxBatch) {
    const long long rc = launch_histograms<kMaxBatch>(prepared, first, std::min<size_t>(kMaxBatch, count - first), stream);
    if (rc < 0) return rc;
  }
  return static_cast<long long>(count);
}

extern "C" KVQ_API long long kvq_splitzip_top16_tables_from_histograms(unsigned long long hist_ptr,
                                                                      unsigned long long layers,
                                                                      unsigned long long tables_ptr,
                                                                      unsigned long long observed_ptr,
                                                                      unsigned long long stream_ptr) {
  if (!hist_ptr || !tables_ptr || !observed_ptr || layers == 0 || layers > (1ULL << 20) || hist_ptr % 4 ||
      observed_ptr % 4)
    return 0;
  const auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  const long long prof = prof_begin(stream);
  Top16TablesKernel<<<static_cast<unsigned>(layers), 256, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(hist_ptr), static_cast<uint32_t>(layers), reinterpret_cast<uint8_t*>(tables_ptr),
      reinterpret_cast<uint32_t*>(observed_ptr));
  prof_end(prof, "Top16TablesKernel", stream);
  const cudaError_t st = cudaGetLastError();
  return st == cudaSuccess ? static_cast<long long>(layers) : Fail("Top16TablesKernel", st);
}

// ---------------------------------------------------------------- attention

namespace {

using AttnLaunch = AttnBatch<kAttnMaxReqs, kAttnMaxItems>;

// The blocks of all requests, in order, split evenly over the resident CTAs
// of the attention kernel; an item is one CTA's run of blocks of one
// request.  The batch is declined when a request is malformed.
bool plan_attention(const kvq_splitzip_attn_request* reqs, uint64_t count, uint64_t group, AttnLaunch& b,
                    uint64_t* workspace) {
  if (reqs == nullptr || count == 0 || count > kAttnMaxReqs || group == 0 || group > kAttnMaxGroup) return false;
  uint64_t total = 0;
  for (uint64_t r = 0; r < count; ++r) {
    const kvq_splitzip_attn_request& q = reqs[r];
    if (q.stream_ptr == 0 || q.q_ptr == 0 || q.out_ptr == 0 || q.blocks == 0 || q.blocks > (1u << 24)) return false;
    if (q.ctx_tokens == 0 || q.ctx_tokens > q.blocks * kAttnBlockTokens ||
        q.ctx_tokens <= (q.blocks - 1) * kAttnBlockTokens)
      return false;
    if (q.q_ptr % 4 || q.out_ptr % 8) return false;
    total += q.blocks;
  }
  unsigned grid = 0;
  bool top16 = false;
  for (uint64_t r = 0; r < count; ++r) top16 = top16 || reqs[r].tables_ptr != 0;
  const long long geometry =
      top16 ? grid_for(AttnKernel<kAttnMaxReqs, kAttnMaxItems, true>, kAttnSmemBytes, kAttnMaxCtas, &grid, kAttnThreads + 32)
            : grid_for(AttnKernel<kAttnMaxReqs, kAttnMaxItems, false>, kAttnSmemBytes, kAttnMaxCtas, &grid, kAttnThreads);
  if (geometry < 0) return false;
  const uint64_t ctas = std::min<uint64_t>(std::min<uint64_t>(grid, total), kAttnMaxCtas);
  b = AttnLaunch{};
  for (uint64_t r = 0; r < count; ++r) {
    const kvq_splitzip_attn_request& q = reqs[r];
    AttnReq& a = b.req[r];
    a.stream = reinterpret_cast<const uint8_t*>(q.stream_ptr);
    a.stream_bytes = q.stream_bytes;
    a.n = 2 * q.blocks * kAttnBlockWords;
    a.q = reinterpret_cast<const uint16_t*>(q.q_ptr);
    a.out = reinterpret_cast<uint16_t*>(q.out_ptr);
    a.tables = reinterpret_cast<const uint8_t*>(q.tables_ptr);
    a.ctx = static_cast<uint32_t>(q.ctx_tokens);
  }
  uint32_t items = 0;
  uint64_t r = 0, req_first = 0;  // request holding global block `at`, and its first global block
  for (uint64_t c = 0; c < ctas; ++c) {
    b.cta_item[c] = static_cast<uint16_t>(items);
    uint64_t at = total * c / ctas;
    const uint64_t end = total * (c + 1) / ctas;
    while (at < end) {
      while (at >= req_first + reqs[r].blocks) req_first += reqs[r++].blocks;
      const uint64_t stop = std::min<uint64_t>(end, req_first + reqs[r].blocks);
      if (items >= kAttnMaxItems) return false;
      b.item[items].req = static_cast<uint32_t>(r);
      b.item[items].block0 = static_cast<uint32_t>(at - req_first);
      b.item[items].blocks = static_cast<uint32_t>(stop - at);
      b.item[items].gblock0 = static_cast<uint32_t>(at);
      if (b.req[r].items == 0) b.req[r].first_item = items;
      ++b.req[r].items;
      ++items;
      at = stop;
    }
  }
  b.cta_item[ctas] = static_cast<uint16_t>(items);
  b.ctas = static_cast<uint32_t>(ctas);
  b.reqs = static_cast<uint32_t>(count);
  b.items = items;
  b.group = static_cast<uint32_t>(group);
  b.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kAttnHeadDim));
  // the items' partials, then (top16 batches) the blocks' scaled scores
  *workspace = 16 + static_cast<uint64_t>(items) * kAttnKvHeads * group * kAttnRecord * sizeof(float) +
               (top16 ? total * kAttnKvHeads * kAttnBlockTokens * group * sizeof(float) : 0);
  return true;
}

}  // namespace

extern "C" KVQ_API long long kvq_splitzip_attention_workspace_bytes(const kvq_splitzip_attn_request* reqs,
                                                                    unsigned long long count,
                                                                    unsigned long long group) {
  static thread_local AttnLaunch b;
  uint64_t ws = 0;
  return plan_attention(reqs, count, group, b, &ws) ? static_cast<long long>(ws) : 0;
}

extern "C" KVQ_API long long kvq_splitzip_attention_decode(const kvq_splitzip_attn_request* reqs,
                                                           unsigned long long count, unsigned long long group,
                                                           unsigned long long workspace_ptr,
                                                           unsigned long long workspace_bytes,
                                                           unsigned long long stream_ptr) {
  static thread_local AttnLaunch b;
  uint64_t ws = 0;
  if (!plan_attention(reqs, count, group, b, &ws) || workspace_ptr == 0 || workspace_ptr % 16 ||
      workspace_bytes < ws)
    return 0;
  const cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  b.partials = reinterpret_cast<float*>(workspace_ptr + 16);
  bool top16 = false;
  for (uint32_t r = 0; r < b.reqs; ++r) top16 = top16 || b.req[r].tables != nullptr;
  b.scores = top16 ? b.partials + static_cast<uint64_t>(b.items) * kAttnKvHeads * b.group * kAttnRecord : nullptr;
  long long prof = prof_begin(stream);
  if (top16) {
    // + the escape warp
    AttnKernel<kAttnMaxReqs, kAttnMaxItems, true><<<b.ctas, kAttnThreads + 32, kAttnSmemBytes, stream>>>(b);
  } else {
    AttnKernel<kAttnMaxReqs, kAttnMaxItems, false><<<b.ctas, kAttnThreads, kAttnSmemBytes, stream>>>(b);
  }
  prof_end(prof, "AttnKernel", stream);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return Fail("AttnKernel", st);
  if (top16) {  // the V escapes' shares of the top16 items' partials
    unsigned unused = 0;  // (sets the kernel's shared-memory limit once per device)
    if (grid_for(AttnEscapeKernel<kAttnMaxReqs, kAttnMaxItems>, kAttnEscSmem, b.items, &unused, kAttnEscThreads) < 0)
      return -1;
    prof = prof_begin(stream);
    AttnEscapeKernel<kAttnMaxReqs, kAttnMaxItems><<<b.items, kAttnEscThreads, kAttnEscSmem, stream>>>(b);
    prof_end(prof, "AttnEscapeKernel", stream);
    st = cudaGetLastError();
    if (st != cudaSuccess) return Fail("AttnEscapeKernel", st);
  }
  const uint64_t warps = static_cast<uint64_t>(b.reqs) * kAttnKvHeads * b.group;
  prof = prof_begin(stream);
  AttnCombineKernel<kAttnMaxReqs, kAttnMaxItems><<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(b);
  prof_end(prof, "AttnCombineKernel", stream);
  st = cudaGetLastError();
  if (st != cudaSuccess) return Fail("AttnCombineKernel", st);
  return static_cast<long long>(count);
}

extern "C" KVQ_API long long kvq_splitzip_device_errors() {
  unsigned int value = 0;
  const cudaError_t st = cudaMemcpyFromSymbol(&value, ukv::g_device_errors, sizeof(value));
  if (st != cudaSuccess) return Fail("cudaMemcpyFromSymbol", st);
  return static_cast<long long>(value);
}

extern "C" KVQ_API long long kvq_splitzip_device_errors_reset() {
  const unsigned int zero = 0;
  const cudaError_t st = cudaMemcpyToSymbol(ukv::g_device_errors, &zero, sizeof(zero));
  if (st != cudaSuccess) return Fail("cudaMemcpyToSymbol", st);
  return 0;
}

// Test hook of the bounded waits: the fixed6/fixed5 encode of
// kvq_splitzip_bf16_encode_mode, with its statistics pass instantiated with
// a limit of 4 tries per wait instead of 4096, and its producer leaving the
// full barrier of tile `skip_tile` one arrival short.  The consumers' wait
// for that stage runs out (at most 2 x 4 suspended tries of up to 1 ms):
// the kernel counts it in kvq_splitzip_device_errors(), marks the job, and
// carries on; the encode then writes a mode-255 header, which no receiver
// decodes.  Nothing faults or waits without a limit.  Same arguments and
// return values as kvq_splitzip_bf16_encode_mode otherwise.
extern "C" KVQ_API long long kvq_splitzip_test_encode_mode_skip_arrival(
    unsigned long long src_ptr, unsigned long long dst_ptr, unsigned long long count,
    unsigned long long capacity, unsigned long long stream_ptr, int bits, unsigned long long skip_tile) {
  if (src_ptr == 0 || dst_ptr == 0 || count == 0 || (bits != 5 && bits != 6)) return 0;
  std::vector<Prepared> p(1);
  if (!prepare_fixed(reinterpret_cast<const uint16_t*>(src_ptr), flat_layout(count),
                     reinterpret_cast<uint8_t*>(dst_ptr), capacity, bits, p[0]))
    return 0;
  const auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  long long rc = launch_zero<1>(p, 0, 1, stream);
  if (rc < 0) return rc;
  EncBatch<1> b{};
  b.jobs = 1;
  b.skip_tile = static_cast<uint32_t>(std::min<unsigned long long>(skip_tile, 0xFFFFFFFFull));
  b.job[0] = p[0].job;
  b.tile_start[0] = 0;
  b.tile_start[1] = b.job[0].tiles;
  rc = launch_persistent(PresenceKernel<1, kStatsPresence, 4, true>, "PresenceKernel", kEncSmemBytes, b,
                         b.job[0].tiles, stream);
  if (rc < 0) return rc;
  rc = bits == 6 ? launch_persistent(EncodeFixedKernel<1, 6>, "EncodeFixed6Kernel", kEncSmemBytes, b,
                                     b.job[0].tiles, stream)
                 : launch_persistent(EncodeFixedKernel<1, 5>, "EncodeFixed5Kernel", kEncSmemBytes, b,
                                     b.job[0].tiles, stream);
  return rc < 0 ? rc : static_cast<long long>(p[0].result);
}

extern "C" KVQ_API long long kvq_splitzip_abi_version() { return 3; }

extern "C" KVQ_API long long kvq_splitzip_profile_enable(int on) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  for (ProfRecord& r : g_prof_pending) {
    cudaEventSynchronize(r.end);
    g_prof_pool.push_back(r.begin);
    g_prof_pool.push_back(r.end);
  }
  g_prof_pending.clear();
  g_prof_names.clear();
  g_prof_ms.clear();
  g_prof_launches.clear();
  g_prof_on.store(on != 0);
  return 0;
}

extern "C" KVQ_API long long kvq_splitzip_profile_collect() {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  std::map<std::string, size_t> index;
  for (size_t i = 0; i < g_prof_names.size(); ++i) index[g_prof_names[i]] = i;
  for (ProfRecord& r : g_prof_pending) {
    const cudaError_t st = cudaEventSynchronize(r.end);
    if (st != cudaSuccess) return Fail("cudaEventSynchronize", st);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.begin, r.end);
    const std::string name = r.name ? r.name : "?";
    auto it = index.find(name);
    if (it == index.end()) {
      it = index.emplace(name, g_prof_names.size()).first;
      g_prof_names.push_back(name);
      g_prof_ms.push_back(0.0);
      g_prof_launches.push_back(0);
    }
    g_prof_ms[it->second] += ms;
    g_prof_launches[it->second] += 1;
    g_prof_pool.push_back(r.begin);
    g_prof_pool.push_back(r.end);
  }
  g_prof_pending.clear();
  return static_cast<long long>(g_prof_names.size());
}

extern "C" KVQ_API const char* kvq_splitzip_profile_name(int i) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  return i >= 0 && i < static_cast<int>(g_prof_names.size()) ? g_prof_names[i].c_str() : "";
}

extern "C" KVQ_API double kvq_splitzip_profile_ms(int i) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  return i >= 0 && i < static_cast<int>(g_prof_ms.size()) ? g_prof_ms[i] : 0.0;
}

extern "C" KVQ_API long long kvq_splitzip_profile_launches(int i) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  return i >= 0 && i < static_cast<int>(g_prof_launches.size()) ? g_prof_launches[i] : 0;
}

// ---------------------------------------------------------------------
// top16 encode that allocates nothing and keeps no scratch in the caller's
// buffer.
//
// Some callers cannot allocate device memory on the encode path:
// - serving engines that hand nearly all of HBM to their own paged KV pool
//   (vLLM's gpu_memory_utilization), where a transient allocation can fail;
// - latency-critical paths that must not call cudaMalloc / cudaFree, which
//   can synchronise the device.
// This variant keeps the escape counts of its statistics pass in a fixed
// device array of this library, so it writes no byte past the stream.  The
// array is part of the module image: every GPU that loads the library holds
// it until process exit, and no call here (or in the kernels) allocates or
// frees memory.
// ---------------------------------------------------------------------

namespace {

// Largest `count` the static scratch covers: 2^27 words (256 MiB of raw bf16,
// 8192 tiles); the array holds the escape total and error flag, 256 group
// sums and a u16 count per (tile, warp): 64 + 8*256 + 16*8192 = 133184 bytes.
constexpr uint64_t kNoAllocMaxWords = 1ull << 27;
constexpr uint64_t kNoAllocTiles = (kNoAllocMaxWords + kTileWords - 1) / kTileWords;
constexpr uint64_t kNoAllocScratchBytes = auto_scratch_bytes(kNoAllocTiles);
static_assert(kNoAllocScratchBytes == 133184, "the documented size of the no-alloc scratch");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on each device.  Host code cannot use
// the symbol itself (it names a host-side shadow); the address is looked up
// once per device, with that device current, the first time this entry point
// runs on it, and kept for the process (a device reset invalidates it; the
// header says so).
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_address[kNoAllocMaxDevices] = {};

void* noalloc_scratch_for_current_device() {
  int device = 0;
  cudaError_t st = cudaGetDevice(&device);
  if (st != cudaSuccess) {
    Fail("cudaGetDevice", st);
    return nullptr;
  }
  if (device < 0 || device >= kNoAllocMaxDevices) {
    g_last_error = "kvq_splitzip_bf16_encode_top16_noalloc: device index out of range";
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_address[device] == nullptr) {
    void* address = nullptr;
    st = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (st != cudaSuccess) {
      Fail("cudaGetSymbolAddress", st);
      return nullptr;
    }
    g_noalloc_address[device] = address;
  }
  return g_noalloc_address[device];
}

}  // namespace

extern "C" KVQ_API long long kvq_splitzip_bf16_encode_top16_noalloc(unsigned long long src_ptr,
                                                                    unsigned long long dst_ptr,
                                                                    unsigned long long count,
                                                                    unsigned long long capacity,
                                                                    unsigned long long tables_ptr,
                                                                    unsigned long long stream_ptr) {
  if (src_ptr == 0 || dst_ptr == 0 || tables_ptr == 0 || count == 0 || count > 0xFFFFFFFFULL) {
    return 0;
  }
  if (count > kNoAllocMaxWords) {
    g_last_error = "kvq_splitzip_bf16_encode_top16_noalloc: count " + std::to_string(count) +
                   " words exceeds the static scratch maximum of " +
                   std::to_string(kNoAllocMaxWords) + " words";
    return -1;
  }
  const uint64_t n = count;
  const uint64_t encoded = top16_size(n);
  // the reference's decline rules (.cu:385-395); no room past the stream is
  // needed beyond the reference's own 8 bytes
  if (encoded >= n * 2 || ((encoded + 3) & ~3ULL) + 8 > capacity) return 0;
  void* scratch = noalloc_scratch_for_current_device();
  if (scratch == nullptr) return -1;
  auto* dst = reinterpret_cast<uint8_t*>(dst_ptr);
  const auto stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  EncBatch<1> b{};
  b.jobs = 1;
  b.job[0] = base_job(reinterpret_cast<const uint16_t*>(src_ptr), flat_layout(n), dst,
                      reinterpret_cast<const uint8_t*>(tables_ptr));
  b.job[0].scratch = static_cast<uint8_t*>(scratch);
  b.job[0].error = reinterpret_cast<uint32_t*>(b.job[0].scratch + 4);
  b.tile_start[0] = 0;
  b.tile_start[1] = b.job[0].tiles;
  // Every call shares the array and finds the previous call's contents in
  // it: clear the escape total, error flag, group words and tile counts (the
  // encode kernel clears the stream's unused escape slots).
  const cudaError_t st = cudaMemsetAsync(scratch, 0, auto_scratch_bytes(b.job[0].tiles), stream);
  if (st != cudaSuccess) return Fail("cudaMemsetAsync", st);
  const long long rc = launch_encode_kernels(EncOp::kTop16Scratch, b, b.job[0].tiles, stream);
  return rc < 0 ? rc : static_cast<long long>(encoded);
}
