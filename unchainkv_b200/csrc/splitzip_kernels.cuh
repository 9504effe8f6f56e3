// Batched, persistent splitzip kernels (sm_100a).
//
// Every kernel takes a batch of jobs as a __grid_constant__ parameter (one
// job = one reference ABI call: one layer of one request).  The work is the
// 16384-word tiles of all jobs.  Kernels are persistent: the grid is sized
// to the resident CTAs, each CTA walks a contiguous chunk of tiles, and a
// ring of 2 (encode) or 3 (decode) shared-memory stages filled by TMA bulk
// copies keeps the next tiles in flight while the current one is coded.  Only the top16
// encoder, whose escape offsets chain tile to tile, takes tiles by atomic
// ticket instead (so every tile it waits for is held by a running CTA).
//
// Per tile: one CTA of 256 threads = 8 warps x 4 steps x 32 lanes x 16 words.
//   encode: 16 words per lane in registers -> body/low plane by byte_perm,
//     codes by one shared-memory lookup per word -> warp funnel stores into
//     the unaligned stream regions (aligned 8/4/2-byte stores);
//   decode: stream bytes staged by TMA -> 16 output words per lane -> two
//     16-byte stores into the paged cache block.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "splitzip_device.cuh"

namespace ukv {

constexpr int kMaxBatch = 96;
constexpr int kEncStages = 2;  // ring depth of the encode kernels (32 KiB stages, 3 CTAs per SM)
// Ring depth of the decode kernel: 3 stages of 32.1 KiB, one CTA per SM.
// Two CTAs would fit; the launch asks for kDecCtaSmemBytes of dynamic
// shared memory so that they do not.  Two CTAs per SM took 192 us on
// configs[1]'s 32 layers against 172 for one; a grid capped at one CTA per
// SM left the block scheduler free to put two of them on one SM while the
// previous kernel's CTAs drained (launches overlap): 0.548 ms per round trip
// against 0.49.  4 and 6 stages ran as fast in the timed loop, but their
// event-timed launches on an idle GPU took 182-190 us.
constexpr int kDecStages = 3;
constexpr uint32_t kEncStageBytes = kTileWords * 2;  // 32 KiB of words
constexpr uint32_t kDecStageBytes = 2 * kTileWords + 128;
constexpr uint32_t kDecCodesOffset = kTileWords + 128;  // top16/fixed6 codes inside a stage
constexpr uint32_t kEncSmemBytes = kEncStages * kEncStageBytes;
constexpr uint32_t kDecSmemBytes = kDecStages * kDecStageBytes;
constexpr uint32_t kDecCtaSmemBytes = 128 * 1024;  // > half an SM's shared memory: one CTA per SM
static_assert(kDecCtaSmemBytes >= kDecSmemBytes, "the decode ring fits the request");

// ------------------------------------------------------------------ jobs

// Encode job.  `scratch` is 16-byte aligned device memory inside the
// caller's stream buffer, past the stream (see the layout constants below).
struct EncJob {
  const uint16_t* src;
  Layout L;
  uint8_t* dst;
  uint8_t* scratch;
  uint32_t* error;  // set to 1 when a wait of this job's tiles ran out (or null)
  uint64_t n;
  uint64_t half;
  uint64_t cap;  // top16 escape capacity ceil(n/200)
  const uint8_t* tables;
  uint32_t tiles;
  int bulk;
  int raw_ok;  // auto encode may write raw mode 6 ([6] + words)
  int pad;
};

template <int kMax>
struct EncBatch {
  uint32_t jobs;
  uint32_t skip_tile;  // test-only instantiations: the tile whose full-barrier arrival is skipped
  uint32_t tile_start[kMax + 1];
  EncJob job[kMax];
};

struct DecJob {
  const uint8_t* src;
  uint64_t src_bytes;  // bytes available in the stream buffer
  uint16_t* dst;
  Layout L;
  uint64_t n;
  uint64_t half;
  uint64_t cap;
  const uint8_t* tables;
  uint32_t tiles;
  uint32_t pad0;
  int vec;  // 16-byte stores of whole units into the destination layout
  int pad;
};

template <int kMax>
struct DecBatch {
  uint32_t jobs;
  uint32_t tile_start[kMax + 1];
  DecJob job[kMax];
};

template <int kMax>
struct ZeroBatch {
  uint32_t count;
  uint8_t* ptr[kMax];
  uint64_t bytes[kMax];
};

template <int kMax>
__device__ __forceinline__ int find_job(const uint32_t* start, uint32_t jobs, uint32_t t) {
  if (kMax == 1) return 0;
  int lo = 0, hi = static_cast<int>(jobs) - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Tiles are visited in increasing order, so the job index only moves forward.
template <int kMax>
__device__ __forceinline__ int advance_job(const uint32_t* start, int j, uint32_t t) {
  if constexpr (kMax == 1) {
    return 0;
  } else {
    while (t >= start[j + 1]) ++j;
    return j;
  }
}

struct Chunk {
  uint32_t first;
  uint32_t last;
};

__device__ __forceinline__ Chunk cta_chunk(uint32_t total) {
  const uint32_t per = (total + gridDim.x - 1) / gridDim.x;
  const uint32_t first = min(blockIdx.x * per, total);
  return {first, min(first + per, total)};
}

// Scratch layouts (byte offsets from EncJob::scratch).
//   fixed encode: [0,32) high-byte bitmap, [32,36) error flag.
//   auto and top16 encode: [0,4) escape total, [4,8) error flag, [16,48)
//     bitmap (auto only), [64, 64+8G) group words (escapes of 32 tiles),
//     then from the next 16-byte boundary 16T bytes of escape counts per
//     (tile, warp) as u16.
__host__ __device__ constexpr uint64_t groups_for(uint64_t tiles) { return (tiles + 31) / 32; }
__host__ __device__ constexpr uint64_t auto_counts_offset(uint64_t tiles) {
  return 64 + (8 * groups_for(tiles) + 15) / 16 * 16;
}
__host__ __device__ constexpr uint64_t auto_scratch_bytes(uint64_t tiles) {
  return auto_counts_offset(tiles) + 2 * kWarps * tiles;
}
constexpr uint64_t kFixedScratchBytes = 36;

// Scratch of the reference-ABI top16 encode, kept inside the stream itself:
// the reference's capacity rule (align4(encoded) + 8, kvq_splitzip_cuda.cu:
// 390-394) leaves no room past the stream for per-tile counts.  Tile t's
// 32-byte count record is the first 16-byte aligned slot of the tile's own
// body region; only the encode of tile t overwrites it, after that tile's
// producer has read it.  A last tile too short to hold one (it then holds
// the words of warp 0 alone) keeps a 4-byte record in the reference's own
// scratch bytes at align4(encoded).
//   stats pass: u16[8] at +0 = escapes of each warp's run of the tile;
//   scan pass:  u16[8] at +0 = escapes of the tile before each warp's run,
//               u32 at +16 = escapes of the job before the tile; header;
//   encode:     the producer copies the record into the stage descriptor.
constexpr uint64_t kTailRecord = ~0ull;
__host__ __device__ constexpr uint64_t top16_stream_bytes(uint64_t n) {
  return 5 + n + (n + 1) / 2 + 5 * ((n + 199) / 200);
}
__host__ __device__ constexpr uint64_t top16_tail_offset(uint64_t n) { return (top16_stream_bytes(n) + 3) & ~3ull; }
__host__ __device__ inline uint64_t top16_record_offset(uint64_t dst_addr, uint64_t n, uint64_t t) {
  const uint64_t body = 5 + t * kTileWords;
  const uint64_t left = n - t * kTileWords;
  const uint64_t len = left < kTileWords ? left : kTileWords;
  const uint64_t off = ((dst_addr + body + 15) & ~15ull) - dst_addr;
  return off + 32 <= body + len ? off : kTailRecord;
}

// Little-endian u32 at any byte address.
__device__ __forceinline__ uint32_t ld_u32_bytes(const uint8_t* p) {
  return p[0] | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}
__device__ __forceinline__ void st_u32_bytes(uint8_t* p, uint32_t v) {
  p[0] = static_cast<uint8_t>(v);
  p[1] = static_cast<uint8_t>(v >> 8);
  p[2] = static_cast<uint8_t>(v >> 16);
  p[3] = static_cast<uint8_t>(v >> 24);
}

__device__ unsigned int g_device_errors;

__device__ __forceinline__ void raise_error(uint32_t* flag) {
  if (flag) atomicOr(flag, 1u);
  atomicAdd(&g_device_errors, 1u);
}

// A wait of this tile ran out in the encode pass: the stream's mode byte
// becomes 255, which no receiver decodes (lane 0 of the late warp; the job's
// error flag is already set).
__device__ __forceinline__ void mark_stream_late(const EncJob& J) {
  __threadfence();
  J.dst[0] = 255;
}

// After the header write (thread 0 of the CTA that wrote it): a wait that ran
// out in the stats pass, or in this pass before the header landed, set the
// job's flag; the fences order this re-check against mark_stream_late, so
// whichever store comes last is 255.
__device__ __forceinline__ void recheck_header(const EncJob& J) {
  if (J.error == nullptr) return;
  __threadfence();
  if (ld_volatile_u32(J.error) != 0) J.dst[0] = 255;
}

__device__ __forceinline__ uint32_t tile_len(uint64_t n, uint64_t t0) {
  return static_cast<uint32_t>(n - t0 < kTileWords ? n - t0 : kTileWords);
}

// 16 words (8 registers) of a lane's unit from a staged tile.
__device__ __forceinline__ void load_unit(const uint16_t* sin, uint32_t w0, uint32_t (&x)[8]) {
  const uint4 v0 = *reinterpret_cast<const uint4*>(sin + w0);
  const uint4 v1 = *reinterpret_cast<const uint4*>(sin + w0 + 8);
  x[0] = v0.x; x[1] = v0.y; x[2] = v0.z; x[3] = v0.w;
  x[4] = v1.x; x[5] = v1.y; x[6] = v1.z; x[7] = v1.w;
}

__device__ __forceinline__ uint32_t step_valid_words(uint32_t len, uint32_t sb) {
  return len > sb ? min(len - sb, static_cast<uint32_t>(kStepWords)) : 0u;
}

// ------------------------------------------------------- ring pipeline
//
// Warp-specialized: warp kProducerWarp stages tiles into a ring of
// shared-memory buffers (TMA bulk copies issued by its lane 0, plus the
// per-tile descriptor the consumers need); warps 0..kWarps-1 code the
// tiles.  full[s] completes when the 32 producer lanes have arrived and the
// stage's TMA bytes have landed; empty[s] when every consumer warp has
// released the stage.  The producer ends the sequence with a descriptor
// whose tile is kEndTile.  Consumers synchronise among themselves with
// named barrier 1 (consumer_sync), never with __syncthreads.

constexpr int kCtaThreads = kThreads + 32;
constexpr int kProducerWarp = kWarps;
constexpr uint32_t kEndTile = 0xFFFFFFFFu;

template <int S>
struct Ring {
  uint64_t full[S];
  uint64_t empty[S];
};

template <int S>
__device__ __forceinline__ void ring_init(Ring<S>& R) {
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(&R.full[s], 32);
      mbar_init(&R.empty[s], kWarps);
    }
    fence_mbar_init();
  }
}

// Position in a ring of S stages: uses so far, stage, parity of the stage's
// current use.
template <int S>
struct RingPos {
  uint32_t k = 0;
  int s = 0;
  uint32_t phase = 0;
  bool late = false;  // consumer: the wait for the current stage (or its producer's) ran out
  __device__ __forceinline__ void next() {
    ++k;
    if (++s == S) {
      s = 0;
      phase ^= 1u;
    }
  }
};

// Bounded wait for a ring barrier phase.  A timeout raises the error flag and
// waits once more so that no copy is left in flight.  Returns true when the
// wait ran out.
template <uint32_t kTries = kBarrierTries>
__device__ __forceinline__ bool wait_stage(uint64_t* bar, uint32_t parity, uint32_t* error) {
  if (!mbar_wait<kTries>(bar, parity)) {
    raise_error(error);
    mbar_wait<kTries>(bar, parity);
    return true;
  }
  return false;
}

// Producer: wait until every consumer warp released the stage's previous use.
template <int S, uint32_t kTries = kBarrierTries>
__device__ __forceinline__ bool producer_acquire(Ring<S>& R, const RingPos<S>& p, uint32_t* error) {
  return p.k >= S && wait_stage<kTries>(&R.empty[p.s], p.phase ^ 1u, error);
}

// Producer, every lane: publish the stage (after its descriptor writes).
template <int S>
__device__ __forceinline__ void producer_commit(Ring<S>& R, const RingPos<S>& p) {
  mbar_arrive(&R.full[p.s]);
}

template <int S, uint32_t kTries = kBarrierTries>
__device__ __forceinline__ bool consumer_wait(Ring<S>& R, const RingPos<S>& p, uint32_t* error) {
  return wait_stage<kTries>(&R.full[p.s], p.phase, error);
}

// Consumer warp: done with the stage (all lanes' reads precede lane 0's arrive).
template <int S>
__device__ __forceinline__ void consumer_release(Ring<S>& R, const RingPos<S>& p) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&R.empty[p.s]);
}

// Barrier among the kThreads consumer threads (the producer warp never joins).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
}

using EncRing = Ring<kEncStages>;
using EncPos = RingPos<kEncStages>;
using DecRing = Ring<kDecStages>;
using DecPos = RingPos<kDecStages>;

// Encode stage descriptor: global tile index (or kEndTile), its job, and
// what the kernel's producer hook computed for the tile.
struct EncDesc {
  uint32_t tile;
  uint32_t job;
  uint32_t aux;
  uint32_t late;  // the producer's wait for this stage ran out
  uint64_t prefix;        // auto top16: escapes of the job before this tile
  uint32_t wpre[kWarps];  // auto top16: escapes of the tile before each warp's run
};

// Producer hook (run by all 32 producer lanes once the tile is staged; lane
// 0 writes the descriptor) that annotates nothing.
struct NoAux {
  template <typename Job>
  __device__ __forceinline__ void operator()(const Job&, uint32_t, EncDesc&) const {}
};

// Producer warp of the encode kernels: stages the tiles [first, last) of
// this CTA's chunk into the ring, in order.  The tiles are planned 32 at a
// time, one per lane (job, bounds and -- when the tile is one contiguous run
// of a bulk-capable job -- its TMA source, block-table load included), so a
// tile costs the producer a few shuffles and one copy issued by lane 0.
// Tiles of several runs (blocks shorter than a tile) take one copy per run
// over the 32 lanes, and other layouts are gathered word by word.
template <int kMax, uint32_t kTries = kBarrierTries, bool kSkipTest = false, typename Aux = NoAux>
__device__ __forceinline__ void encode_producer(const EncBatch<kMax>& b, uint8_t* ring, EncRing& R, EncDesc* D,
                                                uint32_t first, uint32_t last, Aux aux = Aux()) {
  const int lane = threadIdx.x & 31;
  EncPos p;
  int ji = find_job<kMax>(b.tile_start, b.jobs, first);  // job of the group's first tile
  for (uint32_t g = first; g < last; g += 32) {
    // ---- plan tile g + lane
    const uint32_t mine = g + lane;
    int pj = ji;
    uint64_t pt0 = 0;
    uint32_t plen = 0;
    const uint16_t* psrc = nullptr;  // non-null: a single-run tile, staged from here
    if (mine < last) {
      pj = advance_job<kMax>(b.tile_start, ji, mine);
      const EncJob& J = b.job[pj];
      pt0 = static_cast<uint64_t>(mine - b.tile_start[pj]) * kTileWords;
      plen = tile_len(J.n, pt0);
      if (J.bulk != 0 && (J.L.block_words == 0 || J.L.block_words % kTileWords == 0))
        psrc = J.src + layout_addr(J.L, pt0);
    }
    const uint32_t count = min(32u, last - g);
    for (uint32_t k = 0; k < count; ++k) {
      const uint32_t t = g + k;
      const int tj = __shfl_sync(kFull, pj, k);
      const uint64_t t0 = __shfl_sync(kFull, pt0, k);
      const uint32_t len = __shfl_sync(kFull, plen, k);
      const uint16_t* src = reinterpret_cast<const uint16_t*>(
          __shfl_sync(kFull, reinterpret_cast<unsigned long long>(psrc), k));
      const bool late = producer_acquire<kEncStages, kTries>(R, p, nullptr);
      const EncJob& J = b.job[tj];
      uint16_t* sin = reinterpret_cast<uint16_t*>(ring + p.s * kEncStageBytes);
      if (lane == 0) {
        D[p.s].tile = t;
        D[p.s].job = static_cast<uint32_t>(tj);
        D[p.s].late = late;
      }
      if (src != nullptr) {
        if (lane == 0) {
          const uint32_t whole = len & ~7u;  // the flat layout's last < 8 words go by plain loads
          if (whole) {
            mbar_expect_tx(&R.full[p.s], whole * 2);
            bulk_g2s(sin, src, whole * 2, &R.full[p.s]);
          }
          for (uint32_t j = whole; j < len; ++j) sin[j] = src[j];
        }
      } else if (J.bulk != 0) {
        issue_runs(plan_run(J.src, J.L, t0, len, lane), J.src, J.L, t0, len, sin, &R.full[p.s]);
      } else {
        gather_words_warp(J.src, J.L, t0, len, sin);
      }
      aux(J, t - b.tile_start[tj], D[p.s]);
      if (kSkipTest && t == b.skip_tile && lane == 31) {
        // test-only: this stage's full barrier stays one arrival short, so the
        // consumers' bounded wait for it runs out
      } else {
        producer_commit(R, p);
      }
      p.next();
    }
    ji = __shfl_sync(kFull, pj, count - 1);
  }
  producer_acquire<kEncStages, kTries>(R, p, nullptr);
  if (lane == 0) D[p.s].tile = kEndTile;
  producer_commit(R, p);
}

// Consumer warps of the encode kernels: fn(job, job_index, tile, words,
// ring position, descriptor) for every staged tile until the end descriptor.
template <int kMax, uint32_t kTries = kBarrierTries, typename Fn>
__device__ __forceinline__ void encode_consumer(const EncBatch<kMax>& b, uint8_t* ring, EncRing& R,
                                                const EncDesc* D, Fn&& fn) {
  EncPos p;
  for (;;) {
    const bool late = consumer_wait<kEncStages, kTries>(R, p, nullptr);
    const EncDesc& d = D[p.s];  // read in place; the stage is released after fn
    if (d.tile == kEndTile) return;
    const EncJob& J = b.job[d.job];
    // a wait that ran out marks the job's stream (the encode then writes
    // the mode-255 header, which no receiver decodes)
    p.late = late || d.late != 0;
    if (p.late && J.error != nullptr && (threadIdx.x & 31) == 0) atomicOr(J.error, 1u);
    fn(J, static_cast<int>(d.job), d.tile - b.tile_start[d.job],
       reinterpret_cast<const uint16_t*>(ring + p.s * kEncStageBytes), p, d);
    consumer_release(R, p);
    p.next();
  }
}

// Chunk-scheduled encode kernel body: producer warp + consumer warps.
template <int kMax, uint32_t kTries = kBarrierTries, bool kSkipTest = false, typename Fn, typename Aux = NoAux>
__device__ __forceinline__ void encode_pipeline(const EncBatch<kMax>& b, uint8_t* ring, EncRing& R, EncDesc* D,
                                                Fn&& fn, Aux aux = Aux()) {
  if ((threadIdx.x >> 5) == kProducerWarp) {
    const Chunk c = cta_chunk(b.tile_start[b.jobs]);
    encode_producer<kMax, kTries, kSkipTest>(b, ring, R, D, c.first, c.last, aux);
    return;
  }
  encode_consumer<kMax, kTries>(b, ring, R, D, fn);
}

// ------------------------------------------------------------ top16 encode

// Table entry per (plane, exponent): code nibble copied into both nibbles,
// bits 16 and 17 set for "escape" (code 255 of the reference table; the
// stored nibble is then 0).
__device__ __forceinline__ void load_top16_table(const uint8_t* tables, uint32_t* stbl) {
  for (int i = threadIdx.x; i < 512; i += kThreads) {
    const uint32_t c = __ldg(tables + i);
    stbl[i] = c == 255u ? 0x30000u : (c & 0xFu) * 0x11u;
  }
}

// Merge the entries of an even and an odd word: bits 0-7 code byte, bit 16
// even escape, bit 17 odd escape (one LOP3).
__device__ __forceinline__ uint32_t merge_pair(uint32_t t0, uint32_t t1) {
  return (t0 & 0x1000Fu) | (t1 & ~0x1000Fu);
}

// Codes (c0, c1: 8 code bytes) and escape mask (16 bits) of 16 words.
__device__ __forceinline__ void top16_unit_codes(const uint32_t (&x)[8], const uint32_t* tbl,
                                                 uint64_t g, uint64_t half, uint32_t& c0,
                                                 uint32_t& c1, uint32_t& esc) {
  uint32_t u[8];
  if (g >= half || g + kUnitWords <= half) {
    // byte offset of a word's entry: exponent * 4, plus 1 KiB for plane 1
    const uint32_t plane = g >= half ? 1024u : 0u;
    const uint8_t* t = reinterpret_cast<const uint8_t*>(tbl);
#pragma unroll
    for (int p = 0; p < 8; ++p)
      u[p] = merge_pair(*reinterpret_cast<const uint32_t*>(t + (((x[p] >> 5) & 0x3FCu) | plane)),
                        *reinterpret_cast<const uint32_t*>(t + (((x[p] >> 21) & 0x3FCu) | plane)));
  } else {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const uint32_t* t0 = tbl + ((g + 2 * p) >= half ? 256 : 0);
      const uint32_t* t1 = tbl + ((g + 2 * p + 1) >= half ? 256 : 0);
      u[p] = merge_pair(t0[(x[p] >> 7) & 0xFFu], t1[(x[p] >> 23) & 0xFFu]);
    }
  }
  c0 = __byte_perm(__byte_perm(u[0], u[1], 0x0040), __byte_perm(u[2], u[3], 0x0040), 0x5410);
  c1 = __byte_perm(__byte_perm(u[4], u[5], 0x0040), __byte_perm(u[6], u[7], 0x0040), 0x5410);
  // escape flags (bits 16-17 of each u[p]) -> bits 2p, 2p+1, branch-free:
  // gather byte 2 of every u[p], then pack the 2-bit fields of 4 bytes
  const uint32_t f0 = __byte_perm(__byte_perm(u[0], u[1], 0x0062), __byte_perm(u[2], u[3], 0x0062), 0x5410);
  const uint32_t f1 = __byte_perm(__byte_perm(u[4], u[5], 0x0062), __byte_perm(u[6], u[7], 0x0062), 0x5410);
  const uint32_t a0 = f0 | (f0 >> 6);  // pairs 0,1 at bits 0-3; pairs 2,3 at bits 16-19
  const uint32_t a1 = f1 | (f1 >> 6);
  esc = (a0 & 0xFu) | ((a0 >> 12) & 0xF0u) | ((a1 & 0xFu) << 8) | ((a1 >> 4) & 0xF000u);
}

// Body + codes of one tile; returns this lane's escape masks per step.
__device__ __forceinline__ void top16_tile_body(const EncJob& J, uint64_t t0, uint32_t len,
                                                const uint16_t* sin, const uint32_t* stbl,
                                                uint32_t (&masks)[kStepsPerWarp]) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (len == kTileWords) {  // full tile: the warp's steps form one run per region
    uint32_t bb[kStepsPerWarp][4];
    uint32_t cw[kStepsPerWarp][2];
#pragma unroll
    for (int s = 0; s < kStepsPerWarp; ++s) {
      const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
      uint32_t x[8];
      load_unit(sin, w0, x);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t lo = __byte_perm(x[2 * q], x[2 * q + 1], 0x6420);
        const uint32_t hi = __byte_perm(x[2 * q], x[2 * q + 1], 0x7531);
        bb[s][q] = (lo & 0x7F7F7F7Fu) | (hi & 0x80808080u);
      }
      top16_unit_codes(x, stbl, t0 + w0, J.half, cw[s][0], cw[s][1], masks[s]);
    }
    const uint64_t r0 = t0 + static_cast<uint64_t>(warp) * kStepsPerWarp * kStepWords;
    warp_store_run<4, 8, kStepsPerWarp>(J.dst + 5 + r0, bb, lane);
    warp_store_run<2, 8, kStepsPerWarp>(J.dst + 5 + J.n + r0 / 2, cw, lane);
    return;
  }
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = step_valid_words(len, sb);
    masks[s] = 0;
    if (step_valid == 0) continue;  // uniform per warp
    uint32_t x[8];
    load_unit(sin, w0, x);
    uint32_t bb[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t lo = __byte_perm(x[2 * q], x[2 * q + 1], 0x6420);
      const uint32_t hi = __byte_perm(x[2 * q], x[2 * q + 1], 0x7531);
      bb[q] = (lo & 0x7F7F7F7Fu) | (hi & 0x80808080u);
    }
    uint32_t c0, c1, esc;
    top16_unit_codes(x, stbl, t0 + w0, J.half, c0, c1, esc);
    uint8_t* bdst = J.dst + 5 + t0 + sb;
    uint8_t* cdst = J.dst + 5 + J.n + (t0 + sb) / 2;
    if (step_valid == kStepWords) {
      const uint32_t cw[2] = {c0, c1};
      warp_store_words<4, 8>(bdst, bb, lane);
      warp_store_words<2, 8>(cdst, cw, lane);
    } else {
      const uint64_t body[2] = {bb[0] | (static_cast<uint64_t>(bb[1]) << 32),
                                bb[2] | (static_cast<uint64_t>(bb[3]) << 32)};
      const uint32_t valid = w0 < len ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
      if (valid < kUnitWords) {
        esc &= (1u << valid) - 1u;
        const uint64_t keep = valid == 0 ? 0ull : (~0ull >> (64 - 4 * valid));
        const uint64_t cc = (static_cast<uint64_t>(c1) << 32 | c0) & keep;
        c0 = static_cast<uint32_t>(cc);
        c1 = static_cast<uint32_t>(cc >> 32);
      }
      const uint64_t codes[1] = {c0 | (static_cast<uint64_t>(c1) << 32)};
      warp_store<uint64_t, 2>(bdst, step_valid, body, lane);
      warp_store<uint64_t, 1>(cdst, (step_valid + 1) / 2, codes, lane);
    }
    masks[s] = esc;
  }
}

// Escape entries of this warp's run (its kStepsPerWarp steps, in position
// order), the first at slot `base`.  A step without escapes costs one
// ballot; when no lane has two escapes in the step (the common case) a
// lane's offset is the number of lower lanes with one, else a warp scan.
__device__ __forceinline__ void warp_write_escapes(const EncJob& J, uint64_t t0, const uint16_t* sin,
                                                   const uint32_t (&masks)[kStepsPerWarp], uint64_t base) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t lower = (1u << lane) - 1u;
  // slots are counted from `base`: the run of entries starts at `run`, and
  // `room` of its slots lie below the capacity (at most ceil(n/200) < 2^32)
  uint8_t* run = J.dst + 5 + J.n + (J.n + 1) / 2 + 5 * base;
  const uint32_t room = base < J.cap ? static_cast<uint32_t>(J.cap - base) : 0u;
  uint32_t rel = 0;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t m = masks[s];
    const uint32_t lanes = __ballot_sync(kFull, m != 0);
    if (lanes == 0) continue;  // uniform
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (__ballot_sync(kFull, (m & (m - 1)) != 0) == 0) {
      // at most one escape per lane: no loop
      const uint32_t slot = rel + __popc(lanes & lower);
      if (m != 0 && slot < room) {
        const uint32_t w = w0 + (__ffs(m) - 1);
        const uint32_t pos = static_cast<uint32_t>(t0) + w;
        uint8_t* en = run + 5 * static_cast<uint64_t>(slot);
        en[0] = static_cast<uint8_t>(pos);
        en[1] = static_cast<uint8_t>(pos >> 8);
        en[2] = static_cast<uint8_t>(pos >> 16);
        en[3] = static_cast<uint8_t>(pos >> 24);
        en[4] = static_cast<uint8_t>(sin[w] >> 7);
      }
      rel += __popc(lanes);
      continue;
    }
    const uint32_t mine = __popc(m);
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    if (m != 0) {
      uint32_t slot = rel + incl - mine;
      uint32_t bits = m;
      do {
        const uint32_t w = w0 + (__ffs(bits) - 1);
        bits &= bits - 1;
        if (slot < room) {
          const uint32_t pos = static_cast<uint32_t>(t0) + w;
          uint8_t* en = run + 5 * static_cast<uint64_t>(slot);
          en[0] = static_cast<uint8_t>(pos);
          en[1] = static_cast<uint8_t>(pos >> 8);
          en[2] = static_cast<uint8_t>(pos >> 16);
          en[3] = static_cast<uint8_t>(pos >> 24);
          en[4] = static_cast<uint8_t>(sin[w] >> 7);
        }
        ++slot;
      } while (bits);
    }
    rel += __shfl_sync(kFull, incl, 31);
  }
}

__device__ __forceinline__ void write_top16_header(uint8_t* dst, uint64_t total, uint64_t cap,
                                                   bool error) {
  dst[0] = (total > cap || error) ? 255 : 5;
  const uint32_t cnt = static_cast<uint32_t>(total > cap ? cap : total);
  dst[1] = static_cast<uint8_t>(cnt);
  dst[2] = static_cast<uint8_t>(cnt >> 8);
  dst[3] = static_cast<uint8_t>(cnt >> 16);
  dst[4] = static_cast<uint8_t>(cnt >> 24);
}

// ------------------------------------------------- presence / auto stats

// Statistics pass, by kKind:
//   kStatsPresence: high-byte presence of every word (-> job bitmap), for the
//     fixed6 / fixed5 palette;
//   kStatsAuto: the bitmap and the top16 escape count of every tile (-> tile
//     count per warp, group sum, job total; each warp adds its own share, so
//     no CTA barrier is needed for the counts), for the auto encode;
//   kStatsTop16: the escape counts alone into the scratch array (the top16
//     encode that allocates nothing);
//   kStatsTop16Rec: the escape counts alone into each tile's record inside
//     the stream (the reference-ABI top16 encode).
//
// The presence table holds high byte h at index h ^ (sign << 2), so that a
// value and its negation (which share every other bit of h) fall in
// different shared-memory banks.  Word order does not matter here, so each
// lane reads two 16-byte chunks that are contiguous across the warp
// (conflict-free).  For kStatsAuto, once a job's running escape total
// exceeds its top16 capacity the job cannot be top16 and its remaining tiles
// skip the escape count (the producer reads the total for each tile).  The
// explicit top16 encode counts every tile: an overflowing stream still holds
// the first `cap` escapes, so every tile's offset must be exact.
__device__ __forceinline__ uint32_t presence_index(uint32_t h) { return h ^ ((h >> 5) & 4u); }
template <uint32_t kOff> struct StatsPlane { static constexpr uint32_t kOffset = kOff; };
template <bool kB> struct CompileFlag { static constexpr bool kValue = kB; };

// Sign-and-exponent index (the word's bits 7..15) with the sign copied into
// bank bit 4 (byte bit 6), for the 512-entry stats tables.
__device__ __forceinline__ uint32_t stats_index(uint32_t i9) { return i9 ^ ((i9 >> 2) & 0x40u); }

enum StatsKind { kStatsPresence = 0, kStatsAuto = 1, kStatsTop16 = 2, kStatsTop16Rec = 3 };

template <int kMax, int kKind, uint32_t kTries = kBarrierTries, bool kSkipTest = false>
__global__ void __launch_bounds__(kCtaThreads, 3) PresenceKernel(const __grid_constant__ EncBatch<kMax> b) {
  constexpr bool kStats = kKind != kStatsPresence;
  constexpr bool kPresence = kKind != kStatsTop16 && kKind != kStatsTop16Rec;
  extern __shared__ __align__(128) uint8_t ring[];
  // Presence is kept per high byte (256 entries) when only presence is wanted,
  // and per sign-and-exponent (512 entries) when escapes are counted too: one
  // 9-bit index then serves both tables.  Both layouts put the sign into a
  // bank bit (stats_index, presence_index), so +e and -e land in other banks.
  __shared__ __align__(16) uint8_t spres[kStats ? 512 : 256];
  __shared__ __align__(16) uint8_t sesc[1024];  // [plane][stats_index]: 1 where the exponent has no top16 code
  __shared__ EncRing R;
  __shared__ EncDesc D[kEncStages];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  constexpr int kPresWords = sizeof(spres) / 4;
  if (tid < kPresWords) reinterpret_cast<uint32_t*>(spres)[tid] = 0;
  ring_init(R);
  __syncthreads();
  grid_dependency_sync();
  int pres_job = -1, table_job = -1;
  // OR the presence bits gathered for a job into its bitmap, then clear them
  // (consumers only; every warp is past its last presence store)
  auto flush = [&](const EncJob& P) {
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(P.scratch + (kStats ? 16 : 0));
    // high byte h covers the sign-and-exponent pair 2h, 2h + 1 (one u16)
    const bool seen = kStats ? *reinterpret_cast<const uint16_t*>(spres + stats_index(2u * tid)) != 0
                             : spres[presence_index(tid)] != 0;
    const uint32_t bits = __ballot_sync(kFull, seen);
    if (lane == 0 && bits) atomicOr(&bitmap[warp], bits);
    consumer_sync();
    if (tid < kPresWords) reinterpret_cast<uint32_t*>(spres)[tid] = 0;
  };
  // aux = 1 when the job's escapes already exceed its top16 capacity
  // (the total only grows, so a job once seen over stays over: the producer
  // remembers it and skips the global load for its remaining tiles)
  // The total is read one tile ahead (the load's latency overlaps the next
  // tile's staging): a job is seen over its capacity a tile later, which
  // only means one more tile counted.
  const EncJob* over_job = nullptr;  // producer warp: the job last seen over its capacity
  const EncJob* seen_job = nullptr;  // the job whose total was read last
  uint32_t seen_total = 0;
  auto over_cap = [&](const EncJob& J, uint32_t, EncDesc& d) {
    bool over = false;
    if (kKind == kStatsAuto) {
      over = &J == over_job || (&J == seen_job && seen_total > J.cap);
      if (over) {
        over_job = &J;
      } else {
        seen_total = ld_volatile_u32(reinterpret_cast<const uint32_t*>(J.scratch));
        seen_job = &J;
      }
    }
    if ((threadIdx.x & 31) == 0) d.aux = over;
  };
  encode_pipeline<kMax, kTries, kSkipTest>(b, ring, R, D, [&](const EncJob& J, int j, uint32_t tile,
                                                               const uint16_t* sin, const EncPos& pos,
                                                               const EncDesc& desc) {
    const uint32_t skip_escapes = desc.aux;
    if (j != pres_job || (kStats && j != table_job)) {  // uniform across the consumers
      consumer_sync();
      if (j != pres_job) {
        if (kPresence && pres_job >= 0) flush(b.job[pres_job]);
        pres_job = j;
      }
      if (kStats && j != table_job) {
        for (int i = tid; i < 1024; i += kThreads)
          sesc[(i & 512) | stats_index(i & 511)] = __ldg(J.tables + ((i >> 1) & 256) + (i & 255)) == 255u;
        table_job = j;
      }
      consumer_sync();
    }
    const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
    const uint32_t len = tile_len(J.n, t0);
    const bool count = kStats && !skip_escapes;
    uint32_t escapes = 0;
    if (len == kTileWords && (t0 >= J.half || t0 + kTileWords <= J.half)) {
      // whole tile in one plane: no bounds, and the plane's escape table is a
      // constant offset (one copy of the loop per plane)
      auto scan = [&](auto plane, auto counting) {
        constexpr uint32_t kOff = decltype(plane)::kOffset;
        constexpr bool kCountHere = decltype(counting)::kValue;
#pragma unroll
        for (int s = 0; s < kStepsPerWarp; ++s) {
          const uint16_t* w = sin + (warp * kStepsPerWarp + s) * kStepWords + 8 * lane;
          const uint4 v0 = *reinterpret_cast<const uint4*>(w);
          const uint4 v1 = *reinterpret_cast<const uint4*>(w + 256);
          const uint32_t x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
          if (!kStats) {
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              const uint32_t y = x[p] ^ ((x[p] >> 5) & 0x04000400u);
              spres[__byte_perm(y, 0, 0x4441)] = 1;
              spres[y >> 24] = 1;
            }
          } else {
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              // stats_index of both words at once: bits 7..15 (even word), 23..31 (odd)
              const uint32_t y = x[p] ^ ((x[p] >> 2) & 0x20002000u);
              const uint32_t e = (y >> 7) & 0x1FFu, o = y >> 23;
              if (kPresence) {
                spres[e] = 1;
                spres[o] = 1;
              }
              if (kCountHere) escapes += sesc[kOff + e] + sesc[kOff + o];
            }
          }
        }
      };
      // one copy of the loop per plane and per counting choice: a tile that
      // does not count issues no escape-table loads at all
      if (!count)
        scan(StatsPlane<0>{}, CompileFlag<false>{});
      else if (t0 < J.half)
        scan(StatsPlane<0>{}, CompileFlag<true>{});
      else
        scan(StatsPlane<512>{}, CompileFlag<true>{});
    } else {
#pragma unroll
      for (int s = 0; s < kStepsPerWarp; ++s) {
        const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
        if (w0 >= len) continue;
        const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
        const uint64_t g = t0 + w0;
        for (uint32_t i = 0; i < valid; ++i) {
          const uint32_t w = sin[w0 + i];
          if (!kStats) {
            spres[presence_index(w >> 8)] = 1;
          } else {
            const uint32_t si = stats_index(w >> 7);
            if (kPresence) spres[si] = 1;
            if (count) escapes += sesc[((g + i) >= J.half ? 512 : 0) + si];
          }
        }
      }
    }
    if (kKind == kStatsTop16Rec) {
      // every warp writes its count (the record is not cleared beforehand);
      // after a wait that ran out it writes a count no run can have (a run
      // holds at most kStepsPerWarp * kStepWords = 2048 words), which the
      // scan turns into a mode-255 header
      escapes = warp_sum(escapes);
      if (lane == 0) {
        const uint64_t off = top16_record_offset(reinterpret_cast<uint64_t>(J.dst), J.n, tile);
        if (off != kTailRecord)
          reinterpret_cast<uint16_t*>(J.dst + off)[warp] = pos.late ? 0xFFFFu : static_cast<uint16_t>(escapes);
        else if (warp == 0)
          st_u32_bytes(J.dst + top16_tail_offset(J.n), pos.late ? 0xFFFFFFFFu : escapes);
      }
    } else if (count) {
      escapes = warp_sum(escapes);
      if (lane == 0 && escapes) {
        uint64_t* groups = reinterpret_cast<uint64_t*>(J.scratch + 64);
        uint16_t* counts = reinterpret_cast<uint16_t*>(J.scratch + auto_counts_offset(J.tiles));
        counts[tile * kWarps + warp] = static_cast<uint16_t>(escapes);
        atomicAdd(reinterpret_cast<unsigned long long*>(&groups[tile >> 5]), static_cast<unsigned long long>(escapes));
        atomicAdd(reinterpret_cast<uint32_t*>(J.scratch), escapes);
      }
    }
  }, over_cap);
  if (warp == kProducerWarp || !kPresence) return;
  consumer_sync();
  if (pres_job >= 0) flush(b.job[pres_job]);
}

// ------------------------------------------------------------ fixed encode

// Palette rank of every high byte from a 256-bit presence bitmap (ascending
// order) into srank[rank_slot(h)]; thread tid handles high byte tid.  The
// slot copies the sign (bit 7) into bit 5, so a positive and a negative high
// byte of the same magnitude sit 8 banks apart: a warp's lookups of +e and
// -e do not collide.  rank_words applies the same swap to both words of a
// pair at once, ahead of the byte extraction.
__device__ __forceinline__ uint32_t rank_slot(uint32_t h) { return h ^ ((h >> 2) & 0x20u); }
__device__ __forceinline__ uint32_t rank_words(uint32_t x) { return x ^ ((x >> 2) & 0x20002000u); }
__device__ __forceinline__ void palette_ranks(const uint32_t* bitmap, uint8_t* srank, uint32_t& distinct,
                                              bool& present, uint32_t& rank) {
  const int tid = threadIdx.x;
  uint32_t bm[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) bm[w] = bitmap[w];
  distinct = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) distinct += __popc(bm[w]);
  const uint32_t word = bm[tid >> 5];
  present = (word >> (tid & 31)) & 1u;
  rank = __popc(word & ((1u << (tid & 31)) - 1u));
#pragma unroll
  for (int w = 0; w < 8; ++w)
    if (w < (tid >> 5)) rank += __popc(bm[w]);
  srank[rank_slot(tid)] = static_cast<uint8_t>(rank);
}

// Header + palette of a fixed stream (written by one CTA).
template <int kBits>
__device__ __forceinline__ void write_fixed_header(uint8_t* dst, uint32_t distinct, bool present,
                                                   uint32_t rank, bool error) {
  constexpr uint32_t kLimit = kBits == 6 ? 64 : 32;
  const int tid = threadIdx.x;
  if (present && rank < kLimit) dst[1 + rank] = static_cast<uint8_t>(tid);
  if (tid >= static_cast<int>(distinct) && tid < static_cast<int>(kLimit)) dst[1 + tid] = 0;
  if (tid == 0) dst[0] = (distinct > kLimit || error) ? 255 : (kBits == 6 ? 3 : 4);
}

// A full fixed6 tile: each warp codes its run of kStepsPerWarp steps, then
// stores the run's low bytes and its codes as two contiguous runs.
__device__ __forceinline__ void fixed6_tile_full(const EncJob& J, uint64_t t0, const uint16_t* sin,
                                                 const uint8_t* srank) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint32_t low[kStepsPerWarp][4];
  uint32_t qw[kStepsPerWarp][3];
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    // the lane's 16 words are 32 bytes: lanes 4-7 of each quarter warp load
    // their second 16 bytes first, so that each 16-byte load instruction of
    // a quarter warp covers all 32 banks once; the halves' results are put
    // back in word order with selects
    const bool sw = (lane & 4) != 0;
    const uint4* pu = reinterpret_cast<const uint4*>(sin + w0);
    const uint4 va = pu[sw ? 1 : 0];
    const uint4 vb = pu[sw ? 0 : 1];
    const uint32_t xh[2][4] = {{va.x, va.y, va.z, va.w}, {vb.x, vb.y, vb.z, vb.w}};
    uint32_t lh[2][2], gh[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        lh[h][q] = __byte_perm(xh[h][2 * q], xh[h][2 * q + 1], 0x6420);
        const uint32_t y0 = rank_words(xh[h][2 * q]), y1 = rank_words(xh[h][2 * q + 1]);
        const uint32_t c0 = srank[__byte_perm(y0, 0, 0x4441)];
        const uint32_t c1 = srank[y0 >> 24];
        const uint32_t c2 = srank[__byte_perm(y1, 0, 0x4441)];
        const uint32_t c3 = srank[y1 >> 24];
        gh[h][q] = c0 | (c1 << 6) | (c2 << 12) | (c3 << 18);
      }
    }
    uint32_t g[4];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      low[s][q] = sw ? lh[1][q] : lh[0][q];
      low[s][2 + q] = sw ? lh[0][q] : lh[1][q];
      g[q] = sw ? gh[1][q] : gh[0][q];
      g[2 + q] = sw ? gh[0][q] : gh[1][q];
    }
    qw[s][0] = g[0] | (g[1] << 24);
    qw[s][1] = (g[1] >> 8) | (g[2] << 16);
    qw[s][2] = (g[2] >> 16) | (g[3] << 8);
  }
  const uint64_t r0 = t0 + static_cast<uint64_t>(warp) * kStepsPerWarp * kStepWords;
  warp_store_run<4, 8, kStepsPerWarp>(J.dst + 65 + r0, low, lane);
  warp_store_run<3, 4, kStepsPerWarp>(J.dst + 65 + J.n + 3 * r0 / 4, qw, lane);
}

template <int kBits>
__device__ __forceinline__ void fixed_tile_body(const EncJob& J, uint64_t t0, uint32_t len,
                                                const uint16_t* sin, const uint8_t* srank) {
  constexpr uint32_t kHeader = kBits == 6 ? 65 : 33;
  if (kBits == 6 && len == kTileWords) {
    fixed6_tile_full(J, t0, sin, srank);
    return;
  }
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = step_valid_words(len, sb);
    if (step_valid == 0) continue;
    uint32_t x[8];
    load_unit(sin, w0, x);
    uint32_t low[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) low[q] = __byte_perm(x[2 * q], x[2 * q + 1], 0x6420);
    uint32_t c[16];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const uint32_t y = rank_words(x[p]);
      c[2 * p] = srank[__byte_perm(y, 0, 0x4441)];
      c[2 * p + 1] = srank[y >> 24];
    }
    const bool full = step_valid == kStepWords;
    if (!full) {
      const uint32_t valid = w0 < len ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i >= static_cast<int>(valid)) c[i] = 0;
    }
    uint8_t* ldst = J.dst + kHeader + t0 + sb;
    if (full) {
      warp_store_words<4, 8>(ldst, low, lane);
    } else {
      const uint64_t lowd[2] = {low[0] | (static_cast<uint64_t>(low[1]) << 32),
                                low[2] | (static_cast<uint64_t>(low[3]) << 32)};
      warp_store<uint64_t, 2>(ldst, step_valid, lowd, lane);
    }
    if (kBits == 6) {
      uint32_t g[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) g[q] = c[4 * q] + c[4 * q + 1] * 64u + c[4 * q + 2] * 4096u + c[4 * q + 3] * 262144u;
      const uint32_t qw[3] = {g[0] | (g[1] << 24), (g[1] >> 8) | (g[2] << 16), (g[2] >> 16) | (g[3] << 8)};
      uint8_t* cdst = J.dst + kHeader + J.n + 3 * (t0 + sb) / 4;
      if (full) warp_store_words<3, 4>(cdst, qw, lane);
      else warp_store<uint32_t, 3>(cdst, 3 * ((step_valid + 3) / 4), qw, lane);
    } else {
      uint64_t lo = 0;
      uint32_t hi = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int bit = 5 * i;
        if (bit + 5 <= 64) {
          lo |= static_cast<uint64_t>(c[i]) << bit;
        } else if (bit >= 64) {
          hi |= c[i] << (bit - 64);
        } else {
          lo |= static_cast<uint64_t>(c[i]) << bit;
          hi |= c[i] >> (64 - bit);
        }
      }
      const uint16_t qh[5] = {static_cast<uint16_t>(lo), static_cast<uint16_t>(lo >> 16),
                              static_cast<uint16_t>(lo >> 32), static_cast<uint16_t>(lo >> 48),
                              static_cast<uint16_t>(hi)};
      uint8_t* cdst = J.dst + kHeader + J.n + 5 * (t0 + sb) / 8;
      if (full) warp_store_full<uint16_t, 5>(cdst, qh, lane);
      else warp_store<uint16_t, 5>(cdst, 5 * ((step_valid + 7) / 8), qh, lane);
    }
  }
}

template <int kMax, int kBits>
__global__ void __launch_bounds__(kCtaThreads, 3) EncodeFixedKernel(const __grid_constant__ EncBatch<kMax> b) {
  constexpr uint32_t kLimit = kBits == 6 ? 64 : 32;
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint8_t srank[256];
  __shared__ EncRing R;
  __shared__ EncDesc D[kEncStages];
  ring_init(R);
  __syncthreads();
  grid_dependency_sync();
  int rank_job = -1;
  bool skip = false;
  encode_pipeline<kMax>(b, ring, R, D, [&](const EncJob& J, int j, uint32_t tile, const uint16_t* sin,
                                           const EncPos& pos, const EncDesc&) {
    if (pos.late && (threadIdx.x & 31) == 0) mark_stream_late(J);
    if (j != rank_job) {  // uniform across the consumers
      consumer_sync();    // every warp is done with the previous ranks
      uint32_t distinct, rank;
      bool present;
      palette_ranks(reinterpret_cast<const uint32_t*>(J.scratch), srank, distinct, present, rank);
      uint32_t* error = reinterpret_cast<uint32_t*>(J.scratch + 32);
      if (tile == 0) {
        write_fixed_header<kBits>(J.dst, distinct, present, rank, ld_volatile_u32(error) != 0);
        if (threadIdx.x == 0) recheck_header(J);
      }
      skip = distinct > kLimit;
      rank_job = j;
      consumer_sync();
    }
    if (skip) return;  // palette overflow: header only (uniform across the job)
    const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
    fixed_tile_body<kBits>(J, t0, tile_len(J.n, t0), sin, srank);
  });
  // a job whose tile 0 this CTA did not see still needs its header: the
  // owner of tile 0 wrote it (tile 0 is always the first tile of some chunk
  // or preceded by the same job's tiles in the same chunk).
}

// ------------------------------------------------------------- auto encode

// Raw mode 6: [6] + the words little endian.
__device__ __forceinline__ void raw_tile_body(const EncJob& J, uint64_t t0, uint32_t len,
                                              const uint16_t* sin) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (len == kTileWords) {
    uint32_t x[kStepsPerWarp][8];
#pragma unroll
    for (int s = 0; s < kStepsPerWarp; ++s)
      load_unit(sin, (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords, x[s]);
    const uint64_t r0 = t0 + static_cast<uint64_t>(warp) * kStepsPerWarp * kStepWords;
    warp_store_run<8, 8, kStepsPerWarp>(J.dst + 1 + 2 * r0, x, lane);
    return;
  }
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = step_valid_words(len, sb);
    if (step_valid == 0) continue;
    uint32_t x[8];
    load_unit(sin, w0, x);
    if (step_valid == kStepWords) {
      warp_store_words<8, 8>(J.dst + 1 + 2 * (t0 + sb), x, lane);
    } else {
      const uint64_t d[4] = {x[0] | (static_cast<uint64_t>(x[1]) << 32), x[2] | (static_cast<uint64_t>(x[3]) << 32),
                             x[4] | (static_cast<uint64_t>(x[5]) << 32), x[6] | (static_cast<uint64_t>(x[7]) << 32)};
      warp_store<uint64_t, 4>(J.dst + 1 + 2 * (t0 + sb), 2 * step_valid, d, lane);
    }
  }
}

// Kinds decided on the device from the stats pass, in the reference's
// fallback order (vllm_connector.py:3104-3118, 4557-4633): top16 if the
// escapes fit, else fixed6 if <= 64 high bytes, else raw mode 6 when the
// buffer holds it, else a fixed6 overflow stream (mode 255) for the host.
// The top16 variants (the explicit top16 encode) code every job as top16;
// one whose escapes exceed its capacity gets the reference's overflow form
// (mode byte 255, count = cap, the first cap escapes).  kEncTop16Scratch
// follows a kStatsTop16 pass (counts in the scratch array); kEncTop16Rec
// follows kStatsTop16Rec + Top16ScanKernel (per-tile records in the stream,
// header already written).
enum AutoKind { kAutoTop16 = 0, kAutoFixed6 = 1, kAutoRaw = 2, kAutoOverflow = 3 };
enum EncVariant { kEncAuto = 0, kEncTop16Scratch = 1, kEncTop16Rec = 2 };

template <int kMax, int kVariant>
__global__ void __launch_bounds__(kCtaThreads, 3) EncodeAutoKernel(const __grid_constant__ EncBatch<kMax> b) {
  constexpr bool kTop16Only = kVariant != kEncAuto;
  constexpr bool kRec = kVariant == kEncTop16Rec;
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint32_t stbl[512];
  __shared__ uint8_t srank[256];
  __shared__ EncRing R;
  __shared__ EncDesc D[kEncStages];
  const int tid = threadIdx.x;
  ring_init(R);
  __syncthreads();
  grid_dependency_sync();
  int setup_job = -1;
  int kind = kAutoOverflow;
  uint64_t escapes = 0;
  // top16 escape offsets from the stats pass, prepared by the producer warp
  // so that the consumers neither wait nor synchronise for them: the tile's
  // offset in the job and each warp's offset inside the tile.  Job-level
  // values are read once per job; consecutive tiles keep a running prefix
  // and a register window of 32 tiles' per-warp counts (one load round per
  // 32 tiles).  The producer also clears the tile's share of the unused
  // escape slots.
  const EncJob* hook_job = nullptr;
  uint32_t hook_next = 0, win_first = 0;
  bool hook_top16 = false;
  uint64_t running = 0, zlo0 = 0, zhi = 0, zshare = 0;
  uint4 win = make_uint4(0, 0, 0, 0);
  auto prefix_hook = [&](const EncJob& J, uint32_t tile, EncDesc& d) {
    const int lane = threadIdx.x & 31;
    if constexpr (kRec) {
      if (&J != hook_job) {
        hook_job = &J;
        // the scan pass wrote the header: count = min(escapes, cap)
        zlo0 = 5ull * ld_u32_bytes(J.dst + 1);
        zhi = 5 * J.cap;
        zshare = zlo0 < zhi ? (zhi - zlo0 + J.tiles - 1) / J.tiles : 0;
      }
      const uint64_t off = top16_record_offset(reinterpret_cast<uint64_t>(J.dst), J.n, tile);
      uint32_t wpre = 0;
      uint32_t prefix;
      if (off == kTailRecord) {
        prefix = ld_u32_bytes(J.dst + top16_tail_offset(J.n));
      } else {
        if (lane < kWarps) wpre = reinterpret_cast<const uint16_t*>(J.dst + off)[lane];
        prefix = *reinterpret_cast<const uint32_t*>(J.dst + off + 16);
      }
      if (lane == 0) d.prefix = prefix;
      if (lane < kWarps) d.wpre[lane] = wpre;
      uint8_t* entries = J.dst + 5 + J.n + (J.n + 1) / 2;
      const uint64_t a = min(zhi, zlo0 + zshare * tile);
      const uint64_t e = min(zhi, a + zshare);
      for (uint64_t i = a + lane; i < e; i += 32) entries[i] = 0;
      return;
    }
    const uint16_t* counts = reinterpret_cast<const uint16_t*>(J.scratch + auto_counts_offset(J.tiles));
    auto load_win = [&](uint32_t first) {
      win_first = first;
      const uint32_t t = first + lane;
      win = t < J.tiles ? *reinterpret_cast<const uint4*>(counts + static_cast<uint64_t>(t) * kWarps)
                        : make_uint4(0, 0, 0, 0);
    };
    if (&J != hook_job || tile != hook_next) {
      hook_job = &J;
      const uint64_t escapes = *reinterpret_cast<const uint32_t*>(J.scratch);
      // the consumers' choice of kind: top16 unless the stats pass failed
      hook_top16 = kTop16Only ||
                   (escapes <= J.cap && ld_volatile_u32(reinterpret_cast<const uint32_t*>(J.scratch + 4)) == 0);
      zlo0 = 5 * escapes;
      zhi = 5 * J.cap;
      zshare = hook_top16 && zlo0 < zhi ? (zhi - zlo0 + J.tiles - 1) / J.tiles : 0;
      running = 0;
      if (hook_top16) {
        const uint64_t* groups = reinterpret_cast<const uint64_t*>(J.scratch + 64);
        const uint32_t g = tile >> 5;
        uint64_t v = 0;
        if (lane < static_cast<int>(tile & 31)) {
          const uint4 c = *reinterpret_cast<const uint4*>(counts + ((g << 5) + lane) * kWarps);
          const uint32_t pairs = (c.x + c.y) + (c.z + c.w);  // two u16 sums per word, each < 2^16
          v = (pairs & 0xFFFFu) + (pairs >> 16);
        }
        running = warp_sum(v);
        for (uint32_t base = 0; base < g; base += 32) {
          v = base + lane < g ? (groups[base + lane] & 0xFFFFFFFFull) : 0;
          running += warp_sum(v);
        }
        load_win(tile);
      }
    }
    uint32_t wpre = 0;
    uint64_t prefix = running;
    if (hook_top16) {
      if (tile - win_first >= 32) load_win(tile);
      const int k = static_cast<int>(tile - win_first);
      const uint32_t c[4] = {__shfl_sync(kFull, win.x, k), __shfl_sync(kFull, win.y, k),
                             __shfl_sync(kFull, win.z, k), __shfl_sync(kFull, win.w, k)};
      uint32_t total = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        if (w == lane) wpre = total;
        total += (c[w >> 1] >> (16 * (w & 1))) & 0xFFFFu;
      }
      running += total;
    }
    hook_next = tile + 1;
    if (lane == 0) d.prefix = prefix;
    if (lane < kWarps) d.wpre[lane] = wpre;
    // the tile's share of the unused escape slots, cleared here (no consumer
    // writes them)
    uint8_t* entries = J.dst + 5 + J.n + (J.n + 1) / 2;
    const uint64_t a = min(zhi, zlo0 + zshare * tile);
    const uint64_t e = min(zhi, a + zshare);
    for (uint64_t i = a + lane; i < e; i += 32) entries[i] = 0;
  };
  encode_pipeline<kMax>(b, ring, R, D, [&](const EncJob& J, int j, uint32_t tile, const uint16_t* sin,
                                           const EncPos& pos, const EncDesc& desc) {
    if (pos.late && (tid & 31) == 0) mark_stream_late(J);
    if (j != setup_job) {  // uniform across the consumers
      consumer_sync();     // every warp is done with the previous ranks/table
      uint32_t distinct = 0, rank = 0;
      bool present = false;
      if (!kTop16Only) palette_ranks(reinterpret_cast<const uint32_t*>(J.scratch + 16), srank, distinct, present, rank);
      escapes = kRec ? 0 : *reinterpret_cast<const uint32_t*>(J.scratch);
      const bool err = !kRec && ld_volatile_u32(reinterpret_cast<const uint32_t*>(J.scratch + 4)) != 0;
      kind = kTop16Only ? kAutoTop16
           : err ? kAutoOverflow
           : escapes <= J.cap ? kAutoTop16
           : distinct <= 64 ? kAutoFixed6
           : J.raw_ok ? kAutoRaw : kAutoOverflow;
      if (tile == 0 || setup_job < 0) {
        // the CTA holding tile 0 writes the header
        if (tile == 0) {
          if (kTop16Only) {
            if (!kRec && tid == 0) write_top16_header(J.dst, escapes, J.cap, err);
          } else if (kind == kAutoOverflow) write_fixed_header<6>(J.dst, distinct > 64 ? distinct : 65, present, rank, true);
          else if (kind == kAutoFixed6) write_fixed_header<6>(J.dst, distinct, present, rank, false);
          else if (kind == kAutoRaw && tid == 0) J.dst[0] = 6;
          else if (kind == kAutoTop16 && tid == 0) write_top16_header(J.dst, escapes, J.cap, false);
          if (tid == 0) recheck_header(J);
        }
      }
      if (kind == kAutoTop16) load_top16_table(J.tables, stbl);
      setup_job = j;
      consumer_sync();
    }
    const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
    const uint32_t len = tile_len(J.n, t0);
    if (kind == kAutoOverflow) return;
    if (kind == kAutoFixed6) {
      fixed_tile_body<6>(J, t0, len, sin, srank);
      return;
    }
    if (kind == kAutoRaw) {
      raw_tile_body(J, t0, len, sin);
      return;
    }
    // top16: this warp's escapes start at desc.prefix + desc.wpre[warp]
    uint32_t masks[kStepsPerWarp];
    top16_tile_body(J, t0, len, sin, stbl, masks);
    warp_write_escapes(J, t0, sin, masks, desc.prefix + desc.wpre[tid >> 5]);
  }, prefix_hook);
}

// Exclusive scan of the per-tile escape counts of each job (one CTA per
// job), between the kStatsTop16Rec pass and EncodeAutoKernel<., kEncTop16Rec>:
// every record gets the escapes of the job before its tile and of the tile
// before each warp's run, and thread 0 writes the stream header (mode 5, or
// 255 when the escapes exceed the capacity or a wait of the stats pass ran
// out; the count clamped to the capacity).
constexpr int kScanThreads = 256;
constexpr int kScanTilesPerThread = 4;

template <int kMax>
__global__ void __launch_bounds__(kScanThreads) Top16ScanKernel(const __grid_constant__ EncBatch<kMax> b) {
  __shared__ uint32_t wsum[kScanThreads / 32];
  grid_dependency_sync();
  const uint32_t j = blockIdx.x;
  if (j >= b.jobs) return;
  const EncJob& J = b.job[j];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint64_t addr = reinterpret_cast<uint64_t>(J.dst);
  constexpr uint32_t kChunk = kScanThreads * kScanTilesPerThread;
  uint32_t carry = 0;
  bool failed = false;
  for (uint32_t base = 0; base < J.tiles; base += kChunk) {
    // this thread's kScanTilesPerThread consecutive tiles
    uint32_t tot[kScanTilesPerThread];
    uint4 rec[kScanTilesPerThread];
    uint64_t off[kScanTilesPerThread];
    uint32_t mine = 0;
    bool bad = false;  // a count no warp run can have: a wait of the stats pass ran out
#pragma unroll
    for (int k = 0; k < kScanTilesPerThread; ++k) {
      const uint32_t t = base + tid * kScanTilesPerThread + k;
      rec[k] = make_uint4(0, 0, 0, 0);
      off[k] = kTailRecord;
      tot[k] = 0;
      if (t < J.tiles) {
        off[k] = top16_record_offset(addr, J.n, t);
        if (off[k] != kTailRecord) {
          rec[k] = *reinterpret_cast<const uint4*>(J.dst + off[k]);
          const uint32_t w[4] = {rec[k].x, rec[k].y, rec[k].z, rec[k].w};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            bad |= (w[q] & 0xFFFFu) > kStepsPerWarp * kStepWords || (w[q] >> 16) > kStepsPerWarp * kStepWords;
          const uint32_t pairs = (rec[k].x + rec[k].y) + (rec[k].z + rec[k].w);  // two u16 sums, each < 2^16
          tot[k] = (pairs & 0xFFFFu) + (pairs >> 16);
        } else {
          tot[k] = ld_u32_bytes(J.dst + top16_tail_offset(J.n));
          bad |= tot[k] > kStepsPerWarp * kStepWords;
        }
      }
      mine += tot[k];
    }
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    uint32_t before = carry, chunk = 0;
#pragma unroll
    for (int w = 0; w < kScanThreads / 32; ++w) {
      if (w < warp) before += wsum[w];
      chunk += wsum[w];
    }
    before += incl - mine;
#pragma unroll
    for (int k = 0; k < kScanTilesPerThread; ++k) {
      const uint32_t t = base + tid * kScanTilesPerThread + k;
      if (t < J.tiles) {
        if (off[k] != kTailRecord) {
          // escapes of the tile before each warp's run, as u16
          const uint32_t c[kWarps] = {rec[k].x & 0xFFFFu, rec[k].x >> 16, rec[k].y & 0xFFFFu, rec[k].y >> 16,
                                      rec[k].z & 0xFFFFu, rec[k].z >> 16, rec[k].w & 0xFFFFu, rec[k].w >> 16};
          uint32_t p[kWarps];
          uint32_t run = 0;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) {
            p[w] = run;
            run += c[w];
          }
          *reinterpret_cast<uint4*>(J.dst + off[k]) =
              make_uint4(p[0] | (p[1] << 16), p[2] | (p[3] << 16), p[4] | (p[5] << 16), p[6] | (p[7] << 16));
          *reinterpret_cast<uint32_t*>(J.dst + off[k] + 16) = before;
        } else {
          st_u32_bytes(J.dst + top16_tail_offset(J.n), before);
        }
      }
      before += tot[k];
    }
    carry += chunk;
    failed |= __syncthreads_or(bad) != 0;  // also: wsum is reused by the next chunk
  }
  if (tid == 0) write_top16_header(J.dst, carry, J.cap, failed);
}

// ------------------------------------------------------------ calibration
//
// Exponent histogram of each job's words per plane: counter
// plane * 256 + ((w >> 7) & 0xFF) of the job's 2 x 256 u32 counters (EncJob::dst)
// grows by the words with that exponent byte; counts accumulate over calls.
// The reference computes the same counts with torch.bincount on the packed
// layer for its trace (vllm_connector.py:2871-2904) and ranks them into the
// top16 codebooks (trace.py:27-58).  Here the gather is fused: the producer
// warp stages the job's tiles from the paged cache by TMA, and each consumer
// warp counts into its own shared histogram with shared-memory atomics,
// adding its nonzero bins to the job's counters when its job changes and at
// the end (no CTA-wide synchronisation).
template <int kMax>
__global__ void __launch_bounds__(kCtaThreads, 2) ExpHistogramKernel(const __grid_constant__ EncBatch<kMax> b) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint32_t whist[kWarps][512];
  __shared__ EncRing R;
  __shared__ EncDesc D[kEncStages];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  for (int i = tid; i < kWarps * 512; i += kCtaThreads) (&whist[0][0])[i] = 0;
  ring_init(R);
  __syncthreads();
  grid_dependency_sync();
  uint32_t* mine = whist[warp & (kWarps - 1)];
  int hist_job = -1;
  auto flush = [&](const EncJob& P) {
    __syncwarp();
    uint32_t* out = reinterpret_cast<uint32_t*>(P.dst);
    for (int i = lane; i < 512; i += 32) {
      const uint32_t c = mine[i];
      if (c) {
        atomicAdd(out + i, c);
        mine[i] = 0;
      }
    }
    __syncwarp();
  };
  encode_pipeline<kMax>(b, ring, R, D, [&](const EncJob& J, int j, uint32_t tile, const uint16_t* sin,
                                           const EncPos&, const EncDesc&) {
    if (j != hist_job) {
      if (hist_job >= 0) flush(b.job[hist_job]);
      hist_job = j;
    }
    const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
    const uint32_t len = tile_len(J.n, t0);
    if (len == kTileWords && (t0 >= J.half || t0 + kTileWords <= J.half)) {
      const uint32_t poff = t0 >= J.half ? 256u : 0u;
#pragma unroll
      for (int s = 0; s < kStepsPerWarp; ++s) {
        const uint16_t* w = sin + (warp * kStepsPerWarp + s) * kStepWords + 8 * lane;
        const uint4 v0 = *reinterpret_cast<const uint4*>(w);
        const uint4 v1 = *reinterpret_cast<const uint4*>(w + 256);
        const uint32_t x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          atomicAdd(mine + (((x[q] >> 7) & 0xFFu) | poff), 1u);
          atomicAdd(mine + (((x[q] >> 23) & 0xFFu) | poff), 1u);
        }
      }
    } else {
#pragma unroll
      for (int s = 0; s < kStepsPerWarp; ++s) {
        const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
        if (w0 >= len) continue;
        const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
        const uint64_t g = t0 + w0;
        for (uint32_t i = 0; i < valid; ++i)
          atomicAdd(mine + (((g + i) >= J.half ? 256u : 0u) | ((sin[w0 + i] >> 7) & 0xFFu)), 1u);
      }
    }
  });
  if (warp == kProducerWarp) return;
  if (hist_job >= 0) flush(b.job[hist_job]);
}

// Top16 tables from exponent histograms, one CTA per layer: per plane the
// 16 most frequent observed exponents ranked by (-count, exponent), code =
// rank (trace.py:30-33, scripts/extract_llama_top16_codebooks.py:39-40),
// then the layer's 544-byte table as the reference builds it from its
// codebooks (splitzip_cuda.py:283-298): [0,256) K exponent -> code (255 =
// escape), [256,512) V, [512,528) K codebook, [528,544) V codebook.
// observed[2 layer + plane] = exponents with a nonzero count; with fewer
// than 16 the remaining codes take the unobserved exponents in ascending
// order (the reference's extractor rejects such a layer; the host decides).
__global__ void __launch_bounds__(256) Top16TablesKernel(const uint32_t* __restrict__ hist, uint32_t layers,
                                                         uint8_t* tables, uint32_t* observed) {
  __shared__ uint32_t cnt[256];
  __shared__ uint8_t book[16];
  const uint32_t layer = blockIdx.x;
  if (layer >= layers) return;
  const int e = threadIdx.x;
  uint8_t* T = tables + static_cast<uint64_t>(layer) * 544;
  for (int plane = 0; plane < 2; ++plane) {
    cnt[e] = hist[(static_cast<uint64_t>(layer) * 2 + plane) * 256 + e];
    __syncthreads();
    const uint32_t c = cnt[e];
    uint32_t rank = 0, below_unseen = 0, seen = 0;
    for (int k = 0; k < 256; ++k) {
      const uint32_t ck = cnt[k];
      rank += (ck > c) || (ck == c && k < e);
      below_unseen += ck == 0 && k < e;
      seen += ck != 0;
    }
    if (c > 0 && rank < 16) book[rank] = static_cast<uint8_t>(e);
    if (c == 0 && seen + below_unseen < 16) book[seen + below_unseen] = static_cast<uint8_t>(e);
    T[plane * 256 + e] = 255;
    if (e == 0) observed[layer * 2 + plane] = seen;
    __syncthreads();
    if (e < 16) {
      T[plane * 256 + book[e]] = static_cast<uint8_t>(e);
      T[512 + plane * 16 + e] = book[e];
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ decode
//
// Producer warp per tile: reads the job's mode byte (once per job), stages
// the tile's stream bytes by TMA, resolves the destination of each 512-word
// step in the paged cache (one block-table load per step, off the
// consumers' path) and, for top16, gathers the tile's escapes into the
// stage descriptor.  Consumer warps: codes -> 16 words per lane -> two
// 16-byte stores per lane at the resolved step address.

constexpr uint32_t kStepsPerTile = kTileWords / kStepWords;
static_assert(kStepsPerTile <= 32, "the producer's lanes resolve one step each");

// Decode stage descriptor, written by the producer warp.
struct DecDesc {
  uint32_t tile;   // global tile index, or kEndTile
  uint32_t job;
  uint32_t mode;   // stream mode of the job; 0: leave the tile alone
  uint32_t pad_x;  // offset of the body / low / raw bytes in the stage
  uint32_t pad_y;  // offset of the codes in the stage's codes region
  uint32_t unused;
  uint16_t* step_dst[kStepsPerTile];   // 16-byte aligned contiguous destination of a step, or null
};

// fixed6 pair table of the consumers' current job: the high bytes of a word
// pair whose codes are c0 and c1, pal[c0] | pal[c1] << 8, as 16 bits at
// entry (c0 | c1 << 6) ^ ((c1 & 31) << 1).  The swizzle spreads the lanes of
// a warp that share c0 over the banks by c1 (a warp's code pairs share c0
// often: the palette ranks of one layer are few), and a 2-byte entry merges
// with the pair's low bytes in one byte permute.
struct DecodeExtra {
  uint8_t pal[64];
  uint16_t pair[4096];
};

// Destination of the 16-word unit at packed index g (valid words `valid`).
__device__ __forceinline__ void store_unit(uint16_t* dst, const Layout& L, uint64_t g, uint32_t valid,
                                           const uint32_t (&o)[8], bool vec) {
  if (vec && valid == kUnitWords) {
    uint4* p = reinterpret_cast<uint4*>(dst + layout_addr(L, g));
    p[0] = make_uint4(o[0], o[1], o[2], o[3]);
    p[1] = make_uint4(o[4], o[5], o[6], o[7]);
  } else {
#pragma unroll
    for (uint32_t i = 0; i < kUnitWords; ++i)
      if (i < valid) dst[layout_addr(L, g + i)] = static_cast<uint16_t>(o[i >> 1] >> ((i & 1) * 16));
  }
}

// Store this lane's unit of warp step `step`: two 16-byte stores at the
// step's resolved address, else through the layout word by word.
__device__ __forceinline__ void store_step(const DecJob& J, const DecDesc& d, uint64_t t0, uint32_t step,
                                           uint32_t valid, int lane, const uint32_t (&o)[8]) {
  uint16_t* q = d.step_dst[step];
  if (q != nullptr) {
    uint4* p = reinterpret_cast<uint4*>(q + lane * kUnitWords);
    p[0] = make_uint4(o[0], o[1], o[2], o[3]);
    p[1] = make_uint4(o[4], o[5], o[6], o[7]);
  } else if (valid) {
    store_unit(J.dst, J.L, t0 + step * kStepWords + lane * kUnitWords, valid, o, J.vec != 0);
  }
}

__device__ __forceinline__ uint32_t entry_pos(const uint8_t* entries, uint64_t idx) {
  return load_u32le(entries + idx * 5);
}

// prmt.b32 in its default mode: a selector nibble with bit 3 set replicates
// the sign bit of the selected byte.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Exponents of four consecutive words from their four 4-bit codes (`nib16`,
// first word in the low nibble) and a plane's 16-entry codebook held in four
// registers: two byte permutes pick book[c & 7] from bytes 0-7 and 8-15, a
// third turns each code's bit 3 into a byte mask.  No table in memory.
__device__ __forceinline__ uint32_t book_exps4(const uint32_t (&bk)[4], uint32_t nib16) {
  const uint32_t sel = nib16 & 0x7777u;
  const uint32_t lo = prmt(bk[0], bk[1], sel);
  const uint32_t hi = prmt(bk[2], bk[3], sel);
  const uint32_t m = prmt(nib16 << 4, nib16, 0xD9C8u);
  return (lo & ~m) | (hi & m);
}

// Producer lane 0: stage one tile's stream bytes into a ring stage (TMA
// bytes registered on `bar`, no arrive).  Returns the pads of the two regions.
__device__ __forceinline__ uint2 decode_stage(const DecJob& J, uint32_t mode, uint64_t t0, uint32_t len,
                                              uint8_t* stage, uint64_t* bar) {
  uint2 pad{0, 0};
  if (mode == 5) {
    pad.x = stage_bytes_one(J.src, J.src_bytes, 5 + t0, len, stage, bar);
    pad.y = stage_bytes_one(J.src, J.src_bytes, 5 + J.n + t0 / 2, (len + 1) / 2, stage + kDecCodesOffset, bar);
  } else if (mode == 3) {
    pad.x = stage_bytes_one(J.src, J.src_bytes, 65 + t0, len, stage, bar);
    pad.y = stage_bytes_one(J.src, J.src_bytes, 65 + J.n + 3 * t0 / 4, 3 * ((len + 3) / 4),
                            stage + kDecCodesOffset, bar);
  } else if (mode == 6) {
    pad.x = stage_bytes_one(J.src, J.src_bytes, 1 + 2 * t0, 2 * len, stage, bar);
  }
  return pad;
}

template <int kMode>
__device__ __forceinline__ uint32_t job_mode(const DecJob& J) {
  const uint32_t mode = __ldg(J.src);
  if (kMode != 0) return mode == static_cast<uint32_t>(kMode) ? mode : 0;
  uint64_t need = 0;
  if (mode == 5) need = 5 + J.n + (J.n + 1) / 2 + 5 * J.cap;
  else if (mode == 3) need = 65 + J.n + 3 * ((J.n + 3) / 4);
  else if (mode == 6) need = 1 + 2 * J.n;
  return (need == 0 || need > J.src_bytes) ? 0 : mode;
}

// Producer warp of DecodeKernel.  The next tile is planned (job, mode byte
// once per job, the block-table loads of its steps' destinations) before
// the current one waits for its stage, so those loads' latency overlaps the
// staging instead of sitting between two tiles' copies.
template <int kMax, int kMode>
__device__ __forceinline__ void decode_producer(const DecBatch<kMax>& b, uint8_t* ring, DecRing& R, DecDesc* D) {
  const int lane = threadIdx.x & 31;
  const Chunk c = cta_chunk(b.tile_start[b.jobs]);
  DecPos p;
  int ji = find_job<kMax>(b.tile_start, b.jobs, c.first);
  int mode_job = -1;
  uint32_t mode = 0;
  struct Planned {
    uint32_t t;
    int ji;
    uint32_t mode;
    uint32_t len;
    uint64_t t0;
    uint16_t* q;  // this lane's step destination (lanes < kStepsPerTile)
  };
  auto plan = [&](uint32_t t) {
    Planned x{t, ji, 0, 0, 0, nullptr};
    if (t >= c.last) return x;
    ji = advance_job<kMax>(b.tile_start, ji, t);
    const DecJob& N = b.job[ji];
    if (ji != mode_job) {
      mode = job_mode<kMode>(N);
      mode_job = ji;
    }
    x.ji = ji;
    x.mode = mode;
    x.t0 = static_cast<uint64_t>(t - b.tile_start[ji]) * kTileWords;
    x.len = tile_len(N.n, x.t0);
    if (lane < static_cast<int>(kStepsPerTile)) {
      const uint32_t sb = lane * kStepWords;
      if (mode != 0 && N.vec != 0 && sb + kStepWords <= x.len) {
        const uint64_t g = x.t0 + sb;
        if (layout_run(N.L, g) >= kStepWords) x.q = N.dst + layout_addr(N.L, g);
      }
    }
    return x;
  };
  Planned cur = plan(c.first);
  for (;;) {
    const Planned nxt = cur.t < c.last ? plan(cur.t + 1) : cur;
    producer_acquire(R, p, nullptr);
    DecDesc& d = D[p.s];
    if (cur.t >= c.last) {
      if (lane == 0) d.tile = kEndTile;
      producer_commit(R, p);
      return;
    }
    if (lane == 0) {
      const uint2 pad = decode_stage(b.job[cur.ji], cur.mode, cur.t0, cur.len, ring + p.s * kDecStageBytes,
                                     &R.full[p.s]);
      d.tile = cur.t;
      d.job = static_cast<uint32_t>(cur.ji);
      d.mode = cur.mode;
      d.pad_x = pad.x;
      d.pad_y = pad.y;
    }
    if (lane < static_cast<int>(kStepsPerTile)) d.step_dst[lane] = cur.q;
    producer_commit(R, p);
    p.next();
    cur = nxt;
  }
}

// Every word with its book exponent; EscapePatchKernel then rewrites the
// escaped words.
__device__ __forceinline__ void decode_top16_compute(const DecJob& J, const DecDesc& d, const uint8_t* stage,
                                                     uint64_t t0, uint32_t len, uint32_t hrel,
                                                     const uint32_t (&bk0)[4], const uint32_t (&bk1)[4]) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t pad_x = d.pad_x, pad_y = d.pad_y;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t step = warp * kStepsPerWarp + s;
    const uint32_t sb = step * kStepWords;
    if (sb >= len) continue;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t valid = w0 < len ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
    uint32_t B[4];
    smem_read16_window(stage, pad_x + w0, B);
    uint32_t C[2];
    smem_read8_window(stage + kDecCodesOffset, pad_y + w0 / 2, C);
    uint32_t e[4];  // exponents of words 4q..4q+3
    if (w0 >= hrel || w0 + kUnitWords <= hrel) {
      const bool p1 = w0 >= hrel;
      uint32_t bk[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) bk[k] = p1 ? bk1[k] : bk0[k];
#pragma unroll
      for (int q = 0; q < 4; ++q) e[q] = book_exps4(bk, (C[q >> 1] >> (16 * (q & 1))) & 0xFFFFu);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t nib = (C[q >> 1] >> (16 * (q & 1))) & 0xFFFFu;
        const uint32_t a = book_exps4(bk0, nib);
        const uint32_t b = book_exps4(bk1, nib);
        uint32_t m = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (w0 + 4 * q + k >= hrel) m |= 0xFFu << (8 * k);
        e[q] = (a & ~m) | (b & m);
      }
    }
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t body2 = __byte_perm(B[i >> 1], 0, (i & 1) ? 0x3322 : 0x1100);
      const uint32_t ex = __byte_perm(e[i >> 1], 0, (i & 1) ? 0x4342 : 0x4140) << 7;
      o[i] = (body2 & 0x807F807Fu) | ex;
    }
    store_step(J, d, t0, step, valid, lane, o);
  }
}

__device__ __forceinline__ void decode_fixed6_compute(const DecJob& J, const DecDesc& d, const uint8_t* stage,
                                                      uint64_t t0, uint32_t len, const DecodeExtra& X) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t pad_x = d.pad_x, pad_y = d.pad_y;
  const uint8_t* pair = reinterpret_cast<const uint8_t*>(X.pair);
  // byte offset of the swizzled entry of a 12-bit field held at bits 1..12
  auto swz = [](uint32_t fo) { return fo ^ ((fo >> 5) & 0x7Cu); };
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t step = warp * kStepsPerWarp + s;
    const uint32_t sb = step * kStepWords;
    if (sb >= len) continue;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t valid = w0 < len ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
    uint32_t Lw[4];
    smem_read16_window(stage, pad_x + w0, Lw);
    uint32_t Q[3];
    smem_read_words<3>(stage + kDecCodesOffset, pad_y + 3 * w0 / 4, Q);
    // byte offsets into the pair table of the 12-bit fields 12i..12i+11
    uint32_t f[8];
    f[0] = swz((Q[0] << 1) & 0x1FFEu);
    f[1] = swz((Q[0] >> 11) & 0x1FFEu);
    f[2] = swz(__funnelshift_r(Q[0], Q[1], 23) & 0x1FFEu);
    f[3] = swz((Q[1] >> 3) & 0x1FFEu);
    f[4] = swz((Q[1] >> 15) & 0x1FFEu);
    f[5] = swz(__funnelshift_r(Q[1], Q[2], 27) & 0x1FFEu);
    f[6] = swz((Q[2] >> 7) & 0x1FFEu);
    f[7] = swz((Q[2] >> 19) & 0x1FFEu);
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o[i] = __byte_perm(Lw[i >> 1], *reinterpret_cast<const uint16_t*>(pair + f[i]), (i & 1) ? 0x5342 : 0x5140);
    store_step(J, d, t0, step, valid, lane, o);
  }
}

__device__ __forceinline__ void decode_raw_compute(const DecJob& J, const DecDesc& d, const uint8_t* stage,
                                                   uint64_t t0, uint32_t len) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t pad_x = d.pad_x;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t step = warp * kStepsPerWarp + s;
    const uint32_t sb = step * kStepWords;
    if (sb >= len) continue;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t valid = w0 < len ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
    uint32_t o[8];
    smem_read_words<8>(stage, pad_x + 2 * w0, o);
    store_step(J, d, t0, step, valid, lane, o);
  }
}

// kMode: 5 = top16, 3 = fixed6, 0 = dispatch on each stream's mode byte.
template <int kMax, int kMode>
__global__ void __launch_bounds__(kCtaThreads, 3) DecodeKernel(const __grid_constant__ DecBatch<kMax> b) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(16) DecodeExtra X;
  __shared__ __align__(16) DecDesc D[kDecStages];
  __shared__ DecRing R;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  ring_init(R);
  __syncthreads();
  grid_dependency_sync();
  if (warp == kProducerWarp) {
    decode_producer<kMax, kMode>(b, ring, R, D);
    return;
  }
  int book_job = -1, pair_job = -1;
  uint32_t bk0[4] = {0, 0, 0, 0}, bk1[4] = {0, 0, 0, 0};  // top16 codebooks of book_job
  DecPos p;
  for (;;) {
    consumer_wait(R, p, nullptr);
    const DecDesc& d = D[p.s];
    const uint32_t t = d.tile;
    if (t == kEndTile) break;
    const uint32_t mode = d.mode;
    if (mode != 0) {  // uniform across the consumers
      const int ji = static_cast<int>(d.job);
      const DecJob& J = b.job[ji];
      const uint64_t t0 = static_cast<uint64_t>(t - b.tile_start[ji]) * kTileWords;
      const uint32_t len = tile_len(J.n, t0);
      const uint8_t* stage = ring + p.s * kDecStageBytes;
      if (mode == 5) {
        if (ji != book_job) {
          const uint8_t* books = J.tables + 512;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            bk0[k] = load_u32le(books + 4 * k);
            bk1[k] = load_u32le(books + 16 + 4 * k);
          }
          book_job = ji;
        }
        const uint32_t hrel =
            J.half <= t0 ? 0u : static_cast<uint32_t>(min(J.half - t0, static_cast<uint64_t>(kTileWords)));
        decode_top16_compute(J, d, stage, t0, len, hrel, bk0, bk1);
      } else if (mode == 3) {
        if (ji != pair_job) {
          consumer_sync();  // every warp is done with the previous table
          if (tid < 64) X.pal[tid] = __ldg(J.src + 1 + tid);
          consumer_sync();
          for (int i = tid; i < 4096; i += kThreads)
            X.pair[i ^ (((i >> 6) & 31) << 1)] =
                static_cast<uint16_t>(X.pal[i & 63] | (static_cast<uint32_t>(X.pal[i >> 6]) << 8));
          pair_job = ji;
          consumer_sync();
        }
        decode_fixed6_compute(J, d, stage, t0, len, X);
      } else {
        decode_raw_compute(J, d, stage, t0, len);
      }
    }
    consumer_release(R, p);
    p.next();
  }
}

// Runs after DecodeKernel in stream order: every escape entry of every top16
// job, one thread per entry (entry indices of a job run to its capacity
// ceil(n/200); those at or past the stream's count do nothing).  The decode
// wrote each word with its book exponent; the escaped word is rewritten
// from its body byte and the entry's exponent, which is what the
// reference's (w & 0x807F) | (exp << 7) patch of the decoded word gives
// (kvq_splitzip_cuda.cu:254-284).  Entries may come in any order; positions
// at or past n are skipped.
template <int kMax>
struct PatchBatch {
  uint32_t jobs;
  DecJob job[kMax];
};

template <int kMax, int kMode>
__global__ void __launch_bounds__(256) EscapePatchKernel(const __grid_constant__ PatchBatch<kMax> b) {
  // blockIdx.y is the job: every job's entries are patched at once; the
  // blocks of a job stride over the entries its stream holds
  grid_dependency_sync();
  const uint32_t j = blockIdx.y;
  if (j >= b.jobs) return;
  const DecJob& J = b.job[j];
  if (job_mode<kMode>(J) != 5) return;
  const uint64_t count = min(static_cast<uint64_t>(load_u32le(J.src + 1)), J.cap);
  const uint8_t* entries = J.src + 5 + J.n + (J.n + 1) / 2;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    const uint32_t q = entry_pos(entries, i);
    if (q >= J.n) continue;
    const uint32_t body = __ldg(J.src + 5 + q);
    const uint32_t w =
        (body & 0x7Fu) | ((body & 0x80u) << 8) | (static_cast<uint32_t>(__ldg(entries + i * 5 + 4)) << 7);
    J.dst[layout_addr(J.L, q)] = static_cast<uint16_t>(w);
  }
}

// ------------------------------------------------------------------- zero

// --------------------------------------------- receiver modes 0, 1, 2, 4
//
// Decode of the reference's torch-op streams (modes 0, 1, 2) and of fixed5
// (mode 4) into the paged cache, with the receiver's checks
// (vllm_connector.py:5168-5278; a stream that fails them leaves its blocks
// untouched).  Every plane of these forms holds a whole number of bytes per
// 16-word unit (16 codes of w bits are 2w bytes), so one thread decodes one
// unit from its bytes of each plane, read with aligned 4-byte loads that
// stay inside the stream; the mode and widths come through the read-only
// cache and each warp copies its job's palette into shared memory.  These
// forms are the receiver's fallbacks (the hot path is modes 5, 3 and 6), so
// this is a grid-stride kernel without a staging ring.

template <int kMax>
struct ModeBatch {
  uint32_t jobs;
  uint64_t unit_start[kMax + 1];
  DecJob job[kMax];
};

// Up to 16 bytes at p (nbytes of them defined) as a little-endian bit
// string in out[0..4] (out[4] = 0 pads the funnel shifts).
__device__ __forceinline__ void ldg_bytes16(const uint8_t* p, uint32_t nbytes, uint32_t (&out)[5]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  const uint32_t lead = static_cast<uint32_t>(a & 3);
  const uint32_t words = (lead + nbytes + 3) / 4;  // <= 5
  uint32_t v[6];
#pragma unroll
  for (int k = 0; k < 5; ++k) v[k] = static_cast<uint32_t>(k) < words ? __ldg(w + k) : 0u;
  v[5] = 0;
#pragma unroll
  for (int k = 0; k < 5; ++k) out[k] = __funnelshift_r(v[k], v[k + 1], 8 * lead);
}

// Field i (width w <= 8) of a bit string.
__device__ __forceinline__ uint32_t bit_field(const uint32_t (&bits)[5], uint32_t i, uint32_t w) {
  const uint32_t b = i * w, k = b >> 5;  // selects, not a dynamic index (keeps bits in registers)
  const uint32_t lo = k == 0 ? bits[0] : k == 1 ? bits[1] : k == 2 ? bits[2] : bits[3];
  const uint32_t hi = k == 0 ? bits[1] : k == 1 ? bits[2] : k == 2 ? bits[3] : bits[4];
  return __funnelshift_r(lo, hi, b & 31) & ((1u << w) - 1u);
}

__device__ __forceinline__ uint64_t plane_bytes(uint64_t n, uint32_t w) { return (n * w + 7) / 8; }

// High bytes of a unit's 16 words from their W-bit codes (W a constant, so
// every field is a fixed funnel shift) through a palette in shared memory.
template <int W>
__device__ __forceinline__ void palette_his(const uint32_t (&c)[5], const uint8_t* pal, uint32_t (&hi)[kUnitWords]) {
#pragma unroll
  for (int i = 0; i < kUnitWords; ++i) hi[i] = pal[bit_field(c, i, W)];
}

__device__ __forceinline__ void palette_his(uint32_t w, const uint32_t (&c)[5], const uint8_t* pal,
                                            uint32_t (&hi)[kUnitWords]) {
  switch (w) {  // uniform across the warp (a job's width)
    case 1: palette_his<1>(c, pal, hi); break;
    case 2: palette_his<2>(c, pal, hi); break;
    case 3: palette_his<3>(c, pal, hi); break;
    case 4: palette_his<4>(c, pal, hi); break;
    case 5: palette_his<5>(c, pal, hi); break;
    case 6: palette_his<6>(c, pal, hi); break;
    default: palette_his<7>(c, pal, hi); break;
  }
}

// Sign/magnitude high bytes of a unit (mode 2) with W-bit magnitudes.
template <int W>
__device__ __forceinline__ void signmag_his(const uint32_t (&sg)[5], const uint32_t (&mg)[5], uint32_t mag_min,
                                            uint32_t (&hi)[kUnitWords]) {
#pragma unroll
  for (int i = 0; i < kUnitWords; ++i) hi[i] = (bit_field(sg, i, 1) << 7) | (bit_field(mg, i, W) + mag_min);
}

__device__ __forceinline__ void signmag_his(uint32_t w, const uint32_t (&sg)[5], const uint32_t (&mg)[5],
                                            uint32_t mag_min, uint32_t (&hi)[kUnitWords]) {
  switch (w) {
    case 1: signmag_his<1>(sg, mg, mag_min, hi); break;
    case 2: signmag_his<2>(sg, mg, mag_min, hi); break;
    case 3: signmag_his<3>(sg, mg, mag_min, hi); break;
    case 4: signmag_his<4>(sg, mg, mag_min, hi); break;
    case 5: signmag_his<5>(sg, mg, mag_min, hi); break;
    default: signmag_his<6>(sg, mg, mag_min, hi); break;
  }
}

// One nibble plane of a unit (mode 1): OR the plane's nibbles into hi.
template <int W>
__device__ __forceinline__ void nibble_his(const uint32_t (&c)[5], const uint8_t* pal, int shift,
                                           uint32_t (&hi)[kUnitWords]) {
#pragma unroll
  for (int i = 0; i < kUnitWords; ++i) hi[i] |= static_cast<uint32_t>(pal[bit_field(c, i, W)]) << shift;
}

// One thread per 16-word unit.  A job's units are padded to whole warps
// (the host's unit_start), so a warp works on one job at a time and keeps
// that job's palette (mode 0: 256 high bytes, mode 1: four 16-entry nibble
// palettes, mode 4: 32 high bytes) in shared memory; the code widths are
// dispatched once per job to code paths with constant field offsets.
template <int kMax>
__global__ void __launch_bounds__(256) ModeDecodeKernel(const __grid_constant__ ModeBatch<kMax> b) {
  __shared__ __align__(16) uint8_t spal[8][256];
  const uint64_t total = b.unit_start[b.jobs];  // a multiple of 32
  const int lane = threadIdx.x & 31;
  uint8_t* pal = spal[threadIdx.x >> 5];
  int j = 0, pal_job = -1;
  for (uint64_t u = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total;
       u += static_cast<uint64_t>(gridDim.x) * blockDim.x) {  // whole warps: the loop is uniform
    while (u >= b.unit_start[j + 1]) ++j;  // a thread's units increase; uniform across the warp
    const DecJob& J = b.job[j];
    const uint8_t* s = J.src;
    const uint32_t mode = __ldg(s);
    if (j != pal_job) {  // the job's palette bytes, from the stream's header
      __syncwarp();      // the lanes are done with the previous job's palette
      const uint32_t at = mode == 0 ? 2 : mode == 1 ? 5 : 1;
      const uint32_t bytes = mode == 0 ? 256 : mode == 1 ? 64 : mode == 4 ? 32 : 0;
      if (J.src_bytes >= at + bytes)
        for (uint32_t i = lane; i < bytes; i += 32) pal[i] = __ldg(s + at + i);
      __syncwarp();
      pal_job = j;
    }
    const uint64_t n = J.n, unit = u - b.unit_start[j], g = kUnitWords * unit;
    if (g >= n) continue;  // a unit of the padding
    const uint32_t valid = static_cast<uint32_t>(min(n - g, static_cast<uint64_t>(kUnitWords)));
    uint32_t hi[kUnitWords];  // high byte (modes 0, 2, 4) or the whole word (mode 1)
    uint32_t low[5] = {0, 0, 0, 0, 0};
    if (mode == 0) {
      const uint32_t w = __ldg(s + 1);
      if (J.src_bytes < 258 || w < 1 || w >= 8 || J.src_bytes != 258 + n + plane_bytes(n, w)) continue;
      uint32_t c[5];
      const uint64_t off = uint64_t{2} * w * unit;
      ldg_bytes16(s + 258 + n + off, static_cast<uint32_t>(min(uint64_t{2} * w, plane_bytes(n, w) - off)), c);
      ldg_bytes16(s + 258 + g, valid, low);
      palette_his(w, c, pal, hi);
    } else if (mode == 2) {
      const uint32_t w = __ldg(s + 1), mag_min = __ldg(s + 2);
      const uint64_t sign_bytes = (n + 7) / 8;
      if (J.src_bytes < 3 || w < 1 || w >= 7 || J.src_bytes != 3 + n + sign_bytes + plane_bytes(n, w)) continue;
      uint32_t sg[5], mg[5];
      const uint64_t off = uint64_t{2} * w * unit;
      ldg_bytes16(s + 3 + n + 2 * unit, static_cast<uint32_t>(min(uint64_t{2}, sign_bytes - 2 * unit)), sg);
      ldg_bytes16(s + 3 + n + sign_bytes + off, static_cast<uint32_t>(min(uint64_t{2} * w, plane_bytes(n, w) - off)), mg);
      ldg_bytes16(s + 3 + g, valid, low);
      signmag_his(w, sg, mg, mag_min, hi);
    } else if (mode == 4) {
      if (J.src_bytes != 33 + n + plane_bytes(n, 5)) continue;
      uint32_t c[5];
      const uint64_t off = uint64_t{10} * unit;
      ldg_bytes16(s + 33 + n + off, static_cast<uint32_t>(min(uint64_t{10}, plane_bytes(n, 5) - off)), c);
      ldg_bytes16(s + 33 + g, valid, low);
      palette_his<5>(c, pal, hi);
    } else if (mode == 1) {
      if (J.src_bytes < 69) continue;
      uint32_t w[4];
      uint64_t total_bytes = 69;
      bool ok = true;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        w[q] = __ldg(s + 1 + q);
        ok = ok && (w[q] == 1 || w[q] == 2 || w[q] == 4);
        total_bytes += plane_bytes(n, w[q]);
      }
      if (!ok || J.src_bytes != total_bytes) continue;
#pragma unroll
      for (int i = 0; i < kUnitWords; ++i) hi[i] = 0;
      const uint8_t* plane = s + 69;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t c[5];
        const uint64_t off = uint64_t{2} * w[q] * unit;
        ldg_bytes16(plane + off, static_cast<uint32_t>(min(uint64_t{2} * w[q], plane_bytes(n, w[q]) - off)), c);
        if (w[q] == 1) nibble_his<1>(c, pal + 16 * q, 4 * q, hi);
        else if (w[q] == 2) nibble_his<2>(c, pal + 16 * q, 4 * q, hi);
        else nibble_his<4>(c, pal + 16 * q, 4 * q, hi);
        plane += plane_bytes(n, w[q]);
      }
    } else {
      continue;  // modes 3, 5, 6 belong to DecodeKernel; others are not streams
    }
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t w0, w1;
      if (mode == 1) {
        w0 = hi[2 * k];
        w1 = hi[2 * k + 1];
      } else {
        w0 = (hi[2 * k] << 8) | bit_field(low, 2 * k, 8);
        w1 = (hi[2 * k + 1] << 8) | bit_field(low, 2 * k + 1, 8);
      }
      o[k] = (w0 & 0xFFFFu) | (w1 << 16);
    }
    store_unit(J.dst, J.L, g, valid, o, J.vec != 0);
  }
}

// -------------------------------------------------------------- writeback
//
// Codec writeback (vllm_connector.py:3460-3563, segments :3720-3738): a
// job's stream is copied over its own source blocks, the K-plane run of the
// job's contiguous blocks first, then the V-plane run, so that the transfer
// buffer can be reused while the stream waits in the (no longer needed) KV
// blocks for its copy to the host.  One launch for all jobs; 16-byte copies
// when the stream and the segments are 16-byte aligned.
struct WritebackJob {
  const uint8_t* src;  // the stream
  uint64_t bytes;      // its length
  uint8_t* seg[2];     // K- and V-plane runs of the blocks
  uint64_t seg_bytes;  // bytes per run
  uint64_t chunks;     // 16-byte chunks of the stream (rounded up)
  int vec;
  int pad;
};

template <int kMax>
struct WritebackBatch {
  uint32_t jobs;
  uint64_t chunk_start[kMax + 1];
  WritebackJob job[kMax];
};

template <int kMax>
__global__ void __launch_bounds__(256) WritebackKernel(const __grid_constant__ WritebackBatch<kMax> b) {
  // four 16-byte chunks a thread per round, their loads issued before any
  // store: a plain copy needs bytes in flight more than anything else
  constexpr int kU = 4;
  const uint64_t total = b.chunk_start[b.jobs];
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  int j = 0;
  for (uint64_t c0 = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c0 < total; c0 += kU * stride) {
    uint4 v[kU];
    int jk[kU];
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      const uint64_t c = c0 + k * stride;
      jk[k] = -1;
      v[k] = make_uint4(0, 0, 0, 0);
      if (c >= total) continue;
      while (c >= b.chunk_start[j + 1]) ++j;  // chunks increase
      jk[k] = j;
      const WritebackJob& W = b.job[j];
      const uint64_t off = 16 * (c - b.chunk_start[j]);
      if (W.vec && off + 16 <= W.bytes) v[k] = __ldg(reinterpret_cast<const uint4*>(W.src + off));
    }
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      if (jk[k] < 0) continue;
      const uint64_t c = c0 + k * stride;
      const WritebackJob& W = b.job[jk[k]];
      const uint64_t off = 16 * (c - b.chunk_start[jk[k]]);
      const uint64_t n = min(uint64_t{16}, W.bytes - off);
      const int s = off >= W.seg_bytes ? 1 : 0;
      uint8_t* dst = W.seg[s] + (off - (s ? W.seg_bytes : 0));
      if (W.vec && n == 16) {
        *reinterpret_cast<uint4*>(dst) = v[k];
      } else {
        for (uint64_t q = 0; q < n; ++q) {
          const uint64_t o = off + q;
          const int t = o >= W.seg_bytes ? 1 : 0;
          W.seg[t][o - (t ? W.seg_bytes : 0)] = __ldg(W.src + o);
        }
      }
    }
  }
}

template <int kMax>
__global__ void __launch_bounds__(kThreads) ZeroKernel(const __grid_constant__ ZeroBatch<kMax> z) {
  grid_dependency_sync();
  for (uint32_t r = blockIdx.y; r < z.count; r += gridDim.y) {
    uint8_t* p = z.ptr[r];
    const uint64_t bytes = z.bytes[r];
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint64_t lead = (16 - (a & 15)) & 15;
    const uint64_t head = bytes < lead ? bytes : lead;
    const uint64_t vec = (bytes - head) / 16;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    const uint64_t first = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
    if (first < head) p[first] = 0;
    uint4* v = reinterpret_cast<uint4*>(p + head);
    for (uint64_t i = first; i < vec; i += stride) v[i] = make_uint4(0, 0, 0, 0);
    for (uint64_t i = head + vec * 16 + first; i < bytes; i += stride) p[i] = 0;
  }
}

}  // namespace ukv
