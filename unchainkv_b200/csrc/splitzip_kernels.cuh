// Batched splitzip kernels (sm_100a).
//
// Every kernel takes a batch of jobs as a __grid_constant__ parameter: one job
// is one reference ABI call (one layer of one request).  The grid covers the
// 8192-word tiles of all jobs; a CTA finds its job by binary search of the
// tile offsets.  A single ABI call is a batch of one.
//
// Tile work (one CTA of 256 threads, 8 warps x 2 steps x 32 lanes x 16 words):
//   encode: words staged by TMA bulk copies (one per contiguous run of the
//     block table) -> per lane 16 words in registers -> body/low plane by
//     byte_perm SIMD, codes by a shared-memory table -> warp funnel stores
//     into the unaligned stream regions;
//   decode: stream bytes staged by TMA -> per lane 16 output words -> two
//     16-byte stores into the paged cache block.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "splitzip_device.cuh"

namespace ukv {

constexpr int kMaxBatch = 96;
constexpr uint64_t kStatusFlag = 1ull << 63;
constexpr int kDecodeSlots = 1024;

struct DecodeSlot {
  unsigned int done;
  unsigned int covered;
  unsigned int pad[2];
};

// ------------------------------------------------------------------ jobs

// Encode job.  `scratch` is 16-byte aligned device memory inside the
// caller's stream buffer, past the stream (see the layout constants below).
struct EncJob {
  const uint16_t* src;
  Layout L;
  uint8_t* dst;
  uint8_t* scratch;
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
  uint32_t slot;
  int vec;
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

// Scratch layouts (byte offsets from EncJob::scratch).
//   top16 encode: [0,4) batch tile ticket (job 0), [4,8) error flag,
//     [16, 16+8G) group words (done<<32 | escapes of 32 tiles),
//     [16+8G, 16+8G+8T) tile status words (flag | escapes).
//   fixed encode: [0,32) high-byte bitmap, [32,36) error flag.
//   auto encode:  [0,4) escape total, [4,8) error flag, [16,48) bitmap,
//     [64, 64+8G) group words, [64+8G, 64+8G+4T) tile escape counts.
__host__ __device__ constexpr uint64_t groups_for(uint64_t tiles) { return (tiles + 31) / 32; }
__host__ __device__ constexpr uint64_t top16_scratch_bytes(uint64_t tiles) {
  return 16 + 8 * groups_for(tiles) + 8 * tiles;
}
__host__ __device__ constexpr uint64_t auto_scratch_bytes(uint64_t tiles) {
  return 64 + 8 * groups_for(tiles) + 4 * tiles;
}
constexpr uint64_t kFixedScratchBytes = 36;

__device__ unsigned int g_device_errors;
__device__ DecodeSlot g_decode_slots[kDecodeSlots];

__device__ __forceinline__ void raise_error(uint32_t* flag) {
  if (flag) atomicOr(flag, 1u);
  atomicAdd(&g_device_errors, 1u);
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------ tile staging

__device__ __forceinline__ uint32_t tile_len(uint64_t n, uint64_t t0) {
  return static_cast<uint32_t>(n - t0 < kTileWords ? n - t0 : kTileWords);
}

// Stage the tile's words, wait (bounded) and make them visible to the CTA.
__device__ __forceinline__ void load_tile_words(const EncJob& J, uint64_t t0, uint32_t len,
                                                uint16_t* sin, uint64_t* bar, uint32_t* error) {
  stage_words(J.src, J.L, J.bulk != 0, t0, len, sin, bar);
  const bool ok = mbar_wait(bar, 0);
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) raise_error(error);
    mbar_wait(bar, 0);
    __syncthreads();
  }
}

__device__ __forceinline__ void load_unit(const uint16_t* sin, uint32_t w0, uint32_t (&x)[8]) {
  const uint4 v0 = *reinterpret_cast<const uint4*>(sin + w0);
  const uint4 v1 = *reinterpret_cast<const uint4*>(sin + w0 + 8);
  x[0] = v0.x; x[1] = v0.y; x[2] = v0.z; x[3] = v0.w;
  x[4] = v1.x; x[5] = v1.y; x[6] = v1.z; x[7] = v1.w;
}

// ------------------------------------------------------------ top16 encode

// Codes + escape mask of 16 words.  tbl entries: nibble*0x11, or 0x100 for
// "escape" (code 255 of the reference table; the stored nibble is then 0).
template <bool kPerWordPlane>
__device__ __forceinline__ void top16_codes(const uint32_t (&x)[8], const uint32_t* tbl,
                                            uint32_t plane_mask, uint32_t& c0, uint32_t& c1,
                                            uint32_t& esc) {
  uint32_t bytes[8];
  esc = 0;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const uint32_t e0 = (x[p] >> 7) & 0xFFu;
    const uint32_t e1 = (x[p] >> 23) & 0xFFu;
    uint32_t t0, t1;
    if (kPerWordPlane) {
      t0 = tbl[(((plane_mask >> (2 * p)) & 1u) << 8) + e0];
      t1 = tbl[(((plane_mask >> (2 * p + 1)) & 1u) << 8) + e1];
    } else {
      t0 = tbl[e0];
      t1 = tbl[e1];
    }
    bytes[p] = (t0 & 0x0Fu) | (t1 & 0xF0u);
    esc |= ((t0 >> 8) & 1u) << (2 * p);
    esc |= ((t1 >> 8) & 1u) << (2 * p + 1);
  }
  c0 = bytes[0] | (bytes[1] << 8) | (bytes[2] << 16) | (bytes[3] << 24);
  c1 = bytes[4] | (bytes[5] << 8) | (bytes[6] << 16) | (bytes[7] << 24);
}

__device__ __forceinline__ void load_top16_table(const uint8_t* tables, uint32_t* stbl) {
  for (int i = threadIdx.x; i < 512; i += kThreads) {
    const uint32_t c = __ldg(tables + i);
    stbl[i] = c == 255u ? 0x100u : (c & 0xFu) * 0x11u;
  }
}

// Body + codes of one tile; returns this lane's escape masks per step.
__device__ __forceinline__ void top16_tile_body(const EncJob& J, uint64_t t0, uint32_t len,
                                                const uint16_t* sin, const uint32_t* stbl,
                                                uint32_t (&masks)[kStepsPerWarp]) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = len > sb ? min(len - sb, static_cast<uint32_t>(kStepWords)) : 0u;
    const uint32_t valid = len > w0 ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
    uint32_t x[8];
    load_unit(sin, w0, x);
    uint32_t b[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t lo = __byte_perm(x[2 * q], x[2 * q + 1], 0x6420);
      const uint32_t hi = __byte_perm(x[2 * q], x[2 * q + 1], 0x7531);
      b[q] = (lo & 0x7F7F7F7Fu) | (hi & 0x80808080u);
    }
    const uint64_t g = t0 + w0;
    uint32_t c0, c1, esc;
    if (g >= J.half) {
      top16_codes<false>(x, stbl + 256, 0, c0, c1, esc);
    } else if (g + kUnitWords <= J.half) {
      top16_codes<false>(x, stbl, 0, c0, c1, esc);
    } else {
      const uint32_t pm = (0xFFFFu << static_cast<uint32_t>(J.half - g)) & 0xFFFFu;
      top16_codes<true>(x, stbl, pm, c0, c1, esc);
    }
    if (valid < kUnitWords) {
      esc &= (1u << valid) - 1u;
      const uint64_t keep = valid == 0 ? 0ull : (~0ull >> (64 - 4 * valid));
      const uint64_t cc = (static_cast<uint64_t>(c1) << 32 | c0) & keep;
      c0 = static_cast<uint32_t>(cc);
      c1 = static_cast<uint32_t>(cc >> 32);
    }
    const uint64_t body[2] = {b[0] | (static_cast<uint64_t>(b[1]) << 32),
                              b[2] | (static_cast<uint64_t>(b[3]) << 32)};
    warp_store<uint64_t, 2>(J.dst + 5 + t0 + sb, step_valid, body, lane);
    const uint64_t codes[1] = {c0 | (static_cast<uint64_t>(c1) << 32)};
    warp_store<uint64_t, 1>(J.dst + 5 + J.n + (t0 + sb) / 2, (step_valid + 1) / 2, codes, lane);
    masks[s] = esc;
  }
}

// CTA-wide exclusive offsets of this lane's escapes (position order is warp,
// then step, then lane).  Returns the tile total; off[s] = offset of the
// lane's first escape of step s.  Uses s_wtot[2][kWarps] and syncs.
__device__ __forceinline__ uint32_t escape_offsets(const uint32_t (&masks)[kStepsPerWarp],
                                                   uint32_t (*s_wtot)[kWarps],
                                                   uint32_t (&off)[kStepsPerWarp]) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t n0 = __popc(masks[0]);
  const uint32_t n1 = __popc(masks[1]);
  const uint32_t mine = n0 | (n1 << 16);
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += t;
  }
  const uint32_t excl = incl - mine;
  if (lane == 31) {
    s_wtot[0][warp] = incl & 0xFFFFu;
    s_wtot[1][warp] = incl >> 16;
  }
  __syncthreads();
  uint32_t before = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t t = s_wtot[0][w] + s_wtot[1][w];
    if (w < warp) before += t;
    total += t;
  }
  off[0] = before + (excl & 0xFFFFu);
  off[1] = before + s_wtot[0][warp] + (excl >> 16);
  return total;
}

__device__ __forceinline__ void write_escapes(const EncJob& J, uint64_t t0, const uint16_t* sin,
                                              const uint32_t (&masks)[kStepsPerWarp],
                                              const uint32_t (&off)[kStepsPerWarp], uint64_t prefix) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint8_t* entries = J.dst + 5 + J.n + (J.n + 1) / 2;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    uint32_t m = masks[s];
    if (!m) continue;
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    uint64_t slot = prefix + off[s];
    while (m) {
      const int j = __ffs(m) - 1;
      m &= m - 1;
      if (slot < J.cap) {
        const uint32_t pos = static_cast<uint32_t>(t0 + w0 + j);
        uint8_t* e = entries + slot * 5;
        e[0] = static_cast<uint8_t>(pos);
        e[1] = static_cast<uint8_t>(pos >> 8);
        e[2] = static_cast<uint8_t>(pos >> 16);
        e[3] = static_cast<uint8_t>(pos >> 24);
        e[4] = static_cast<uint8_t>((sin[w0 + j] >> 7) & 0xFFu);
      }
      ++slot;
    }
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

// Bounded wait for a published tile status; returns its count (0 on timeout).
__device__ __forceinline__ uint64_t wait_status(const uint64_t* p, uint32_t* error) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    const uint64_t s = ld_acquire(p);
    if (s & kStatusFlag) return s & ~kStatusFlag;
    __nanosleep(64);
  }
  raise_error(error);
  return 0;
}

// Bounded wait for a complete group of 32 tiles; returns its escape sum.
__device__ __forceinline__ uint64_t wait_group(const uint64_t* p, uint32_t* error) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    const uint64_t s = ld_relaxed_u64(p);
    if ((s >> 32) >= 32) return s & 0xFFFFFFFFull;
    __nanosleep(64);
  }
  raise_error(error);
  return 0;
}

// Two-level counting scan across the tiles of one job, run by one warp.
// Tile `tile` publishes its count to its status word and to its group of 32
// tiles, then sums (a) complete groups before its group and (b) the tiles of
// its own group before it.  Tiles are numbered by ticket, so every tile it
// waits on is held by a running CTA; the wait does not depend on later tiles.
__device__ uint64_t tile_prefix(uint8_t* scratch, uint32_t tiles, uint32_t tile, uint32_t count,
                                uint32_t* error) {
  const int lane = threadIdx.x & 31;
  uint64_t* groups = reinterpret_cast<uint64_t*>(scratch + 16);
  uint64_t* status = groups + groups_for(tiles);
  const uint32_t g = tile >> 5;
  const uint32_t r = tile & 31;
  if (lane == 0) {
    st_release(&status[tile], kStatusFlag | count);
    atomicAdd(reinterpret_cast<unsigned long long*>(&groups[g]), (1ull << 32) | count);
  }
  uint64_t v = 0;
  if (static_cast<uint32_t>(lane) < r) v = wait_status(&status[(g << 5) + lane], error);
  uint64_t prefix = warp_sum(v);
  for (uint32_t base = 0; base < g; base += 32) {
    v = 0;
    if (base + lane < g) v = wait_group(&groups[base + lane], error);
    prefix += warp_sum(v);
  }
  return prefix;
}

template <int kMax>
__global__ void __launch_bounds__(kThreads) EncodeTop16Kernel(const __grid_constant__ EncBatch<kMax> b) {
  __shared__ __align__(128) uint16_t sin[kTileWords];
  __shared__ uint32_t stbl[512];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_ticket;
  __shared__ uint32_t s_wtot[2][kWarps];
  __shared__ uint64_t s_prefix;
  const int tid = threadIdx.x;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    s_ticket = atomicAdd(reinterpret_cast<uint32_t*>(b.job[0].scratch), 1u);
  }
  __syncthreads();
  const uint32_t t = s_ticket;
  const int j = find_job<kMax>(b.tile_start, b.jobs, t);
  const EncJob& J = b.job[j];
  const uint32_t tile = t - b.tile_start[j];
  uint32_t* error = reinterpret_cast<uint32_t*>(J.scratch + 4);
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = tile_len(J.n, t0);
  load_top16_table(J.tables, stbl);
  load_tile_words(J, t0, len, sin, &bar, error);

  uint32_t masks[kStepsPerWarp];
  top16_tile_body(J, t0, len, sin, stbl, masks);
  uint32_t off[kStepsPerWarp];
  const uint32_t total = escape_offsets(masks, s_wtot, off);
  if ((tid >> 5) == 0) {
    const uint64_t prefix = tile_prefix(J.scratch, J.tiles, tile, total, error);
    if (tid == 0) s_prefix = prefix;
  }
  __syncthreads();
  const uint64_t prefix = s_prefix;
  write_escapes(J, t0, sin, masks, off, prefix);
  if (tile == J.tiles - 1 && tid == 0) {
    write_top16_header(J.dst, prefix + total, J.cap, ld_volatile_u32(error) != 0);
  }
}

// ------------------------------------------------- presence / auto stats

// Per tile: high-byte presence (-> job bitmap) and, for kStats, the top16
// escape count (-> tile count, group sum, job total).
template <int kMax, bool kStats>
__global__ void __launch_bounds__(kThreads) PresenceKernel(const __grid_constant__ EncBatch<kMax> b) {
  __shared__ __align__(128) uint16_t sin[kTileWords];
  __shared__ __align__(16) uint8_t spres[256];
  __shared__ uint8_t sesc[512];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_wsum[kWarps];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int j = find_job<kMax>(b.tile_start, b.jobs, blockIdx.x);
  const EncJob& J = b.job[j];
  const uint32_t tile = blockIdx.x - b.tile_start[j];
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(J.scratch + (kStats ? 16 : 0));
  uint32_t* error = reinterpret_cast<uint32_t*>(J.scratch + (kStats ? 4 : 32));
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (tid < 64) reinterpret_cast<uint32_t*>(spres)[tid] = 0;
  if (kStats) {
    for (int i = tid; i < 512; i += kThreads) sesc[i] = __ldg(J.tables + i) == 255u;
  }
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = tile_len(J.n, t0);
  load_tile_words(J, t0, len, sin, &bar, error);
  uint32_t escapes = 0;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (w0 >= len) continue;
    const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
    const uint64_t g = t0 + w0;
    if (valid == kUnitWords) {
      uint32_t x[8];
      load_unit(sin, w0, x);
      const uint8_t* et = sesc + (g >= J.half ? 256 : 0);
      const bool uniform = g >= J.half || g + kUnitWords <= J.half;
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        spres[(x[p] >> 8) & 0xFFu] = 1;
        spres[x[p] >> 24] = 1;
        if (kStats) {
          if (uniform) {
            escapes += et[(x[p] >> 7) & 0xFFu] + et[(x[p] >> 23) & 0xFFu];
          } else {
            escapes += sesc[((g + 2 * p) >= J.half ? 256 : 0) + ((x[p] >> 7) & 0xFFu)];
            escapes += sesc[((g + 2 * p + 1) >= J.half ? 256 : 0) + ((x[p] >> 23) & 0xFFu)];
          }
        }
      }
    } else {
      for (uint32_t i = 0; i < valid; ++i) {
        const uint32_t w = sin[w0 + i];
        spres[w >> 8] = 1;
        if (kStats) escapes += sesc[((g + i) >= J.half ? 256 : 0) + ((w >> 7) & 0xFFu)];
      }
    }
  }
  if (kStats) {
    escapes = warp_sum(escapes);
    if (lane == 0) s_wsum[warp] = escapes;
  }
  __syncthreads();
  const uint32_t bits = __ballot_sync(kFull, spres[tid] != 0);
  if (lane == 0 && bits) atomicOr(&bitmap[warp], bits);
  if (kStats && tid == 0) {
    uint32_t c = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) c += s_wsum[w];
    uint64_t* groups = reinterpret_cast<uint64_t*>(J.scratch + 64);
    uint32_t* counts = reinterpret_cast<uint32_t*>(groups + groups_for(J.tiles));
    counts[tile] = c;
    atomicAdd(reinterpret_cast<unsigned long long*>(&groups[tile >> 5]), (1ull << 32) | c);
    atomicAdd(reinterpret_cast<uint32_t*>(J.scratch), c);
  }
}

// ------------------------------------------------------------ fixed encode

// Palette rank of high byte `tid` from a 256-bit presence bitmap.
__device__ __forceinline__ void palette_ranks(const uint32_t* sbm, uint32_t* srank, uint32_t& distinct,
                                              bool& present, uint32_t& rank) {
  const int tid = threadIdx.x;
  distinct = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) distinct += __popc(sbm[w]);
  const uint32_t word = sbm[tid >> 5];
  present = (word >> (tid & 31)) & 1u;
  rank = __popc(word & ((1u << (tid & 31)) - 1u));
  for (int w = 0; w < (tid >> 5); ++w) rank += __popc(sbm[w]);
  srank[tid] = rank;
}

// Header + palette of a fixed stream (written by the job's tile 0).
template <int kBits>
__device__ __forceinline__ void write_fixed_header(uint8_t* dst, uint32_t distinct, bool present,
                                                   uint32_t rank, bool error) {
  constexpr uint32_t kLimit = kBits == 6 ? 64 : 32;
  const int tid = threadIdx.x;
  if (present && rank < kLimit) dst[1 + rank] = static_cast<uint8_t>(tid);
  if (tid >= static_cast<int>(distinct) && tid < static_cast<int>(kLimit)) dst[1 + tid] = 0;
  if (tid == 0) dst[0] = (distinct > kLimit || error) ? 255 : (kBits == 6 ? 3 : 4);
}

template <int kBits>
__device__ __forceinline__ void fixed_tile_body(const EncJob& J, uint64_t t0, uint32_t len,
                                                const uint16_t* sin, const uint32_t* srank) {
  constexpr uint32_t kHeader = kBits == 6 ? 65 : 33;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = len > sb ? min(len - sb, static_cast<uint32_t>(kStepWords)) : 0u;
    const uint32_t valid = len > w0 ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
    uint32_t x[8];
    load_unit(sin, w0, x);
    uint32_t low[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) low[q] = __byte_perm(x[2 * q], x[2 * q + 1], 0x6420);
    const uint64_t lowd[2] = {low[0] | (static_cast<uint64_t>(low[1]) << 32),
                              low[2] | (static_cast<uint64_t>(low[3]) << 32)};
    warp_store<uint64_t, 2>(J.dst + kHeader + t0 + sb, step_valid, lowd, lane);
    uint32_t c[16];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      c[2 * p] = srank[(x[p] >> 8) & 0xFFu];
      c[2 * p + 1] = srank[x[p] >> 24];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i >= static_cast<int>(valid)) c[i] = 0;
    if (kBits == 6) {
      uint32_t q[3];
      q[0] = c[0] | (c[1] << 6) | (c[2] << 12) | (c[3] << 18) | (c[4] << 24) | (c[5] << 30);
      q[1] = (c[5] >> 2) | (c[6] << 4) | (c[7] << 10) | (c[8] << 16) | (c[9] << 22) | (c[10] << 28);
      q[2] = (c[10] >> 4) | (c[11] << 2) | (c[12] << 8) | (c[13] << 14) | (c[14] << 20) | (c[15] << 26);
      warp_store<uint32_t, 3>(J.dst + kHeader + J.n + 3 * (t0 + sb) / 4, 3 * ((step_valid + 3) / 4), q,
                              lane);
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
      const uint16_t q[5] = {static_cast<uint16_t>(lo), static_cast<uint16_t>(lo >> 16),
                             static_cast<uint16_t>(lo >> 32), static_cast<uint16_t>(lo >> 48),
                             static_cast<uint16_t>(hi)};
      warp_store<uint16_t, 5>(J.dst + kHeader + J.n + 5 * (t0 + sb) / 8, 5 * ((step_valid + 7) / 8), q,
                              lane);
    }
  }
}

template <int kMax, int kBits>
__global__ void __launch_bounds__(kThreads) EncodeFixedKernel(const __grid_constant__ EncBatch<kMax> b) {
  constexpr uint32_t kLimit = kBits == 6 ? 64 : 32;
  __shared__ __align__(128) uint16_t sin[kTileWords];
  __shared__ uint32_t srank[256];
  __shared__ uint32_t sbm[8];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x;
  const int j = find_job<kMax>(b.tile_start, b.jobs, blockIdx.x);
  const EncJob& J = b.job[j];
  const uint32_t tile = blockIdx.x - b.tile_start[j];
  const uint32_t* bitmap = reinterpret_cast<const uint32_t*>(J.scratch);
  uint32_t* error = reinterpret_cast<uint32_t*>(J.scratch + 32);
  if (tid < 8) sbm[tid] = bitmap[tid];
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t distinct, rank;
  bool present;
  palette_ranks(sbm, srank, distinct, present, rank);
  if (tile == 0) write_fixed_header<kBits>(J.dst, distinct, present, rank, ld_volatile_u32(error) != 0);
  if (distinct > kLimit) return;  // uniform across the job's CTAs
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = tile_len(J.n, t0);
  load_tile_words(J, t0, len, sin, &bar, error);
  fixed_tile_body<kBits>(J, t0, len, sin, srank);
}

// ------------------------------------------------------------- auto encode

// Raw mode 6: [6] + the words little endian.
__device__ __forceinline__ void raw_tile_body(const EncJob& J, uint64_t t0, uint32_t len,
                                              const uint16_t* sin) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = len > sb ? min(len - sb, static_cast<uint32_t>(kStepWords)) : 0u;
    uint32_t x[8];
    load_unit(sin, w0, x);
    const uint64_t d[4] = {x[0] | (static_cast<uint64_t>(x[1]) << 32), x[2] | (static_cast<uint64_t>(x[3]) << 32),
                           x[4] | (static_cast<uint64_t>(x[5]) << 32), x[6] | (static_cast<uint64_t>(x[7]) << 32)};
    warp_store<uint64_t, 4>(J.dst + 1 + 2 * (t0 + sb), 2 * step_valid, d, lane);
  }
}

// Kinds decided on the device from the stats pass, in the reference's
// fallback order (vllm_connector.py:3104-3118, 4557-4633): top16 if the
// escapes fit, else fixed6 if <= 64 high bytes, else raw mode 6 when the
// buffer holds it, else a fixed6 overflow stream (mode 255) for the host.
enum AutoKind { kAutoTop16 = 0, kAutoFixed6 = 1, kAutoRaw = 2, kAutoOverflow = 3 };

template <int kMax>
__global__ void __launch_bounds__(kThreads) EncodeAutoKernel(const __grid_constant__ EncBatch<kMax> b) {
  __shared__ __align__(128) uint16_t sin[kTileWords];
  __shared__ uint32_t stbl[512];  // top16 table or fixed ranks
  __shared__ uint32_t sbm[8];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_wtot[2][kWarps];
  __shared__ uint64_t s_prefix;
  const int tid = threadIdx.x;
  const int j = find_job<kMax>(b.tile_start, b.jobs, blockIdx.x);
  const EncJob& J = b.job[j];
  const uint32_t tile = blockIdx.x - b.tile_start[j];
  uint32_t* error = reinterpret_cast<uint32_t*>(J.scratch + 4);
  if (tid < 8) sbm[tid] = reinterpret_cast<const uint32_t*>(J.scratch + 16)[tid];
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t escapes = *reinterpret_cast<const uint32_t*>(J.scratch);
  uint32_t distinct, rank;
  bool present;
  palette_ranks(sbm, stbl + 256, distinct, present, rank);
  const bool err = ld_volatile_u32(error) != 0;
  const int kind = err ? kAutoOverflow
                 : escapes <= J.cap ? kAutoTop16
                 : distinct <= 64 ? kAutoFixed6
                 : J.raw_ok ? kAutoRaw : kAutoOverflow;
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = tile_len(J.n, t0);
  if (kind == kAutoOverflow) {
    if (tile == 0) write_fixed_header<6>(J.dst, distinct > 64 ? distinct : 65, present, rank, true);
    return;
  }
  if (kind == kAutoFixed6) {
    if (tile == 0) write_fixed_header<6>(J.dst, distinct, present, rank, false);
    __syncthreads();
    load_tile_words(J, t0, len, sin, &bar, error);
    fixed_tile_body<6>(J, t0, len, sin, stbl + 256);
    return;
  }
  if (kind == kAutoRaw) {
    if (tile == 0 && tid == 0) J.dst[0] = 6;
    load_tile_words(J, t0, len, sin, &bar, error);
    raw_tile_body(J, t0, len, sin);
    return;
  }
  // top16 with known per-tile offsets: prefix = complete groups before this
  // tile's group + this group's earlier tiles (no waiting: the stats pass ran).
  load_top16_table(J.tables, stbl);
  if ((tid >> 5) == 0) {
    const int lane = tid & 31;
    const uint64_t* groups = reinterpret_cast<const uint64_t*>(J.scratch + 64);
    const uint32_t* counts = reinterpret_cast<const uint32_t*>(groups + groups_for(J.tiles));
    const uint32_t g = tile >> 5;
    uint64_t v = lane < static_cast<int>(tile & 31) ? counts[(g << 5) + lane] : 0;
    uint64_t prefix = warp_sum(v);
    for (uint32_t base = 0; base < g; base += 32) {
      v = base + lane < g ? (groups[base + lane] & 0xFFFFFFFFull) : 0;
      prefix += warp_sum(v);
    }
    if (lane == 0) s_prefix = prefix;
  }
  // zero this tile's share of the unused escape slots [escapes, cap)
  {
    uint8_t* entries = J.dst + 5 + J.n + (J.n + 1) / 2;
    const uint64_t lo = 5 * escapes, hi = 5 * J.cap;
    const uint64_t share = (hi - lo + J.tiles - 1) / J.tiles;
    const uint64_t a = lo + share * tile;
    const uint64_t e = min(hi, a + share);
    for (uint64_t i = a + tid; i < e; i += kThreads) entries[i] = 0;
  }
  load_tile_words(J, t0, len, sin, &bar, error);
  uint32_t masks[kStepsPerWarp];
  top16_tile_body(J, t0, len, sin, stbl, masks);
  uint32_t off[kStepsPerWarp];
  escape_offsets(masks, s_wtot, off);  // syncs: s_prefix visible after
  write_escapes(J, t0, sin, masks, off, s_prefix);
  if (tile == 0 && tid == 0) write_top16_header(J.dst, escapes, J.cap, false);
}

// ------------------------------------------------------------------ decode

// Store the 16 words (8 u32, little-endian pairs) of one lane unit starting
// at packed index g into the paged cache.
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

__device__ __forceinline__ uint32_t entry_pos(const uint8_t* entries, uint64_t idx) {
  return load_u32le(entries + idx * 5);
}

struct Top16DecodeSmem {
  uint8_t body[kTileWords + 64];
  uint8_t codes[kTileWords / 2 + 64];
  uint32_t dtbl[512];
  uint32_t esc_bits[kTileWords / 32];
  uint8_t esc_exp[kTileWords];
};

struct Fixed6DecodeSmem {
  uint8_t low[kTileWords + 64];
  uint8_t codes[kTileWords * 3 / 4 + 64];
  uint32_t pal[64];
};

struct RawDecodeSmem {
  uint8_t words[2 * kTileWords + 64];
};

constexpr size_t kDecodeSmemBytes =
    sizeof(Top16DecodeSmem) > sizeof(Fixed6DecodeSmem)
        ? (sizeof(Top16DecodeSmem) > sizeof(RawDecodeSmem) ? sizeof(Top16DecodeSmem) : sizeof(RawDecodeSmem))
        : (sizeof(Fixed6DecodeSmem) > sizeof(RawDecodeSmem) ? sizeof(Fixed6DecodeSmem) : sizeof(RawDecodeSmem));

__device__ __forceinline__ void decode_top16_tile(const DecJob& J, uint32_t tile, Top16DecodeSmem& S,
                                                  uint64_t* bar, uint32_t* s_last) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint64_t count = min(static_cast<uint64_t>(load_u32le(J.src + 1)), J.cap);
  const uint8_t* books = J.tables + 512;
  for (int i = tid; i < 512; i += kThreads) {
    const int plane = i >> 8;
    const uint32_t cb = i & 255;
    S.dtbl[i] = (static_cast<uint32_t>(__ldg(books + plane * 16 + (cb & 15))) << 7) |
                (static_cast<uint32_t>(__ldg(books + plane * 16 + (cb >> 4))) << 23);
  }
  S.esc_bits[tid] = 0;
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = tile_len(J.n, t0);
  const uint32_t pad_b = stage_bytes(J.src, 5 + t0, len, S.body, bar);
  const uint32_t pad_c = stage_bytes(J.src, 5 + J.n + t0 / 2, (len + 1) / 2, S.codes, bar);
  if (tid == 0) mbar_arrive(bar);

  // this tile's escapes: lower_bound(t0) over the entries assuming ascending
  // positions (warp 32-ary search), then a forward scan while positions fall
  // in the tile.  Streams in another order are repaired by the last CTA.
  const uint8_t* entries = J.src + 5 + J.n + (J.n + 1) / 2;
  if (warp == 0 && count > 0) {
    uint64_t lo = 0, hi = count;  // answer in [lo, hi]
    while (hi - lo > 32) {
      const uint64_t step = (hi - lo + 31) / 32;
      const uint64_t idx = lo + lane * step;
      const bool probe = idx < hi;
      const bool below = probe && entry_pos(entries, idx) < t0;
      const uint32_t nb = __popc(__ballot_sync(kFull, below));
      const uint32_t np = __popc(__ballot_sync(kFull, probe));
      const uint64_t nlo = nb ? lo + (nb - 1) * step + 1 : lo;
      const uint64_t nhi = nb < np ? lo + nb * step : hi;
      lo = nlo;
      hi = nhi;
    }
    {
      const uint64_t idx = lo + lane;
      const bool below = idx < hi && entry_pos(entries, idx) < t0;
      lo += __popc(__ballot_sync(kFull, below));
    }
    uint64_t cur = lo;
    uint32_t covered = 0;
    for (uint64_t guard = 0; guard <= count; guard += 32) {
      const uint64_t idx = cur + lane;
      uint32_t p = 0;
      bool in = false;
      if (idx < count) {
        p = entry_pos(entries, idx);
        in = p >= t0 && p < t0 + len;
      }
      const uint32_t out = __ballot_sync(kFull, !in);
      const int first_out = out ? __ffs(out) - 1 : 32;
      if (lane < first_out) {
        const uint32_t local = static_cast<uint32_t>(p - t0);
        atomicOr(&S.esc_bits[local >> 5], 1u << (local & 31));
        S.esc_exp[local] = __ldg(entries + idx * 5 + 4);
      }
      covered += first_out;
      if (first_out < 32) break;
      cur += 32;
    }
    if (lane == 0 && covered) atomicAdd(&g_decode_slots[J.slot].covered, covered);
  }
  const bool ok = mbar_wait(bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) raise_error(nullptr);
    mbar_wait(bar, 0);
    __syncthreads();
  }

  const bool vec = J.vec != 0;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (w0 >= len) continue;
    const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
    uint32_t B[4];
    smem_read16(S.body, pad_b + w0, B);
    uint32_t C[2];
    smem_read_words<2>(S.codes, pad_c + w0 / 2, C);
    const uint64_t g = t0 + w0;
    uint32_t o[8];
    const bool uniform = g >= J.half || g + kUnitWords <= J.half;
    const uint32_t* tb = S.dtbl + (g >= J.half ? 256 : 0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t cb = (C[i >> 2] >> (8 * (i & 3))) & 0xFFu;
      const uint32_t body2 = __byte_perm(B[i >> 1], 0, (i & 1) ? 0x3322 : 0x1100) & 0x807F807Fu;
      uint32_t ex;
      if (uniform) {
        ex = tb[cb];
      } else {
        const uint32_t p0 = (g + 2 * i) >= J.half;
        const uint32_t p1 = (g + 2 * i + 1) >= J.half;
        ex = (S.dtbl[(p0 << 8) + cb] & 0xFFFFu) | (S.dtbl[(p1 << 8) + cb] & 0xFFFF0000u);
      }
      o[i] = body2 | ex;
    }
    const uint32_t eb = (S.esc_bits[w0 >> 5] >> (w0 & 31)) & 0xFFFFu;
    if (eb) {
#pragma unroll
      for (int i = 0; i < kUnitWords; ++i) {
        if ((eb >> i) & 1u) {
          const uint32_t e = S.esc_exp[w0 + i];
          const uint32_t sh = (i & 1) * 16;
          o[i >> 1] = (o[i >> 1] & ~(0x7F80u << sh)) | ((e << 7) << sh);
        }
      }
    }
    store_unit(J.dst, J.L, g, valid, o, vec);
  }

  // Last CTA of the job: apply every entry if the tiles did not account for
  // all of them (entries out of position order, or positions >= n).
  if (count == 0) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&g_decode_slots[J.slot].done, 1u);
    *s_last = prev == J.tiles - 1;
  }
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  const uint32_t covered = ld_volatile_u32(&g_decode_slots[J.slot].covered);
  if (covered != count) {
    for (uint64_t i = tid; i < count; i += kThreads) {
      const uint32_t p = entry_pos(entries, i);
      if (p >= J.n) continue;
      uint16_t* w = J.dst + layout_addr(J.L, p);
      *w = static_cast<uint16_t>((__ldcg(w) & 0x807Fu) |
                                 (static_cast<uint32_t>(__ldg(entries + i * 5 + 4)) << 7));
    }
  }
  __syncthreads();
  if (tid == 0) {
    g_decode_slots[J.slot].done = 0;
    g_decode_slots[J.slot].covered = 0;
  }
}

__device__ __forceinline__ void decode_fixed6_tile(const DecJob& J, uint32_t tile, Fixed6DecodeSmem& S,
                                                   uint64_t* bar) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid < 64) S.pal[tid] = static_cast<uint32_t>(__ldg(J.src + 1 + tid)) << 8;
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = tile_len(J.n, t0);
  const uint32_t pad_l = stage_bytes(J.src, 65 + t0, len, S.low, bar);
  const uint32_t pad_c = stage_bytes(J.src, 65 + J.n + 3 * t0 / 4, 3 * ((len + 3) / 4), S.codes, bar);
  if (tid == 0) mbar_arrive(bar);
  const bool ok = mbar_wait(bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) raise_error(nullptr);
    mbar_wait(bar, 0);
    __syncthreads();
  }
  const bool vec = J.vec != 0;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (w0 >= len) continue;
    const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
    uint32_t Lw[4];
    smem_read16(S.low, pad_l + w0, Lw);
    uint32_t Q[3];
    smem_read_words<3>(S.codes, pad_c + 3 * w0 / 4, Q);
    uint32_t c[16];
    c[0] = Q[0] & 63; c[1] = (Q[0] >> 6) & 63; c[2] = (Q[0] >> 12) & 63; c[3] = (Q[0] >> 18) & 63;
    c[4] = (Q[0] >> 24) & 63; c[5] = ((Q[0] >> 30) | (Q[1] << 2)) & 63;
    c[6] = (Q[1] >> 4) & 63; c[7] = (Q[1] >> 10) & 63; c[8] = (Q[1] >> 16) & 63;
    c[9] = (Q[1] >> 22) & 63; c[10] = ((Q[1] >> 28) | (Q[2] << 4)) & 63;
    c[11] = (Q[2] >> 2) & 63; c[12] = (Q[2] >> 8) & 63; c[13] = (Q[2] >> 14) & 63;
    c[14] = (Q[2] >> 20) & 63; c[15] = (Q[2] >> 26) & 63;
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t l2 = __byte_perm(Lw[i >> 1], 0, (i & 1) ? 0x4342 : 0x4140);
      o[i] = l2 | S.pal[c[2 * i]] | (S.pal[c[2 * i + 1]] << 16);
    }
    store_unit(J.dst, J.L, t0 + w0, valid, o, vec);
  }
}

__device__ __forceinline__ void decode_raw_tile(const DecJob& J, uint32_t tile, RawDecodeSmem& S,
                                                uint64_t* bar) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = tile_len(J.n, t0);
  const uint32_t pad = stage_bytes(J.src, 1 + 2 * t0, 2 * len, S.words, bar);
  if (tid == 0) mbar_arrive(bar);
  const bool ok = mbar_wait(bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) raise_error(nullptr);
    mbar_wait(bar, 0);
    __syncthreads();
  }
  const bool vec = J.vec != 0;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (w0 >= len) continue;
    const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
    uint32_t o[8];
    smem_read_words<8>(S.words, pad + 2 * w0, o);
    store_unit(J.dst, J.L, t0 + w0, valid, o, vec);
  }
}

// kMode: 5 = top16, 3 = fixed6, 0 = dispatch on each stream's mode byte
// (5, 3 or 6; a stream shorter than its mode's size is skipped).
template <int kMax, int kMode>
__global__ void __launch_bounds__(kThreads) DecodeKernel(const __grid_constant__ DecBatch<kMax> b) {
  __shared__ __align__(128) uint8_t smem[kDecodeSmemBytes];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_last;
  const int j = find_job<kMax>(b.tile_start, b.jobs, blockIdx.x);
  const DecJob& J = b.job[j];
  const uint32_t tile = blockIdx.x - b.tile_start[j];
  const uint32_t mode = __ldg(J.src);
  if (kMode != 0 && mode != static_cast<uint32_t>(kMode)) return;  // reference: write nothing
  if (kMode == 0) {
    uint64_t need = 0;
    if (mode == 5) need = 5 + J.n + (J.n + 1) / 2 + 5 * J.cap;
    else if (mode == 3) need = 65 + J.n + 3 * ((J.n + 3) / 4);
    else if (mode == 6) need = 1 + 2 * J.n;
    if (need == 0 || need > J.src_bytes) return;
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (mode == 5) {
    decode_top16_tile(J, tile, *reinterpret_cast<Top16DecodeSmem*>(smem), &bar, &s_last);
  } else if (mode == 3) {
    decode_fixed6_tile(J, tile, *reinterpret_cast<Fixed6DecodeSmem*>(smem), &bar);
  } else {
    __syncthreads();
    decode_raw_tile(J, tile, *reinterpret_cast<RawDecodeSmem*>(smem), &bar);
  }
}

// ------------------------------------------------------------------- zero

template <int kMax>
__global__ void __launch_bounds__(kThreads) ZeroKernel(const __grid_constant__ ZeroBatch<kMax> z) {
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
