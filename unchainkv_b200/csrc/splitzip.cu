// UnchainKV splitzip bf16 KV codec for B200 (sm_100a): kernels + C ABI.
//
// Drop-in for native/unchain_kv/kvq_splitzip_cuda.cu of the reference: every
// kvq_splitzip_* entry point keeps the reference's name, argument order,
// argument meaning, decline rules (return 0), return values and error strings
// ("<Kernel>: <cudaGetErrorString>", return -1).  Streams are the caller's
// cudaStream_t; nothing is synchronised.  New entry points (fused gather,
// device error query) follow the same conventions.
//
// Stream formats (identical bytes to the reference, with canonical ordering):
//   top16 (mode 5): [0]=5|255, [1..4] u32 LE escape count, body n bytes
//     (mantissa7 | sign<<7), codes ceil(n/2) bytes (4-bit exponent codes, even
//     word in the low nibble), ceil(n/200) five-byte escape entries
//     {u32 LE position, u8 exponent} sorted by position, unused slots zero.
//   fixed6 (mode 3) / fixed5 (mode 4): [0]=3|4|255, 64/32-byte palette of
//     distinct high bytes in ascending order (zero padded), low-byte plane n
//     bytes, 6-bit codes 4->3 bytes LE / 5-bit codes 8->5 bytes LE.
//
// Kernel design (one CTA of 256 threads per 8192-word tile):
//   * input words are staged into shared memory by TMA bulk copies, one per
//     contiguous run of the block table (the gather is fused: the kernel walks
//     the vLLM block table itself instead of reading an index_select copy);
//   * each lane turns 16 words into its output bytes in registers (byte_perm
//     SIMD for the body/low planes, one shared-memory table lookup per word
//     for codes) and the warp writes the unaligned stream regions with
//     aligned 8/4/2-byte funnel stores;
//   * escapes are compacted in position order: warp scan of per-lane counts,
//     CTA scan of warp totals, and a decoupled look-back across tiles (tile
//     order from an atomic ticket, so every predecessor is resident); the
//     entries are then written straight to their final slots;
//   * decode stages the body/codes bytes of its tile by TMA, finds the tile's
//     escapes by a warp-cooperative search of the sorted entry list, patches
//     them in registers and stores 32 bytes per lane into the paged cache.
//     Streams whose entries are not in position order (the reference encoder
//     emits them in atomic order) are detected on the device and fixed by
//     the last CTA to finish, so every valid stream decodes identically.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>

#include "splitzip_device.cuh"
#include "unchain_kv_splitzip.h"

using namespace ukv;

namespace {

thread_local std::string g_last_error;

long long Fail(const char* what, cudaError_t status) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(status);
  return -1;
}

// Device-side error counter (bounded waits that ran out).  Read by
// kvq_splitzip_device_errors().
__device__ unsigned int g_device_errors;

// Per-call state of the top16 decoder's last-CTA protocol.  A host counter
// picks the slot; the last CTA of the call resets it.
constexpr int kDecodeSlots = 1024;
struct DecodeSlot {
  unsigned int done;
  unsigned int covered;
  unsigned int pad[2];
};
__device__ DecodeSlot g_decode_slots[kDecodeSlots];
std::atomic<unsigned int> g_decode_slot_counter{0};

constexpr uint64_t kAgg = 1ull << 62;
constexpr uint64_t kInc = 2ull << 62;
constexpr uint64_t kValueMask = (1ull << 62) - 1;

__device__ __forceinline__ void raise_error(uint32_t* flag) {
  if (flag) atomicOr(flag, 1u);
  atomicAdd(&g_device_errors, 1u);
}

// =====================================================================
// top16 encode (fused gather)
// =====================================================================

struct Top16EncodeArgs {
  const uint16_t* src;
  Layout L;
  int bulk;
  uint8_t* dst;
  uint64_t n;
  uint64_t half;
  uint64_t cap;
  uint32_t num_tiles;
  const uint8_t* tables;
  uint32_t* ticket;
  uint32_t* error;
  uint64_t* status;
};

// Codes + escape mask of 16 words.  tbl entries: nibble*0x11, or 0x100 for
// "escape" (code 255 in the reference table; the stored nibble is then 0).
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

// Decoupled look-back over the per-tile escape counts.  Called by one whole
// warp.  Returns the exclusive prefix of `tile`; publishes its inclusive
// value.  Waits are bounded: on timeout the error flag is raised and the
// missing predecessor is counted as zero (the stream is then marked 255).
__device__ uint64_t lookback(uint64_t* status, uint32_t tile, uint64_t aggregate,
                             uint32_t* error, int lane) {
  if (tile == 0) {
    if (lane == 0) st_release(&status[0], kInc | aggregate);
    return 0;
  }
  if (lane == 0) st_release(&status[tile], kAgg | aggregate);
  uint64_t prefix = 0;
  int64_t j = static_cast<int64_t>(tile) - 1;
  uint32_t spins = 0;
  while (true) {
    const int64_t idx = j - lane;
    uint64_t s = idx >= 0 ? ld_acquire(&status[idx]) : kInc;
    bool timed_out = false;
    while (__any_sync(kFull, (s >> 62) == 0)) {
      if (++spins > kWaitLimit) {
        timed_out = true;
        break;
      }
      if ((s >> 62) == 0) {
        __nanosleep(32);
        s = ld_acquire(&status[idx]);
      }
    }
    if (timed_out) {
      if (lane == 0) raise_error(error);
      if ((s >> 62) == 0) s = kInc;
    }
    const uint32_t inc = __ballot_sync(kFull, (s >> 62) == 2);
    uint64_t v = s & kValueMask;
    if (inc) {
      const int first = __ffs(inc) - 1;
      if (lane > first) v = 0;
      prefix += warp_sum(v);
      break;
    }
    prefix += warp_sum(v);
    j -= 32;
  }
  if (lane == 0) st_release(&status[tile], kInc | (prefix + aggregate));
  return prefix;
}

__global__ void __launch_bounds__(kThreads) EncodeTop16Kernel(const Top16EncodeArgs a) {
  __shared__ __align__(128) uint16_t sin[kTileWords];
  __shared__ uint32_t stbl[512];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_tile;
  __shared__ uint32_t s_wtot[2][kWarps];
  __shared__ uint64_t s_prefix;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    s_tile = atomicAdd(a.ticket, 1u);
  }
  for (int i = tid; i < 512; i += kThreads) {
    const uint32_t c = __ldg(a.tables + i);
    stbl[i] = c == 255u ? 0x100u : (c & 0xFu) * 0x11u;
  }
  __syncthreads();
  const uint32_t tile = s_tile;
  const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
  const uint32_t len = static_cast<uint32_t>(a.n - t0 < kTileWords ? a.n - t0 : kTileWords);
  stage_words(a.src, a.L, a.bulk != 0, t0, len, sin, &bar);
  bool ok = mbar_wait(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) raise_error(a.error);
    mbar_wait(&bar, 0);
    __syncthreads();
  }

  uint32_t masks[kStepsPerWarp];
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = len > sb ? min(len - sb, static_cast<uint32_t>(kStepWords)) : 0u;
    const uint32_t valid = len > w0 ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
    uint32_t x[8];
    {
      const uint4 v0 = *reinterpret_cast<const uint4*>(sin + w0);
      const uint4 v1 = *reinterpret_cast<const uint4*>(sin + w0 + 8);
      x[0] = v0.x; x[1] = v0.y; x[2] = v0.z; x[3] = v0.w;
      x[4] = v1.x; x[5] = v1.y; x[6] = v1.z; x[7] = v1.w;
    }
    uint32_t b[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t lo = __byte_perm(x[2 * q], x[2 * q + 1], 0x6420);
      const uint32_t hi = __byte_perm(x[2 * q], x[2 * q + 1], 0x7531);
      b[q] = (lo & 0x7F7F7F7Fu) | (hi & 0x80808080u);
    }
    const uint64_t g = t0 + w0;
    uint32_t c0, c1, esc;
    if (g >= a.half) {
      top16_codes<false>(x, stbl + 256, 0, c0, c1, esc);
    } else if (g + kUnitWords <= a.half) {
      top16_codes<false>(x, stbl, 0, c0, c1, esc);
    } else {
      const uint32_t pm = (0xFFFFu << static_cast<uint32_t>(a.half - g)) & 0xFFFFu;
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
    warp_store<uint64_t, 2>(a.dst + 5 + t0 + sb, step_valid, body, lane);
    const uint64_t codes[1] = {c0 | (static_cast<uint64_t>(c1) << 32)};
    warp_store<uint64_t, 1>(a.dst + 5 + a.n + (t0 + sb) / 2, (step_valid + 1) / 2, codes, lane);
    masks[s] = esc;
  }

  // ---- escape compaction: lane -> warp -> CTA -> tiles ------------------
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
  if (warp == 0) {
    const uint64_t prefix = lookback(a.status, tile, total, a.error, lane);
    if (lane == 0) s_prefix = prefix;
  }
  __syncthreads();
  const uint64_t P = s_prefix;
  uint8_t* entries = a.dst + 5 + a.n + (a.n + 1) / 2;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    uint32_t m = masks[s];
    if (!m) continue;
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    uint64_t slot = P + before + (s == 0 ? (excl & 0xFFFFu) : s_wtot[0][warp] + (excl >> 16));
    while (m) {
      const int j = __ffs(m) - 1;
      m &= m - 1;
      if (slot < a.cap) {
        const uint32_t pos = static_cast<uint32_t>(t0 + w0 + j);
        const uint8_t exp = static_cast<uint8_t>((sin[w0 + j] >> 7) & 0xFFu);
        uint8_t* e = entries + slot * 5;
        e[0] = static_cast<uint8_t>(pos);
        e[1] = static_cast<uint8_t>(pos >> 8);
        e[2] = static_cast<uint8_t>(pos >> 16);
        e[3] = static_cast<uint8_t>(pos >> 24);
        e[4] = exp;
      }
      ++slot;
    }
  }
  if (tile == a.num_tiles - 1 && tid == 0) {
    const uint64_t all = P + total;
    const uint32_t err = ld_volatile_u32(a.error);
    a.dst[0] = (all > a.cap || err) ? 255 : 5;
    const uint32_t cnt = static_cast<uint32_t>(all > a.cap ? a.cap : all);
    a.dst[1] = static_cast<uint8_t>(cnt);
    a.dst[2] = static_cast<uint8_t>(cnt >> 8);
    a.dst[3] = static_cast<uint8_t>(cnt >> 16);
    a.dst[4] = static_cast<uint8_t>(cnt >> 24);
  }
}

// =====================================================================
// fixed6 / fixed5 encode: presence pass + encode pass
// =====================================================================

struct PresenceArgs {
  const uint16_t* src;
  Layout L;
  int bulk;
  uint64_t n;
  uint32_t* bitmap;  // 8 x u32, zeroed by the host before the launch
  uint32_t* error;
};

__global__ void __launch_bounds__(kThreads) HighBytePresenceKernel(const PresenceArgs a) {
  __shared__ __align__(128) uint16_t sin[kTileWords];
  __shared__ __align__(16) uint8_t spres[256];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (tid < 64) reinterpret_cast<uint32_t*>(spres)[tid] = 0;
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(blockIdx.x) * kTileWords;
  const uint32_t len = static_cast<uint32_t>(a.n - t0 < kTileWords ? a.n - t0 : kTileWords);
  stage_words(a.src, a.L, a.bulk != 0, t0, len, sin, &bar);
  bool ok = mbar_wait(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) raise_error(a.error);
    mbar_wait(&bar, 0);
    __syncthreads();
  }
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (w0 >= len) continue;
    const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
    const uint4 v0 = *reinterpret_cast<const uint4*>(sin + w0);
    const uint4 v1 = *reinterpret_cast<const uint4*>(sin + w0 + 8);
    const uint32_t x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    if (valid == kUnitWords) {
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        spres[(x[p] >> 8) & 0xFFu] = 1;
        spres[x[p] >> 24] = 1;
      }
    } else {
      for (uint32_t j = 0; j < valid; ++j) spres[sin[w0 + j] >> 8] = 1;
    }
  }
  __syncthreads();
  const uint32_t bits = __ballot_sync(kFull, spres[tid] != 0);
  if (lane == 0 && bits) atomicOr(&a.bitmap[warp], bits);
}

struct FixedEncodeArgs {
  const uint16_t* src;
  Layout L;
  int bulk;
  uint8_t* dst;
  uint64_t n;
  const uint32_t* bitmap;
  uint32_t* error;
};

template <int kBits>
__global__ void __launch_bounds__(kThreads) EncodeFixedKernel(const FixedEncodeArgs a) {
  constexpr uint32_t kLimit = kBits == 6 ? 64 : 32;
  constexpr uint32_t kHeader = 1 + kLimit;
  __shared__ __align__(128) uint16_t sin[kTileWords];
  __shared__ uint32_t srank[256];
  __shared__ uint32_t sbm[8];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid < 8) sbm[tid] = a.bitmap[tid];
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t distinct = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) distinct += __popc(sbm[w]);
  // rank of high byte tid among the distinct high bytes (ascending order)
  const uint32_t word = sbm[tid >> 5];
  const bool present = (word >> (tid & 31)) & 1u;
  uint32_t rank = __popc(word & ((1u << (tid & 31)) - 1u));
  for (int w = 0; w < (tid >> 5); ++w) rank += __popc(sbm[w]);
  srank[tid] = rank;
  if (blockIdx.x == 0) {
    if (present && rank < kLimit) a.dst[1 + rank] = static_cast<uint8_t>(tid);
    if (tid >= static_cast<int>(distinct) && tid < static_cast<int>(kLimit)) a.dst[1 + tid] = 0;
    if (tid == 0) {
      const uint32_t err = ld_volatile_u32(a.error);
      a.dst[0] = (distinct > kLimit || err) ? 255 : (kBits == 6 ? 3 : 4);
    }
  }
  if (distinct > kLimit) return;  // uniform across the grid
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(blockIdx.x) * kTileWords;
  const uint32_t len = static_cast<uint32_t>(a.n - t0 < kTileWords ? a.n - t0 : kTileWords);
  stage_words(a.src, a.L, a.bulk != 0, t0, len, sin, &bar);
  bool ok = mbar_wait(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      raise_error(a.error);
      a.dst[0] = 255;
    }
    mbar_wait(&bar, 0);
    __syncthreads();
  }
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t sb = (warp * kStepsPerWarp + s) * kStepWords;
    const uint32_t w0 = sb + lane * kUnitWords;
    const uint32_t step_valid = len > sb ? min(len - sb, static_cast<uint32_t>(kStepWords)) : 0u;
    const uint32_t valid = len > w0 ? min(len - w0, static_cast<uint32_t>(kUnitWords)) : 0u;
    const uint4 v0 = *reinterpret_cast<const uint4*>(sin + w0);
    const uint4 v1 = *reinterpret_cast<const uint4*>(sin + w0 + 8);
    const uint32_t x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t low[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) low[q] = __byte_perm(x[2 * q], x[2 * q + 1], 0x6420);
    const uint64_t lowd[2] = {low[0] | (static_cast<uint64_t>(low[1]) << 32),
                              low[2] | (static_cast<uint64_t>(low[3]) << 32)};
    warp_store<uint64_t, 2>(a.dst + kHeader + t0 + sb, step_valid, lowd, lane);
    uint32_t c[16];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      c[2 * p] = srank[(x[p] >> 8) & 0xFFu];
      c[2 * p + 1] = srank[x[p] >> 24];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j >= static_cast<int>(valid)) c[j] = 0;
    if (kBits == 6) {
      uint32_t q[3];
      q[0] = c[0] | (c[1] << 6) | (c[2] << 12) | (c[3] << 18) | (c[4] << 24) | (c[5] << 30);
      q[1] = (c[5] >> 2) | (c[6] << 4) | (c[7] << 10) | (c[8] << 16) | (c[9] << 22) | (c[10] << 28);
      q[2] = (c[10] >> 4) | (c[11] << 2) | (c[12] << 8) | (c[13] << 14) | (c[14] << 20) | (c[15] << 26);
      const uint32_t cbytes = 3 * ((step_valid + 3) / 4);
      warp_store<uint32_t, 3>(a.dst + kHeader + a.n + 3 * (t0 + sb) / 4, cbytes, q, lane);
    } else {
      uint64_t lo = 0;
      uint32_t hi = 0;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int bit = 5 * j;
        if (bit + 5 <= 64) {
          lo |= static_cast<uint64_t>(c[j]) << bit;
        } else if (bit >= 64) {
          hi |= c[j] << (bit - 64);
        } else {
          lo |= static_cast<uint64_t>(c[j]) << bit;
          hi |= c[j] >> (64 - bit);
        }
      }
      const uint16_t q[5] = {static_cast<uint16_t>(lo), static_cast<uint16_t>(lo >> 16),
                             static_cast<uint16_t>(lo >> 32), static_cast<uint16_t>(lo >> 48),
                             static_cast<uint16_t>(hi)};
      const uint32_t cbytes = 5 * ((step_valid + 7) / 8);
      warp_store<uint16_t, 5>(a.dst + kHeader + a.n + 5 * (t0 + sb) / 8, cbytes, q, lane);
    }
  }
}

// =====================================================================
// decode + scatter
// =====================================================================

// Store the 16 words (8 u32, little endian pairs) of one lane unit that
// starts at packed index g into the paged cache.
__device__ __forceinline__ void store_unit(uint16_t* dst, const Layout& L, uint64_t g,
                                           uint32_t valid, const uint32_t (&o)[8], bool vec) {
  if (vec && valid == kUnitWords) {
    uint4* p = reinterpret_cast<uint4*>(dst + layout_addr(L, g));
    p[0] = make_uint4(o[0], o[1], o[2], o[3]);
    p[1] = make_uint4(o[4], o[5], o[6], o[7]);
  } else {
#pragma unroll
    for (uint32_t j = 0; j < kUnitWords; ++j)
      if (j < valid) dst[layout_addr(L, g + j)] = static_cast<uint16_t>(o[j >> 1] >> ((j & 1) * 16));
  }
}

struct Top16DecodeArgs {
  const uint8_t* src;
  uint16_t* dst;
  Layout L;
  uint64_t n;
  uint64_t half;
  uint64_t cap;
  const uint8_t* tables;
  int vec;
  uint32_t slot;
};

__device__ __forceinline__ uint32_t entry_pos(const uint8_t* entries, uint64_t idx) {
  return load_u32le(entries + idx * 5);
}

__global__ void __launch_bounds__(kThreads) DecodeTop16Kernel(const Top16DecodeArgs a) {
  __shared__ __align__(128) uint8_t sbody[kTileWords + 64];
  __shared__ __align__(128) uint8_t scodes[kTileWords / 2 + 64];
  __shared__ uint32_t dtbl[512];
  __shared__ uint32_t esc_bits[kTileWords / 32];
  __shared__ uint8_t esc_exp[kTileWords];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_last;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (__ldg(a.src) != 5) return;  // .cu:235 of the reference: write nothing
  const uint64_t count = min(static_cast<uint64_t>(load_u32le(a.src + 1)), a.cap);
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  const uint8_t* books = a.tables + 512;
  for (int i = tid; i < 512; i += kThreads) {
    const int plane = i >> 8;
    const uint32_t cb = i & 255;
    dtbl[i] = (static_cast<uint32_t>(__ldg(books + plane * 16 + (cb & 15))) << 7) |
              (static_cast<uint32_t>(__ldg(books + plane * 16 + (cb >> 4))) << 23);
  }
  esc_bits[tid] = 0;
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(blockIdx.x) * kTileWords;
  const uint32_t len = static_cast<uint32_t>(a.n - t0 < kTileWords ? a.n - t0 : kTileWords);
  const uint32_t pad_b = stage_bytes(a.src, 5 + t0, len, sbody, &bar);
  const uint32_t pad_c = stage_bytes(a.src, 5 + a.n + t0 / 2, (len + 1) / 2, scodes, &bar);
  if (tid == 0) mbar_arrive(&bar);

  // ---- this tile's escapes (overlaps the bulk copies) -------------------
  const uint8_t* entries = a.src + 5 + a.n + (a.n + 1) / 2;
  if (warp == 0 && count > 0) {
    // lower_bound(t0) assuming ascending positions (warp 32-ary search)
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
    // forward scan: entries from lo while their positions fall in this tile
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
        atomicOr(&esc_bits[local >> 5], 1u << (local & 31));
        esc_exp[local] = __ldg(entries + idx * 5 + 4);
      }
      covered += first_out;
      if (first_out < 32) break;
      cur += 32;
    }
    if (lane == 0 && covered) atomicAdd(&g_decode_slots[a.slot].covered, covered);
  }
  bool ok = mbar_wait(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) raise_error(nullptr);
    mbar_wait(&bar, 0);
    __syncthreads();
  }

  const bool vec = a.vec != 0;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (w0 >= len) continue;
    const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
    uint32_t B[4];
    smem_read16(sbody, pad_b + w0, B);
    uint32_t C[2];
    smem_read_words<2>(scodes, pad_c + w0 / 2, C);
    const uint64_t g = t0 + w0;
    uint32_t o[8];
    const bool uniform = g >= a.half || g + kUnitWords <= a.half;
    const uint32_t* tb = dtbl + (g >= a.half ? 256 : 0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t cb = (C[j >> 2] >> (8 * (j & 3))) & 0xFFu;
      const uint32_t body2 = __byte_perm(B[j >> 1], 0, (j & 1) ? 0x3322 : 0x1100) & 0x807F807Fu;
      uint32_t ex;
      if (uniform) {
        ex = tb[cb];
      } else {
        const uint32_t p0 = (g + 2 * j) >= a.half;
        const uint32_t p1 = (g + 2 * j + 1) >= a.half;
        ex = (dtbl[(p0 << 8) + cb] & 0xFFFFu) | (dtbl[(p1 << 8) + cb] & 0xFFFF0000u);
      }
      o[j] = body2 | ex;
    }
    const uint32_t eb = (esc_bits[w0 >> 5] >> (w0 & 31)) & 0xFFFFu;
    if (eb) {
#pragma unroll
      for (int j = 0; j < kUnitWords; ++j) {
        if ((eb >> j) & 1u) {
          const uint32_t e = esc_exp[w0 + j];
          const uint32_t sh = (j & 1) * 16;
          o[j >> 1] = (o[j >> 1] & ~(0x7F80u << sh)) | ((e << 7) << sh);
        }
      }
    }
    store_unit(a.dst, a.L, g, valid, o, vec);
  }

  // ---- last CTA: streams whose entries were not all found by the tiles ---
  if (count == 0) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&g_decode_slots[a.slot].done, 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const uint32_t covered = ld_volatile_u32(&g_decode_slots[a.slot].covered);
  if (covered != count) {
    // Entries out of position order (or positions >= n): apply every entry,
    // exactly as ApplyTop16Escapes does (.cu:253-284).
    for (uint64_t i = tid; i < count; i += kThreads) {
      const uint32_t p = entry_pos(entries, i);
      if (p >= a.n) continue;
      uint16_t* w = a.dst + layout_addr(a.L, p);
      *w = static_cast<uint16_t>((__ldcg(w) & 0x807Fu) | (static_cast<uint32_t>(__ldg(entries + i * 5 + 4)) << 7));
    }
  }
  __syncthreads();
  if (tid == 0) {
    g_decode_slots[a.slot].done = 0;
    g_decode_slots[a.slot].covered = 0;
  }
}

struct Fixed6DecodeArgs {
  const uint8_t* src;
  uint16_t* dst;
  Layout L;
  uint64_t n;
  int vec;
};

__global__ void __launch_bounds__(kThreads) DecodeFixed6Kernel(const Fixed6DecodeArgs a) {
  __shared__ __align__(128) uint8_t slow[kTileWords + 64];
  __shared__ __align__(128) uint8_t scodes[kTileWords * 3 / 4 + 64];
  __shared__ uint32_t spal[64];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (__ldg(a.src) != 3) return;  // DecodeFixed6 .cu:121: write nothing
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (tid < 64) spal[tid] = static_cast<uint32_t>(__ldg(a.src + 1 + tid)) << 8;
  __syncthreads();
  const uint64_t t0 = static_cast<uint64_t>(blockIdx.x) * kTileWords;
  const uint32_t len = static_cast<uint32_t>(a.n - t0 < kTileWords ? a.n - t0 : kTileWords);
  const uint32_t pad_l = stage_bytes(a.src, 65 + t0, len, slow, &bar);
  const uint32_t pad_c = stage_bytes(a.src, 65 + a.n + 3 * t0 / 4, 3 * ((len + 3) / 4), scodes, &bar);
  if (tid == 0) mbar_arrive(&bar);
  bool ok = mbar_wait(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) raise_error(nullptr);
    mbar_wait(&bar, 0);
    __syncthreads();
  }
  const bool vec = a.vec != 0;
#pragma unroll
  for (int s = 0; s < kStepsPerWarp; ++s) {
    const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
    if (w0 >= len) continue;
    const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
    uint32_t Lw[4];
    smem_read16(slow, pad_l + w0, Lw);
    uint32_t Q[3];
    smem_read_words<3>(scodes, pad_c + 3 * w0 / 4, Q);
    uint32_t c[16];
    c[0] = Q[0] & 63; c[1] = (Q[0] >> 6) & 63; c[2] = (Q[0] >> 12) & 63; c[3] = (Q[0] >> 18) & 63;
    c[4] = (Q[0] >> 24) & 63; c[5] = ((Q[0] >> 30) | (Q[1] << 2)) & 63;
    c[6] = (Q[1] >> 4) & 63; c[7] = (Q[1] >> 10) & 63; c[8] = (Q[1] >> 16) & 63;
    c[9] = (Q[1] >> 22) & 63; c[10] = ((Q[1] >> 28) | (Q[2] << 4)) & 63;
    c[11] = (Q[2] >> 2) & 63; c[12] = (Q[2] >> 8) & 63; c[13] = (Q[2] >> 14) & 63;
    c[14] = (Q[2] >> 20) & 63; c[15] = (Q[2] >> 26) & 63;
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t l2 = __byte_perm(Lw[j >> 1], 0, (j & 1) ? 0x4342 : 0x4140);
      o[j] = l2 | spal[c[2 * j]] | (spal[c[2 * j + 1]] << 16);
    }
    store_unit(a.dst, a.L, t0 + w0, valid, o, vec);
  }
}

// =====================================================================
// host helpers
// =====================================================================

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

// Scratch of the top16 encoder, placed after the stream at a 16-byte aligned
// absolute address: [0,4) tile ticket, [4,8) error flag, [16, 16+8*tiles)
// look-back status words.
uint64_t top16_scratch_offset(const uint8_t* dst, uint64_t encoded) {
  const uintptr_t end = reinterpret_cast<uintptr_t>(dst) + encoded;
  return ((end + 15) & ~static_cast<uintptr_t>(15)) - reinterpret_cast<uintptr_t>(dst);
}

uint64_t top16_scratch_bytes(uint64_t n) { return 16 + 8 * tiles_for(n); }

long long encode_top16_impl(const uint16_t* src, const Layout& L, uint8_t* dst,
                            unsigned long long capacity, const uint8_t* tables,
                            cudaStream_t stream) {
  const uint64_t n = L.n;
  const uint64_t code_bytes = (n + 1) / 2;
  const uint64_t cap = (n + 199) / 200;
  const uint64_t encoded = 5 + n + code_bytes + cap * 5;
  // Reference decline rules (.cu:385-395) ...
  if (encoded >= n * 2 || ((encoded + 3) & ~3ULL) + 8 > capacity) return 0;
  // ... plus room for this implementation's tile-scan scratch.
  const uint64_t so = top16_scratch_offset(dst, encoded);
  const uint64_t scratch = top16_scratch_bytes(n);
  if (so + scratch > capacity) return 0;
  const uint64_t entries = 5 + n + code_bytes;
  cudaError_t st = cudaMemsetAsync(dst + entries, 0, so + scratch - entries, stream);
  if (st != cudaSuccess) return Fail("cudaMemsetAsync", st);
  Top16EncodeArgs a{};
  a.src = src;
  a.L = L;
  a.bulk = bulk_ok(src, L);
  a.dst = dst;
  a.n = n;
  a.half = n / 2;
  a.cap = cap;
  a.num_tiles = static_cast<uint32_t>(tiles_for(n));
  a.tables = tables;
  a.ticket = reinterpret_cast<uint32_t*>(dst + so);
  a.error = reinterpret_cast<uint32_t*>(dst + so + 4);
  a.status = reinterpret_cast<uint64_t*>(dst + so + 16);
  EncodeTop16Kernel<<<a.num_tiles, kThreads, 0, stream>>>(a);
  st = cudaGetLastError();
  if (st != cudaSuccess) return Fail("EncodeTop16Kernel", st);
  return static_cast<long long>(encoded);
}

long long encode_fixed_impl(const uint16_t* src, const Layout& L, uint8_t* dst,
                            unsigned long long capacity, int bits, cudaStream_t stream) {
  const uint64_t n = L.n;
  const uint64_t code_bytes = bits == 5 ? ((n + 7) / 8) * 5 : ((n + 3) / 4) * 3;
  const uint64_t header = bits == 5 ? 33 : 65;
  const uint64_t encoded = header + n + code_bytes;
  const uint64_t scratch_offset = (encoded + 3) & ~3ULL;
  const uint64_t scratch = 256 * sizeof(int) + 2 * sizeof(int);  // reference rule (.cu:305)
  if (encoded >= n * 2 || scratch_offset + scratch > capacity) return 0;
  // the presence bitmap and error flag live at the (4-byte aligned) scratch
  if ((reinterpret_cast<uintptr_t>(dst) + scratch_offset) % 4) return 0;
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(dst + scratch_offset);
  uint32_t* error = bitmap + 8;
  cudaError_t st = cudaMemsetAsync(bitmap, 0, 9 * sizeof(uint32_t), stream);
  if (st != cudaSuccess) return Fail("cudaMemsetAsync", st);
  const uint32_t tiles = static_cast<uint32_t>(tiles_for(n));
  const int bulk = bulk_ok(src, L);
  PresenceArgs p{src, L, bulk, n, bitmap, error};
  HighBytePresenceKernel<<<tiles, kThreads, 0, stream>>>(p);
  st = cudaGetLastError();
  if (st != cudaSuccess) return Fail("HighBytePresenceKernel", st);
  FixedEncodeArgs e{src, L, bulk, dst, n, bitmap, error};
  if (bits == 5) {
    EncodeFixedKernel<5><<<tiles, kThreads, 0, stream>>>(e);
  } else {
    EncodeFixedKernel<6><<<tiles, kThreads, 0, stream>>>(e);
  }
  st = cudaGetLastError();
  if (st != cudaSuccess) return Fail(bits == 5 ? "EncodeFixed5Kernel" : "EncodeFixed6Kernel", st);
  return static_cast<long long>(encoded);
}

long long decode_top16_impl(const uint8_t* src, unsigned long long encoded_bytes, uint16_t* dst,
                            const Layout& L, const uint8_t* tables, cudaStream_t stream) {
  const uint64_t n = L.n;
  const uint64_t cap = (n + 199) / 200;
  if (encoded_bytes != 5 + n + (n + 1) / 2 + cap * 5) return 0;
  Top16DecodeArgs a{};
  a.src = src;
  a.dst = dst;
  a.L = L;
  a.n = n;
  a.half = n / 2;
  a.cap = cap;
  a.tables = tables;
  a.vec = vec_ok(dst, L);
  a.slot = g_decode_slot_counter.fetch_add(1, std::memory_order_relaxed) % kDecodeSlots;
  DecodeTop16Kernel<<<static_cast<unsigned>(tiles_for(n)), kThreads, 0, stream>>>(a);
  const cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return Fail("DecodeTop16Kernel", st);
  return static_cast<long long>(n * sizeof(uint16_t));
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
  return encode_fixed_impl(reinterpret_cast<const uint16_t*>(src_ptr), flat_layout(count),
                           reinterpret_cast<uint8_t*>(dst_ptr), capacity, bits,
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
    unsigned long long count_words, unsigned long long block_count,
    unsigned long long block_words, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_start,
    unsigned long long block_ids_ptr, unsigned long long stream_ptr) {
  if (src_ptr == 0 || dst_ptr == 0 || count_words == 0 || block_count == 0 ||
      block_words == 0 || count_words != 2 * block_count * block_words) {
    return 0;
  }
  const unsigned long long expected = 65 + count_words + ((count_words + 3) / 4) * 3;
  if (encoded_bytes != expected) return 0;
  Fixed6DecodeArgs a{};
  a.src = reinterpret_cast<const uint8_t*>(src_ptr);
  a.dst = reinterpret_cast<uint16_t*>(dst_ptr);
  a.L = block_layout(block_count, block_words, plane_stride, block_stride, block_start,
                     reinterpret_cast<const int64_t*>(block_ids_ptr));
  a.n = count_words;
  a.vec = vec_ok(a.dst, a.L);
  DecodeFixed6Kernel<<<static_cast<unsigned>(tiles_for(count_words)), kThreads, 0,
                       reinterpret_cast<cudaStream_t>(stream_ptr)>>>(a);
  const cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return Fail("DecodeFixed6Kernel", st);
  return static_cast<long long>(count_words * sizeof(uint16_t));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_fixed6(
    unsigned long long src_ptr, unsigned long long encoded_bytes, unsigned long long dst_ptr,
    unsigned long long count_words, unsigned long long block_count,
    unsigned long long block_words, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_start,
    unsigned long long stream_ptr) {
  return kvq_splitzip_bf16_decode_fixed6_blocks(src_ptr, encoded_bytes, dst_ptr, count_words,
                                                block_count, block_words, plane_stride,
                                                block_stride, block_start, 0, stream_ptr);
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
  return encode_top16_impl(reinterpret_cast<const uint16_t*>(src_ptr), flat_layout(count),
                           reinterpret_cast<uint8_t*>(dst_ptr), capacity,
                           reinterpret_cast<const uint8_t*>(tables_ptr),
                           reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_top16_blocks(
    unsigned long long src_ptr, unsigned long long encoded_bytes, unsigned long long dst_ptr,
    unsigned long long count_words, unsigned long long block_count,
    unsigned long long block_words, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_start,
    unsigned long long block_ids_ptr, unsigned long long tables_ptr,
    unsigned long long stream_ptr) {
  if (src_ptr == 0 || dst_ptr == 0 || tables_ptr == 0 || count_words == 0 || block_count == 0 ||
      block_words == 0 || count_words != 2 * block_count * block_words) {
    return 0;
  }
  return decode_top16_impl(
      reinterpret_cast<const uint8_t*>(src_ptr), encoded_bytes,
      reinterpret_cast<uint16_t*>(dst_ptr),
      block_layout(block_count, block_words, plane_stride, block_stride, block_start,
                   reinterpret_cast<const int64_t*>(block_ids_ptr)),
      reinterpret_cast<const uint8_t*>(tables_ptr), reinterpret_cast<cudaStream_t>(stream_ptr));
}

extern "C" KVQ_API long long kvq_splitzip_bf16_decode_top16(
    unsigned long long src_ptr, unsigned long long encoded_bytes, unsigned long long dst_ptr,
    unsigned long long count_words, unsigned long long block_count,
    unsigned long long block_words, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_start,
    unsigned long long tables_ptr, unsigned long long stream_ptr) {
  return kvq_splitzip_bf16_decode_top16_blocks(src_ptr, encoded_bytes, dst_ptr, count_words,
                                               block_count, block_words, plane_stride,
                                               block_stride, block_start, 0, tables_ptr,
                                               stream_ptr);
}

// ---------------------------------------------------------------------
// Extensions (no counterpart in the reference ABI; same conventions)
// ---------------------------------------------------------------------

// Fused gather + top16 encode.  Produces exactly the bytes of
// torch.index_select(kv_layer, 1, block_ids) followed by
// kvq_splitzip_bf16_encode_top16 on the packed copy, without the copy.
extern "C" KVQ_API long long kvq_splitzip_bf16_encode_top16_blocks(
    unsigned long long cache_ptr, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_words,
    unsigned long long block_ids_ptr, unsigned long long block_start,
    unsigned long long block_count, unsigned long long dst_ptr, unsigned long long capacity,
    unsigned long long tables_ptr, unsigned long long stream_ptr) {
  if (cache_ptr == 0 || dst_ptr == 0 || tables_ptr == 0 || block_count == 0 ||
      block_words == 0) {
    return 0;
  }
  const Layout L = block_layout(block_count, block_words, plane_stride, block_stride,
                                block_start, reinterpret_cast<const int64_t*>(block_ids_ptr));
  if (L.n > 0xFFFFFFFFULL) return 0;
  return encode_top16_impl(reinterpret_cast<const uint16_t*>(cache_ptr), L,
                           reinterpret_cast<uint8_t*>(dst_ptr), capacity,
                           reinterpret_cast<const uint8_t*>(tables_ptr),
                           reinterpret_cast<cudaStream_t>(stream_ptr));
}

// Fused gather + fixed6/fixed5 encode (bits 6 or 5), bytes identical to
// index_select followed by kvq_splitzip_bf16_encode_mode.
extern "C" KVQ_API long long kvq_splitzip_bf16_encode_mode_blocks(
    unsigned long long cache_ptr, unsigned long long plane_stride,
    unsigned long long block_stride, unsigned long long block_words,
    unsigned long long block_ids_ptr, unsigned long long block_start,
    unsigned long long block_count, unsigned long long dst_ptr, unsigned long long capacity,
    unsigned long long stream_ptr, int bits) {
  if (cache_ptr == 0 || dst_ptr == 0 || block_count == 0 || block_words == 0) return 0;
  if (bits != 5 && bits != 6) return 0;
  const Layout L = block_layout(block_count, block_words, plane_stride, block_stride,
                                block_start, reinterpret_cast<const int64_t*>(block_ids_ptr));
  return encode_fixed_impl(reinterpret_cast<const uint16_t*>(cache_ptr), L,
                           reinterpret_cast<uint8_t*>(dst_ptr), capacity, bits,
                           reinterpret_cast<cudaStream_t>(stream_ptr));
}

// Number of device-side bounded waits that ran out on the current device
// since the library was loaded (0 in normal operation).  Synchronous.
extern "C" KVQ_API long long kvq_splitzip_device_errors() {
  unsigned int value = 0;
  const cudaError_t st = cudaMemcpyFromSymbol(&value, g_device_errors, sizeof(value));
  if (st != cudaSuccess) return Fail("cudaMemcpyFromSymbol", st);
  return static_cast<long long>(value);
}

// ABI revision of this library (bumped when an extension entry point changes).
extern "C" KVQ_API long long kvq_splitzip_abi_version() { return 1; }
