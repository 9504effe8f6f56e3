// Device-side building blocks shared by the splitzip kernels (sm_100a).
//
// * TMA bulk staging: cp.async.bulk global->shared with an mbarrier carrying
//   the transaction count; every wait is bounded.
// * Warp "funnel" stores: a warp writes a contiguous run of output bytes whose
//   start is not aligned (the splitzip stream regions begin at byte 5, 65 or
//   33 and at 5+n, ...).  Each lane owns K slots of S bytes; the lane shifts
//   its bytes by the run's misalignment, borrowing the next lane's first
//   bytes, so every interior store is an aligned S-byte store.  Only the two
//   end slots of a run are written bytewise, clipped to the run.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ukv {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnitWords = 16;                        // words per lane per step
constexpr int kStepWords = 32 * kUnitWords;           // 512 words per warp step
constexpr int kStepsPerWarp = 4;
constexpr int kTileWords = kWarps * kStepsPerWarp * kStepWords;  // 16384 (32 KiB of words)
constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------- layouts

// Packed word index i in [0, n) -> element offset.  block_words == 0 is a flat
// buffer.  Otherwise the index walks the [2, block_count, block_words] view of
// a paged cache [2, num_blocks, ...] whose block `id(b)` starts at
// plane*plane_stride + id(b)*block_stride; id(b) = ids[b] or block_start + b.
struct Layout {
  uint64_t n;
  uint64_t plane_words;
  uint64_t block_words;
  uint64_t plane_stride;
  uint64_t block_stride;
  uint64_t block_start;
  const int64_t* ids;
  int bw_shift;  // log2(block_words) when a power of two, else -1
};

__device__ __forceinline__ uint64_t layout_addr(const Layout& L, uint64_t i) {
  if (L.block_words == 0) return i;
  const uint64_t plane = i >= L.plane_words;
  const uint64_t rem = i - (plane ? L.plane_words : 0);
  uint64_t blk, within;
  if (L.bw_shift >= 0) {
    blk = rem >> L.bw_shift;
    within = rem & (L.block_words - 1);
  } else {
    blk = rem / L.block_words;
    within = rem - blk * L.block_words;
  }
  const uint64_t b = L.ids ? static_cast<uint64_t>(__ldg(L.ids + blk)) : L.block_start + blk;
  return plane * L.plane_stride + b * L.block_stride + within;
}

// Words left in the contiguous run that starts at packed index i.
__device__ __forceinline__ uint64_t layout_run(const Layout& L, uint64_t i) {
  if (L.block_words == 0) return L.n - i;
  const uint64_t rem = i >= L.plane_words ? i - L.plane_words : i;
  const uint64_t within = L.bw_shift >= 0 ? (rem & (L.block_words - 1)) : rem % L.block_words;
  return L.block_words - within;
}

// ------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch.  Kernels of this library are launched so
// that each may start while the previous kernel of its stream finishes: a
// kernel touches nothing in global memory before grid_dependency_wait()
// returns (the previous grid has completed and its writes are visible), and
// every CTA calls grid_dependency_release() once it is past that point, so
// the next kernel's CTAs can be scheduled as this grid's CTAs retire.  In a
// launch without the attribute both are no-ops.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependency_release() { asm volatile("griddepcontrol.launch_dependents;" :::); }
__device__ __forceinline__ void grid_dependency_sync() {
  grid_dependency_wait();
  grid_dependency_release();
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

// One try_wait that suspends the thread (up to `hint_ns`) while the phase is
// incomplete, so a waiting warp does not spin on the issue slots of the
// warps that are working.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase: at most kTries suspended tries of up to
// 1 ms each (kBarrierTries in every product kernel; a test-only
// instantiation uses a few).  Returns false if the limit ran out.
constexpr uint32_t kBarrierTries = 4096;
template <uint32_t kTries = kBarrierTries>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kTries; ++i) {
    if (mbar_try_wait(bar, parity, 1000000u)) return true;
  }
  return false;
}

// 1-D TMA bulk copy global -> shared, completion counted on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* sdst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(sdst)),
      "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// ------------------------------------------------------- warp funnel store

// Byte store to global memory under a predicate (no branch).
__device__ __forceinline__ void st_global_u8_if(bool p, uint8_t* a, uint32_t v) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %0, 0;\n\t@q st.global.u8 [%1], %2;\n\t}" ::"r"(
          static_cast<uint32_t>(p)),
      "l"(a), "r"(v)
      : "memory");
}

// Store bytes [max(slot,lo), min(slot+S,hi)) of the little-endian value v
// that belongs at `slot` (an S-aligned address).  Full slots use one aligned
// store; clipped slots fall back to 4/2/1-byte aligned stores.
template <typename T>
__device__ __forceinline__ void store_clipped(uintptr_t slot, uint64_t v, uintptr_t lo,
                                              uintptr_t hi) {
  constexpr uintptr_t S = sizeof(T);
  uintptr_t a = slot > lo ? slot : lo;
  uintptr_t b = slot + S < hi ? slot + S : hi;
  if (a >= b) return;
  if (a == slot && b == slot + S) {
    *reinterpret_cast<T*>(slot) = static_cast<T>(v);
    return;
  }
  while (a < b) {
    const uint32_t off = static_cast<uint32_t>(a - slot);
    const uintptr_t rem = b - a;
    if ((a & 3) == 0 && rem >= 4) {
      *reinterpret_cast<uint32_t*>(a) = static_cast<uint32_t>(v >> (8 * off));
      a += 4;
    } else if ((a & 1) == 0 && rem >= 2) {
      *reinterpret_cast<uint16_t*>(a) = static_cast<uint16_t>(v >> (8 * off));
      a += 2;
    } else {
      *reinterpret_cast<uint8_t*>(a) = static_cast<uint8_t>(v >> (8 * off));
      a += 1;
    }
  }
}

// A warp writes a contiguous byte run starting at g: lane L owns bytes
// [g + L*K*S, g + (L+1)*K*S) given as K little-endian S-byte values d[k].
// Bytes at or past g + valid, and bytes before g, are never written.  All 32
// lanes must call this (it shuffles).
template <typename T, int K>
__device__ __forceinline__ void warp_store(uint8_t* g, uint32_t valid, const T (&d)[K],
                                           int lane) {
  constexpr uint32_t S = sizeof(T);
  const uintptr_t base = reinterpret_cast<uintptr_t>(g);
  const uintptr_t hi = base + valid;
  const uint32_t s = static_cast<uint32_t>(base % S);
  const uintptr_t mine = base + static_cast<uintptr_t>(lane) * K * S;
  const T next0 = __shfl_down_sync(kFull, d[0], 1);
  if (s == 0) {
#pragma unroll
    for (int k = 0; k < K; ++k) store_clipped<T>(mine + k * S, static_cast<uint64_t>(d[k]), base, hi);
    return;
  }
  const uintptr_t s0 = mine - s;
  if (lane == 0) store_clipped<T>(s0, static_cast<uint64_t>(d[0]) << (8 * s), base, hi);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const uint64_t cur = static_cast<uint64_t>(d[k]);
    const uint64_t nxt = static_cast<uint64_t>(k + 1 < K ? d[(k + 1) % K] : next0);
    const uint64_t v = (cur >> (8 * (S - s))) | (nxt << (8 * s));
    const uintptr_t slot = s0 + (k + 1) * S;
    uintptr_t h = hi;
    if (k == K - 1 && lane == 31 && slot + s < h) h = slot + s;
    store_clipped<T>(slot, v, base, h);
  }
}

// Bytes [0, count) of the little-endian value v to the (unaligned) address a.
__device__ __forceinline__ void store_bytes(uintptr_t a, uint64_t v, uint32_t count) {
  for (uint32_t i = 0; i < count; ++i) reinterpret_cast<uint8_t*>(a)[i] = static_cast<uint8_t>(v >> (8 * i));
}

// warp_store for a run whose 32*K*S bytes are all valid: every interior slot
// is one aligned S-byte store; only lane 0's head and lane 31's tail (less
// than S bytes each) are written bytewise.
template <typename T, int K>
__device__ __forceinline__ void warp_store_full(uint8_t* g, const T (&d)[K], int lane) {
  constexpr uint32_t S = sizeof(T);
  const uintptr_t base = reinterpret_cast<uintptr_t>(g);
  const uint32_t s = static_cast<uint32_t>(base % S);
  if (s == 0) {
    T* p = reinterpret_cast<T*>(base) + lane * K;
#pragma unroll
    for (int k = 0; k < K; ++k) p[k] = d[k];
    return;
  }
  const T next0 = __shfl_down_sync(kFull, d[0], 1);
  T* slots = reinterpret_cast<T*>(base - s) + lane * K + 1;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const uint64_t cur = static_cast<uint64_t>(d[k]);
    const uint64_t nxt = static_cast<uint64_t>(k + 1 < K ? d[(k + 1) % K] : next0);
    const uint64_t v = (cur >> (8 * (S - s))) | (nxt << (8 * s));
    if (k < K - 1 || lane < 31) slots[k] = static_cast<T>(v);
  }
  if (lane == 0) store_bytes(base, static_cast<uint64_t>(d[0]), S - s);
  if (lane == 31) store_bytes(base + 32 * K * S - s, static_cast<uint64_t>(d[K - 1]) >> (8 * (S - s)), s);
}

// warp_store_full on 32-bit words: lane L owns the NW words D (bytes
// [g + 4*NW*L, g + 4*NW*(L+1))) and writes aligned S-byte slots (S = 4 or 8,
// 4*NW a multiple of S).  The slot data comes from one uniform word select
// and one funnel shift per word; the less-than-S bytes at each end of the run
// are written by up to 7 lanes with one byte store each (no divergent loop).
template <int NW, int S>
__device__ __forceinline__ void warp_store_words(uint8_t* g, const uint32_t (&D)[NW], int lane) {
  static_assert(S == 4 || S == 8, "slot size");
  static_assert((4 * NW) % S == 0, "whole slots per lane");
  const uintptr_t base = reinterpret_cast<uintptr_t>(g);
  const uint32_t s = static_cast<uint32_t>(base % S);
  if (s == 0) {
    if (S == 8) {
      uint2* p = reinterpret_cast<uint2*>(base) + lane * (NW / 2);
#pragma unroll
      for (int k = 0; k < NW / 2; ++k) p[k] = make_uint2(D[2 * k], D[2 * k + 1]);
    } else {
      uint32_t* p = reinterpret_cast<uint32_t*>(base) + lane * NW;
#pragma unroll
      for (int k = 0; k < NW; ++k) p[k] = D[k];
    }
    return;
  }
  const uint32_t o = S - s;                 // run bytes before the first aligned slot
  const bool q = (o & 4) != 0;              // word offset of that slot in the lane's data
  const uint32_t r = (o & 3) * 8;           // bit offset inside the word
  // the lane's words followed by the next lane's first two
  uint32_t W[NW + 2];
#pragma unroll
  for (int k = 0; k < NW; ++k) W[k] = D[k];
  W[NW] = __shfl_down_sync(kFull, D[0], 1);
  W[NW + 1] = NW > 1 ? __shfl_down_sync(kFull, D[NW > 1 ? 1 : 0], 1) : 0u;
  uint32_t Wq[NW + 1];
#pragma unroll
  for (int k = 0; k < NW + 1; ++k) Wq[k] = q ? W[k + 1] : W[k];
  uint32_t out[NW];
#pragma unroll
  for (int k = 0; k < NW; ++k) out[k] = __funnelshift_r(Wq[k], Wq[k + 1], r);
  // aligned slots; lane 31's last slot reaches past the run and is left to
  // the tail bytes below
  const uintptr_t first = base + o + static_cast<uintptr_t>(lane) * 4 * NW;
  if (S == 8) {
    uint2* p = reinterpret_cast<uint2*>(first);
#pragma unroll
    for (int k = 0; k < NW / 2; ++k)
      if (k < NW / 2 - 1 || lane < 31) p[k] = make_uint2(out[2 * k], out[2 * k + 1]);
  } else {
#pragma unroll
    for (int k = 0; k < NW; ++k)
      if (k < NW - 1 || lane < 31) reinterpret_cast<uint32_t*>(first)[k] = out[k];
  }
  // head: run bytes [0, o) are lane 0's first bytes; tail: the run's last s
  // bytes are lane 31's last bytes
  const uint32_t h0 = __shfl_sync(kFull, D[0], 0);
  const uint32_t h1 = __shfl_sync(kFull, D[NW > 1 ? 1 : 0], 0);
  const uint32_t t0 = __shfl_sync(kFull, D[NW > 1 ? NW - 2 : 0], 31);
  const uint32_t t1 = __shfl_sync(kFull, D[NW - 1], 31);
  {
    const uint32_t word = lane < 4 ? h0 : h1;
    st_global_u8_if(static_cast<uint32_t>(lane) < o, reinterpret_cast<uint8_t*>(base) + lane,
                    (word >> (8 * (lane & 3))) & 0xFFu);
  }
  {
    // byte (4*NW - s + lane) of lane 31's data
    const uint32_t idx = 4 * NW - s + lane;
    const uint32_t word = (idx >> 2) == static_cast<uint32_t>(NW - 1) ? t1 : t0;
    st_global_u8_if(static_cast<uint32_t>(lane) < s, reinterpret_cast<uint8_t*>(base + 32 * 4 * NW - s) + lane,
                    (word >> (8 * (idx & 3))) & 0xFFu);
  }
}

// Read 16 bytes starting at an arbitrary byte offset of a 4-byte aligned
// shared buffer (the buffer must extend 4 bytes past the read).
__device__ __forceinline__ void smem_read16(const uint8_t* buf, uint32_t off, uint32_t (&out)[4]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(buf) + (off >> 2);
  const uint32_t sh = (off & 3) * 8;
  uint32_t a[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) a[k] = w[k];
#pragma unroll
  for (int k = 0; k < 4; ++k) out[k] = __funnelshift_r(a[k], a[k + 1], sh);
}

// Read 16 bytes at byte offset `off` of a 16-byte aligned shared buffer with
// two aligned 16-byte loads (lanes reading consecutive 16-byte units hit
// distinct banks) and a funnel shift.  The buffer must extend 32 bytes past
// off & ~15.
__device__ __forceinline__ void smem_read16_window(const uint8_t* buf, uint32_t off, uint32_t (&out)[4]) {
  const uint4* q = reinterpret_cast<const uint4*>(buf) + (off >> 4);
  const uint4 a = q[0];
  const uint4 b = q[1];
  const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const bool s2 = (off & 8) != 0;
  const bool s1 = (off & 4) != 0;
  uint32_t w[6];
#pragma unroll
  for (int k = 0; k < 6; ++k) w[k] = s2 ? v[k + 2] : v[k];
  uint32_t u[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) u[k] = s1 ? w[k + 1] : w[k];
  const uint32_t sh = (off & 3) * 8;
#pragma unroll
  for (int k = 0; k < 4; ++k) out[k] = __funnelshift_r(u[k], u[k + 1], sh);
}

// Read 8 bytes at byte offset `off` of an 8-byte aligned shared buffer with
// two aligned 8-byte loads and a funnel shift (buffer extends 16 bytes past
// off & ~7).
__device__ __forceinline__ void smem_read8_window(const uint8_t* buf, uint32_t off, uint32_t (&out)[2]) {
  const uint2* q = reinterpret_cast<const uint2*>(buf) + (off >> 3);
  const uint2 a = q[0];
  const uint2 b = q[1];
  const uint32_t v[4] = {a.x, a.y, b.x, b.y};
  const bool s1 = (off & 4) != 0;
  uint32_t w[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) w[k] = s1 ? v[k + 1] : v[k];
  const uint32_t sh = (off & 3) * 8;
  out[0] = __funnelshift_r(w[0], w[1], sh);
  out[1] = __funnelshift_r(w[1], w[2], sh);
}

template <int N>
__device__ __forceinline__ void smem_read_words(const uint8_t* buf, uint32_t off, uint32_t (&out)[N]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(buf) + (off >> 2);
  const uint32_t sh = (off & 3) * 8;
  uint32_t a[N + 1];
#pragma unroll
  for (int k = 0; k < N + 1; ++k) a[k] = w[k];
#pragma unroll
  for (int k = 0; k < N; ++k) out[k] = __funnelshift_r(a[k], a[k + 1], sh);
}

// Store a warp's run of K steps: in step k lane L owns the 4*NW bytes at run
// offset 4*NW*(32k + L), held in D[k].  Aligned S-byte slots (S = 4 or 8,
// 4*NW a multiple of S) take the bytes that straddle two lanes, or two steps
// (lane 31 of step k and lane 0 of step k+1), by one shuffle per word; only
// the < S bytes at each end of the run go out as single byte stores.
template <int NW, int S, int K>
__device__ __forceinline__ void warp_store_run(uint8_t* g, const uint32_t (&D)[K][NW], int lane) {
  static_assert(S == 4 || S == 8, "slot size");
  static_assert(NW >= 2 && (4 * NW) % S == 0, "whole slots per lane");
  constexpr uint32_t kLaneBytes = 4 * NW;
  constexpr uint32_t kStepBytes = 32 * kLaneBytes;
  const uintptr_t base = reinterpret_cast<uintptr_t>(g);
  const uint32_t s = static_cast<uint32_t>(base % S);
  if (s == 0) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (S == 8) {
        uint2* p = reinterpret_cast<uint2*>(base + k * kStepBytes) + lane * (NW / 2);
#pragma unroll
        for (int j = 0; j < NW / 2; ++j) p[j] = make_uint2(D[k][2 * j], D[k][2 * j + 1]);
      } else {
        uint32_t* p = reinterpret_cast<uint32_t*>(base + k * kStepBytes) + lane * NW;
#pragma unroll
        for (int j = 0; j < NW; ++j) p[j] = D[k][j];
      }
    }
    return;
  }
  const uint32_t o = S - s;     // run bytes before the first aligned slot
  const bool q = (o & 4) != 0;  // word offset of that slot in the lane's data
  const uint32_t r = (o & 3) * 8;
  const int src = (lane + 1) & 31;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    // the next lane's first two words; lane 31 reads lane 0 of step k+1
    const bool wrap = lane == 0 && k + 1 < K;
    const uint32_t n0 = wrap ? D[k + 1 < K ? k + 1 : k][0] : D[k][0];
    const uint32_t n1 = wrap ? D[k + 1 < K ? k + 1 : k][1] : D[k][1];
    uint32_t W[NW + 2];
#pragma unroll
    for (int j = 0; j < NW; ++j) W[j] = D[k][j];
    W[NW] = __shfl_sync(kFull, n0, src);
    W[NW + 1] = __shfl_sync(kFull, n1, src);
    uint32_t out[NW];
#pragma unroll
    for (int j = 0; j < NW; ++j) {
      const uint32_t a = q ? W[j + 1] : W[j];
      const uint32_t b = q ? W[j + 2] : W[j + 1];
      out[j] = __funnelshift_r(a, b, r);
    }
    // lane 31's last slot of the last step reaches past the run: the tail
    // bytes below cover its part
    const uintptr_t first = base + o + k * kStepBytes + static_cast<uintptr_t>(lane) * kLaneBytes;
    const bool last_lane = k == K - 1 && lane == 31;
    if (S == 8) {
      uint2* p = reinterpret_cast<uint2*>(first);
#pragma unroll
      for (int j = 0; j < NW / 2; ++j)
        if (j < NW / 2 - 1 || !last_lane) p[j] = make_uint2(out[2 * j], out[2 * j + 1]);
    } else {
      uint32_t* p = reinterpret_cast<uint32_t*>(first);
#pragma unroll
      for (int j = 0; j < NW; ++j)
        if (j < NW - 1 || !last_lane) p[j] = out[j];
    }
  }
  // head: run bytes [0, o) are lane 0's first bytes of step 0; tail: the
  // run's last s bytes are lane 31's last bytes of step K-1
  const uint32_t h0 = __shfl_sync(kFull, D[0][0], 0);
  const uint32_t h1 = __shfl_sync(kFull, D[0][1], 0);
  const uint32_t t0 = __shfl_sync(kFull, D[K - 1][NW - 2], 31);
  const uint32_t t1 = __shfl_sync(kFull, D[K - 1][NW - 1], 31);
  {
    const uint32_t word = lane < 4 ? h0 : h1;
    st_global_u8_if(static_cast<uint32_t>(lane) < o, reinterpret_cast<uint8_t*>(base) + lane,
                    (word >> (8 * (lane & 3))) & 0xFFu);
  }
  {
    const uint32_t idx = kLaneBytes - s + lane;  // byte of lane 31's data
    const uint32_t word = (idx >> 2) == static_cast<uint32_t>(NW - 1) ? t1 : t0;
    st_global_u8_if(static_cast<uint32_t>(lane) < s,
                    reinterpret_cast<uint8_t*>(base + K * kStepBytes - s) + lane, (word >> (8 * (idx & 3))) & 0xFFu);
  }
}

// ---------------------------------------------------------------- staging

// Lane k's run of a tile for TMA staging (runs are the intersections of the
// tile with cache blocks; the flat layout has one, staged by lane 0): its
// first word, global source and bytes (0: none).  The block-table load
// happens here, so a producer can plan the next tile while the current one
// is staged and waited for.
struct RunPlan {
  uint64_t s0;
  const uint16_t* src;
  uint32_t bytes;
};

__device__ __forceinline__ RunPlan plan_run(const uint16_t* __restrict__ base, const Layout& L, uint64_t t0,
                                            uint32_t len, uint32_t k) {
  RunPlan r{0, nullptr, 0};
  if (L.block_words == 0) {
    if (k == 0) {
      r.s0 = t0;
      r.src = base + t0;
      r.bytes = (len & ~7u) * 2;
    }
    return r;
  }
  const uint64_t bw = L.block_words;
  const uint64_t first = L.bw_shift >= 0 ? t0 >> L.bw_shift : t0 / bw;  // no 64-bit division for 2^k blocks
  const uint64_t b0 = (first + k) * bw;
  const uint64_t s0 = b0 > t0 ? b0 : t0;
  const uint64_t end = t0 + len;
  if (s0 >= end) return r;
  const uint64_t e0 = b0 + bw < end ? b0 + bw : end;
  r.s0 = s0;
  r.src = base + layout_addr(L, s0);
  r.bytes = static_cast<uint32_t>((e0 - s0) * 2);
  return r;
}

// Stage a tile by TMA given each lane's planned run (plan_run(.., lane)):
// one bulk copy per contiguous run, registered on `bar` (no arrive); the
// flat layout's last < 8 words go by plain loads of lane 0.  Runs past the
// 32nd (blocks shorter than 256 words) are planned and issued here.
__device__ __forceinline__ void issue_runs(const RunPlan& r, const uint16_t* __restrict__ base, const Layout& L,
                                           uint64_t t0, uint32_t len, uint16_t* sin, uint64_t* bar) {
  const uint32_t lane = threadIdx.x & 31;
  if (r.bytes) {
    mbar_expect_tx(bar, r.bytes);
    bulk_g2s(sin + (r.s0 - t0), r.src, r.bytes, bar);
  }
  if (L.block_words == 0) {
    if (lane == 0)
      for (uint32_t j = len & ~7u; j < len; ++j) sin[j] = base[t0 + j];
    return;
  }
  // a tile meets at most ceil(kTileWords / bw) + 1 blocks: 32 or fewer (one
  // per lane, planned above) once 31 bw >= kTileWords
  if (L.block_words * 31 >= kTileWords) return;
  for (uint32_t k = lane + 32;; k += 32) {
    const RunPlan x = plan_run(base, L, t0, len, k);
    if (x.bytes == 0) break;
    mbar_expect_tx(bar, x.bytes);
    bulk_g2s(sin + (x.s0 - t0), x.src, x.bytes, bar);
  }
}

// Stage words of any layout word by word with the 32 lanes of one warp.
__device__ __forceinline__ void gather_words_warp(const uint16_t* __restrict__ base, const Layout& L, uint64_t t0,
                                                  uint32_t len, uint16_t* sin) {
  for (uint32_t j = threadIdx.x & 31; j < len; j += 32) sin[j] = base[layout_addr(L, t0 + j)];
}

// Stage bytes [off, off+nbytes) of the global buffer [g, g+glen) into shared
// memory so that byte off+i lands at smem[pad+i], pad = (g+off) % 16, by the
// calling thread alone: one TMA bulk copy (bytes registered on `bar`, no
// arrive) covers the range rounded out to 16-byte boundaries as far as the
// buffer allows; only bytes that rounding cannot reach (at the very start or
// end of the buffer) are loaded by plain loads.  Never reads outside
// [g, g+glen).  smem must hold pad + nbytes + 16 bytes.  Returns pad.
__device__ __forceinline__ uint32_t stage_bytes_one(const uint8_t* __restrict__ g, uint64_t glen, uint64_t off,
                                                    uint32_t nbytes, uint8_t* smem, uint64_t* bar) {
  const uintptr_t base = reinterpret_cast<uintptr_t>(g);
  const uintptr_t A = base + off;
  const uintptr_t E = A + nbytes;
  const uintptr_t F = A & ~static_cast<uintptr_t>(15);
  const uintptr_t gal = (base + 15) & ~static_cast<uintptr_t>(15);
  const uintptr_t gend = (base + glen) & ~static_cast<uintptr_t>(15);
  const uintptr_t Ealign = (E + 15) & ~static_cast<uintptr_t>(15);
  const uintptr_t lo = F > gal ? F : gal;
  const uintptr_t hi = Ealign < gend ? Ealign : gend;
  if (hi > lo) {
    mbar_expect_tx(bar, static_cast<uint32_t>(hi - lo));
    bulk_g2s(smem + (lo - F), reinterpret_cast<const void*>(lo), static_cast<uint32_t>(hi - lo), bar);
    for (uintptr_t a = A; a < lo; ++a) smem[a - F] = *reinterpret_cast<const uint8_t*>(a);
    for (uintptr_t a = hi > A ? hi : A; a < E; ++a) smem[a - F] = *reinterpret_cast<const uint8_t*>(a);
  } else {
    for (uintptr_t a = A; a < E; ++a) smem[a - F] = *reinterpret_cast<const uint8_t*>(a);
  }
  return static_cast<uint32_t>(A - F);
}

__device__ __forceinline__ uint32_t load_u32le(const uint8_t* __restrict__ p) {
  return static_cast<uint32_t>(__ldg(p)) | (static_cast<uint32_t>(__ldg(p + 1)) << 8) |
         (static_cast<uint32_t>(__ldg(p + 2)) << 16) | (static_cast<uint32_t>(__ldg(p + 3)) << 24);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

}  // namespace ukv
