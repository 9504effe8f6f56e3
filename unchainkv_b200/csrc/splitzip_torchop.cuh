// GPU encoder of the reference's torch-op codec forms (sm_100a).
//
// The reference connector encodes tensors its CUDA library does not take
// with torch ops (src/unchain_kv/vllm_connector.py:3204-3343, bit packing
// :3345-3366): it keeps the first of these forms that is smaller than raw,
//   mode 2, sign/magnitude, when the 7-bit magnitudes of the high bytes span
//     fewer than 7 bits: [0]=2 [1]=width [2]=least magnitude, the n low
//     bytes, n sign bits, n (magnitude - least) fields of `width` bits;
//   mode 0, palette of the distinct high bytes (at most 128): [0]=0
//     [1]=width=max(1, bitlen(distinct-1)) [2,258) the distinct high bytes
//     ascending then zeros, the n low bytes, n codes;
//   mode 1, nibble planes: [0]=1 [1,5) the widths of nibbles 0-3 (1 for
//     <= 2 distinct values, 2 for <= 4, else 4), [5,69) four 16-byte
//     palettes ascending then zeros, then the four code planes;
// all codes packed LSB first.  When none is smaller the reference sends the
// words as they are; here the stream is then mode 6 ([6] + the words).
//
// Three passes over a batch of jobs:
//   TorchopStatsKernel  presence bitmaps of the high and the low bytes
//                       (the staged pipeline of the other encoders);
//   TorchopDecideKernel one warp per job: the form, its header, and the
//                       code of each high byte / nibble (the job's plan);
//   TorchopEncodeKernel one thread per 16-word unit: every plane of these
//                       forms holds a whole number of bytes per unit (16
//                       codes of w bits are 2w bytes), so a warp's 32 units
//                       fill one contiguous run of each plane, which the
//                       warp stores together.
#pragma once

#include <type_traits>

#include "splitzip_kernels.cuh"

namespace ukv {

// A job's plan, in its scratch (16-byte aligned, zeroed before the stats).
struct TorchopPlan {
  uint32_t hi[8];      // presence of the high bytes
  uint32_t lo[8];      // presence of the low bytes
  uint32_t mode;       // 2, 0, 1, or 6
  uint32_t width;      // mode 2 / 0: bits per code
  uint32_t mag_min;    // mode 2
  uint32_t nib_width;  // mode 1: the widths of nibbles 0-3, one byte each
  uint64_t bytes;      // the stream's length
  uint64_t pad;
  uint8_t rank[256];      // mode 0: code of each high byte
  uint8_t nib_rank[64];   // mode 1: code of nibble value v of plane p at [16 p + v]
};
constexpr uint64_t kTorchopScratch = sizeof(TorchopPlan);
static_assert(kTorchopScratch == 416, "plan size (torchop_capacity in the Python module)");

template <int kMax>
struct TorchopBatch {
  uint32_t jobs;
  uint64_t unit_start[kMax + 1];
  EncJob job[kMax];
  int vec[kMax];  // 16 consecutive words of a unit are 32 aligned bytes of the cache
};

__device__ __forceinline__ TorchopPlan* plan_of(const EncJob& J) {
  return reinterpret_cast<TorchopPlan*>(J.scratch);
}

// Presence of the high and low bytes of every job (the staged pipeline).
template <int kMax>
__global__ void __launch_bounds__(kCtaThreads, 3) TorchopStatsKernel(const __grid_constant__ EncBatch<kMax> b) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(16) uint8_t shi[256];
  __shared__ __align__(16) uint8_t slo[256];
  __shared__ EncRing R;
  __shared__ EncDesc D[kEncStages];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid < 64) reinterpret_cast<uint32_t*>(shi)[tid] = 0;
  else if (tid < 128) reinterpret_cast<uint32_t*>(slo)[tid - 64] = 0;
  ring_init(R);
  __syncthreads();
  grid_dependency_sync();
  int pres_job = -1;
  auto flush = [&](const EncJob& P) {  // consumers only, every warp past its stores
    TorchopPlan* plan = plan_of(P);
    const uint32_t bh = __ballot_sync(kFull, shi[presence_index(tid)] != 0);
    const uint32_t bl = __ballot_sync(kFull, slo[presence_index(tid)] != 0);
    if (lane == 0 && bh) atomicOr(&plan->hi[warp], bh);
    if (lane == 0 && bl) atomicOr(&plan->lo[warp], bl);
    consumer_sync();
    if (tid < 64) reinterpret_cast<uint32_t*>(shi)[tid] = 0;
    else if (tid < 128) reinterpret_cast<uint32_t*>(slo)[tid - 64] = 0;
  };
  encode_pipeline<kMax>(b, ring, R, D, [&](const EncJob& J, int j, uint32_t tile, const uint16_t* sin,
                                           const EncPos&, const EncDesc&) {
    if (j != pres_job) {  // uniform across the consumers
      consumer_sync();
      if (pres_job >= 0) flush(b.job[pres_job]);
      pres_job = j;
      consumer_sync();
    }
    const uint64_t t0 = static_cast<uint64_t>(tile) * kTileWords;
    const uint32_t len = tile_len(J.n, t0);
    if (len == kTileWords) {
#pragma unroll
      for (int s = 0; s < kStepsPerWarp; ++s) {
        const uint16_t* w = sin + (warp * kStepsPerWarp + s) * kStepWords + 8 * lane;
        const uint4 v0 = *reinterpret_cast<const uint4*>(w);
        const uint4 v1 = *reinterpret_cast<const uint4*>(w + 256);
        const uint32_t x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t y = x[q] ^ ((x[q] >> 5) & 0x04040404u);  // presence_index of each byte
          slo[y & 0xFFu] = 1;
          shi[(y >> 8) & 0xFFu] = 1;
          slo[(y >> 16) & 0xFFu] = 1;
          shi[y >> 24] = 1;
        }
      }
    } else {
#pragma unroll
      for (int s = 0; s < kStepsPerWarp; ++s) {
        const uint32_t w0 = (warp * kStepsPerWarp + s) * kStepWords + lane * kUnitWords;
        if (w0 >= len) continue;
        const uint32_t valid = min(len - w0, static_cast<uint32_t>(kUnitWords));
        for (uint32_t i = 0; i < valid; ++i) {
          const uint32_t w = sin[w0 + i];
          shi[presence_index(w >> 8)] = 1;
          slo[presence_index(w & 0xFFu)] = 1;
        }
      }
    }
  });
  if (warp == kProducerWarp) return;
  consumer_sync();
  if (pres_job >= 0) flush(b.job[pres_job]);
}

__device__ __forceinline__ uint32_t bitlen_u32(uint32_t v) { return 32u - static_cast<uint32_t>(__clz(v)); }
__device__ __forceinline__ uint64_t code_bytes(uint64_t n, uint32_t w) { return (n * w + 7) / 8; }

// Distinct values of the 16 nibbles that a 256-bit byte bitmap holds:
// bit v of `high` if some byte has high nibble v, of `low` for low nibble v.
__device__ __forceinline__ void nibble_sets(const uint32_t (&bm)[8], uint32_t& high, uint32_t& low) {
  high = 0;
  low = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t a = bm[k] & 0xFFFFu, c = bm[k] >> 16;
    high |= (a ? 1u : 0u) << (2 * k);
    high |= (c ? 1u : 0u) << (2 * k + 1);
    low |= a | c;
  }
}

// One warp per job: the form, the header, the plan.
template <int kMax>
__global__ void __launch_bounds__(32) TorchopDecideKernel(const __grid_constant__ EncBatch<kMax> b) {
  if (blockIdx.x >= b.jobs) return;
  const EncJob& J = b.job[blockIdx.x];
  TorchopPlan* plan = plan_of(J);
  const int lane = threadIdx.x;
  const uint32_t mh = lane < 8 ? plan->hi[lane] : 0u, ml = lane < 8 ? plan->lo[lane] : 0u;
  uint32_t hi[8], lo[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    hi[k] = __shfl_sync(kFull, mh, k);
    lo[k] = __shfl_sync(kFull, ml, k);
  }
  const uint64_t n = J.n, raw = 2 * n;
  uint8_t* dst = J.dst;
  // mode 2: the magnitudes (h & 0x7F) present, from both signs
  uint32_t mag[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) mag[k] = hi[k] | hi[k + 4];
  int lowest = -1, highest = -1;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (lowest < 0 && mag[k]) lowest = 32 * k + __ffs(mag[k]) - 1;
    if (mag[k]) highest = 32 * k + 31 - __clz(mag[k]);
  }
  uint32_t mode = 6, width = 0, mag_min = 0, nib_width = 0;
  uint64_t bytes = 1 + raw;
  {
    const uint32_t span = static_cast<uint32_t>(highest - lowest);
    const uint32_t w = max(1u, bitlen_u32(span));
    const uint64_t size = 3 + n + (n + 7) / 8 + code_bytes(n, w);
    if (w < 7 && size < raw) {
      mode = 2;
      width = w;
      mag_min = static_cast<uint32_t>(lowest);
      bytes = size;
    }
  }
  uint32_t distinct = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) distinct += __popc(hi[k]);
  if (mode == 6) {
    const uint32_t w = max(1u, bitlen_u32(distinct - 1));
    const uint64_t size = 258 + n + code_bytes(n, w);
    if (w < 8 && size < raw) {
      mode = 0;
      width = w;
      bytes = size;
    }
  }
  uint32_t sets[4] = {0, 0, 0, 0};  // nibbles 0-3 (bits 0-3, 4-7, 8-11, 12-15)
  nibble_sets(lo, sets[1], sets[0]);
  nibble_sets(hi, sets[3], sets[2]);
  if (mode == 6) {
    uint64_t size = 69;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t d = __popc(sets[p]);
      const uint32_t w = d <= 2 ? 1u : d <= 4 ? 2u : 4u;
      nib_width |= w << (8 * p);
      size += code_bytes(n, w);
    }
    if (size < raw) {
      mode = 1;
      bytes = size;
    }
  }
  // header and codes
  if (mode == 2) {
    if (lane == 0) {
      dst[0] = 2;
      dst[1] = static_cast<uint8_t>(width);
      dst[2] = static_cast<uint8_t>(mag_min);
    }
  } else if (mode == 0) {
    uint32_t below = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t h = 32 * k + lane;
      const bool present = (hi[k] >> lane) & 1u;
      const uint32_t r = below + __popc(hi[k] & ((1u << lane) - 1u));
      plan->rank[h] = static_cast<uint8_t>(r);
      if (present) dst[2 + r] = static_cast<uint8_t>(h);
      below += __popc(hi[k]);
    }
    for (uint32_t i = lane; i < 256; i += 32)
      if (i >= distinct) dst[2 + i] = 0;
    if (lane == 0) {
      dst[0] = 0;
      dst[1] = static_cast<uint8_t>(width);
    }
  } else if (mode == 1) {
    if (lane < 16) {
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint32_t r = __popc(sets[p] & ((1u << lane) - 1u));
        plan->nib_rank[16 * p + lane] = static_cast<uint8_t>(r);
        dst[5 + 16 * p + lane] = 0;
      }
    }
    __syncwarp();
    if (lane < 16) {
#pragma unroll
      for (int p = 0; p < 4; ++p)
        if ((sets[p] >> lane) & 1u) dst[5 + 16 * p + __popc(sets[p] & ((1u << lane) - 1u))] = static_cast<uint8_t>(lane);
    }
    if (lane == 0) {
      dst[0] = 1;
#pragma unroll
      for (int p = 0; p < 4; ++p) dst[1 + p] = static_cast<uint8_t>((nib_width >> (8 * p)) & 0xFFu);
    }
  } else if (lane == 0) {
    dst[0] = 6;
  }
  if (lane == 0) {
    plan->mode = mode;
    plan->width = width;
    plan->mag_min = mag_min;
    plan->nib_width = nib_width;
    plan->bytes = bytes;
  }
}

// 16 fields of W bits packed LSB first into (lo, hi), W a constant.
template <int W>
__device__ __forceinline__ void pack16w(const uint32_t (&c)[16], uint64_t& lo, uint64_t& hi) {
  lo = 0;
  hi = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    constexpr int kW = W;
    const int bit = i * kW;
    const uint64_t v = c[i];
    if (bit < 64) {
      lo |= v << bit;
      if (bit + kW > 64) hi |= v >> (64 - bit);
    } else {
      hi |= v << (bit - 64);
    }
  }
}

// A warp's run of a code plane: lane L packs the 16 fields of the warp's
// unit L (2W bytes) and the warp stores them at g + 2W L as one contiguous
// run, with aligned stores of the widest slot 2W allows (bytes at or past
// g + valid are not written).
template <int W>
__device__ __forceinline__ void put_plane_w(uint8_t* g, uint32_t valid, const uint32_t (&c)[16], int lane) {
  uint64_t lo, hi;
  pack16w<W>(c, lo, hi);
  using Slot = typename std::conditional<(2 * W) % 8 == 0, uint64_t,
                                         typename std::conditional<(2 * W) % 4 == 0, uint32_t, uint16_t>::type>::type;
  constexpr int S = sizeof(Slot);
  constexpr int K = 2 * W / S;
  Slot d[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int bit = 8 * S * k;
    d[k] = static_cast<Slot>(bit < 64 ? lo >> bit : hi >> (bit - 64));
  }
  warp_store<Slot, K>(g, valid, d, lane);
}

__device__ __forceinline__ void put_plane(uint32_t w, uint8_t* g, uint32_t valid, const uint32_t (&c)[16], int lane) {
  switch (w) {  // uniform across the warp (a job's width)
    case 1: put_plane_w<1>(g, valid, c, lane); break;
    case 2: put_plane_w<2>(g, valid, c, lane); break;
    case 3: put_plane_w<3>(g, valid, c, lane); break;
    case 4: put_plane_w<4>(g, valid, c, lane); break;
    case 5: put_plane_w<5>(g, valid, c, lane); break;
    case 6: put_plane_w<6>(g, valid, c, lane); break;
    case 7: put_plane_w<7>(g, valid, c, lane); break;
    case 8: put_plane_w<8>(g, valid, c, lane); break;
    default: break;  // a width of 0 has no plane bytes
  }
}

// Bytes of a plane of `plane_bytes` that a warp's run starting `at` bytes in
// may write (the run is at most 32 units long).
__device__ __forceinline__ uint32_t run_valid(uint64_t plane_bytes, uint64_t at, uint32_t run) {
  return at >= plane_bytes ? 0u : static_cast<uint32_t>(min(plane_bytes - at, static_cast<uint64_t>(run)));
}

// One thread per 16-word unit of every job, by the job's plan.  A job's
// units are padded to whole warps (the host's unit_start), so a warp's 32
// consecutive units belong to one job, and each plane's bytes of those units
// are one contiguous run, stored by the warp together (warp_store: aligned
// slots, shuffles for the bytes between lanes) instead of byte by byte.
template <int kMax>
__global__ void __launch_bounds__(256) TorchopEncodeKernel(const __grid_constant__ TorchopBatch<kMax> b) {
  // each warp's copy of its job's code tables (the plan's rank, then nib_rank)
  __shared__ __align__(16) uint8_t stab[kThreads / 32][320];
  grid_dependency_sync();
  const uint64_t total = b.unit_start[b.jobs];  // a multiple of 32
  const int lane = threadIdx.x & 31;
  uint8_t* tab = stab[threadIdx.x >> 5];
  int j = 0, tab_job = -1;
  for (uint64_t u = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total;
       u += static_cast<uint64_t>(gridDim.x) * blockDim.x) {  // whole warps: the loop is uniform
    while (u >= b.unit_start[j + 1]) ++j;  // a thread's units increase; uniform across the warp
    const EncJob& J = b.job[j];
    const TorchopPlan* plan = plan_of(J);
    if (j != tab_job) {
      __syncwarp();  // the lanes are done with the previous job's tables
      const uint32_t* from = reinterpret_cast<const uint32_t*>(plan->rank);
      for (int i = lane; i < 80; i += 32) reinterpret_cast<uint32_t*>(tab)[i] = from[i];
      __syncwarp();
      tab_job = j;
    }
    const uint64_t n = J.n, unit = u - b.unit_start[j], g = kUnitWords * unit;
    const uint64_t unit0 = unit - static_cast<uint64_t>(lane);  // the warp's first unit
    const uint32_t valid = g < n ? static_cast<uint32_t>(min(n - g, static_cast<uint64_t>(kUnitWords))) : 0u;
    uint32_t w16[kUnitWords];
    if (b.vec[j] && valid == kUnitWords) {
      const uint4* p = reinterpret_cast<const uint4*>(J.src + layout_addr(J.L, g));
      const uint4 a = __ldg(p), c = __ldg(p + 1);
      const uint32_t x[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        w16[2 * i] = x[i] & 0xFFFFu;
        w16[2 * i + 1] = x[i] >> 16;
      }
    } else {
#pragma unroll
      for (int i = 0; i < kUnitWords; ++i)
        w16[i] = static_cast<uint32_t>(i) < valid ? __ldg(J.src + layout_addr(J.L, g + i)) : 0u;
    }
    const uint32_t mode = __ldg(&plan->mode);
    uint8_t* s = J.dst;
    if (mode == 6) {  // the words as they are
      uint32_t x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = w16[2 * i] | (w16[2 * i + 1] << 16);
      warp_store<uint32_t, 8>(s + 1 + 32 * unit0, run_valid(2 * n, 32 * unit0, 32 * 32), x, lane);
      continue;
    }
    if (mode == 2 || mode == 0) {  // the low bytes
      uint32_t lw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        lw[q] = (w16[4 * q] & 0xFFu) | ((w16[4 * q + 1] & 0xFFu) << 8) | ((w16[4 * q + 2] & 0xFFu) << 16) |
                (w16[4 * q + 3] << 24);
      warp_store<uint32_t, 4>(s + (mode == 2 ? 3 : 258) + 16 * unit0, run_valid(n, 16 * unit0, 32 * 16), lw,
                              lane);
    }
    uint32_t c[16];
    if (mode == 2) {
      const uint32_t w = __ldg(&plan->width), m0 = __ldg(&plan->mag_min);
      const uint64_t sign_bytes = (n + 7) / 8;
#pragma unroll
      for (int i = 0; i < 16; ++i) c[i] = static_cast<uint32_t>(i) < valid ? (w16[i] >> 15) : 0u;
      put_plane_w<1>(s + 3 + n + 2 * unit0, run_valid(sign_bytes, 2 * unit0, 32 * 2), c, lane);
#pragma unroll
      for (int i = 0; i < 16; ++i) c[i] = static_cast<uint32_t>(i) < valid ? ((w16[i] >> 8) & 0x7Fu) - m0 : 0u;
      put_plane(w, s + 3 + n + sign_bytes + 2 * w * unit0, run_valid(code_bytes(n, w), 2 * w * unit0, 64 * w), c,
                lane);
    } else if (mode == 0) {
      const uint32_t w = __ldg(&plan->width);
#pragma unroll
      for (int i = 0; i < 16; ++i) c[i] = static_cast<uint32_t>(i) < valid ? tab[w16[i] >> 8] : 0u;
      put_plane(w, s + 258 + n + 2 * w * unit0, run_valid(code_bytes(n, w), 2 * w * unit0, 64 * w), c, lane);
    } else {  // mode 1
      const uint32_t widths = __ldg(&plan->nib_width);
      uint8_t* plane = s + 69;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w = (widths >> (8 * q)) & 0xFFu;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          c[i] = static_cast<uint32_t>(i) < valid ? tab[256 + 16 * q + ((w16[i] >> (4 * q)) & 0xFu)] : 0u;
        put_plane(w, plane + 2 * w * unit0, run_valid(code_bytes(n, w), 2 * w * unit0, 64 * w), c, lane);
        plane += code_bytes(n, w);
      }
    }
  }
}

}  // namespace ukv
